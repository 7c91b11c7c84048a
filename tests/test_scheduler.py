"""Batched continuous-batching scheduler, host logic on CPU (the GPU test is tests/test_gpu_scheduler.py).

A stand-in backend keeps the B200 backend's allocation behaviour (``prefill`` allocates each prompt's
blocks, sharing the whole-block common prefix of a batch once; ``decode`` appends one token per table)
and a deterministic "model": the next token is a function of the last token and its position, so each
request's stream is known without running anything. Checked: the scheduler's streams equal the
per-request streams, decode steps are batched, admission follows priority and the KV block budget,
EOS and max_new_tokens end requests, every block goes back to the allocator, and blocks shared by every
running table are handed to the attention kernel as the shared prefix.
"""

import pytest
import torch

from microgen_b200.backends.b200 import PagedKVCache
from microgen_b200.runtime.paged_kv import PagedKVCacheAllocator
from microgen_b200.scheduler import BatchedScheduler, Request, RequestStatus

V = 97


def next_token(tok: int, pos: int) -> int:
    return (tok * 31 + pos * 7 + 3) % V


def stream(prompt, n):
    out, t, p = [], prompt[-1], len(prompt) - 1
    for _ in range(n):
        t = next_token(t, p)
        out.append(t)
        p += 1
    return out


class _Eng:
    def __init__(self, max_batch, max_blocks):
        self.max_batch, self.max_blocks = max_batch, max_blocks


class FakeBackend:
    def __init__(self, num_blocks=64, max_batch=8, max_blocks=32):
        self.allocator = PagedKVCacheAllocator(num_blocks=num_blocks)
        self.engine = _Eng(max_batch, max_blocks)
        self.calls = []          # ("prefill"|"decode", batch size, n_shared)

    def _need_model(self):
        return self.engine

    def _logits(self, toks, positions):
        lg = torch.zeros((len(toks), V))
        for i, (t, p) in enumerate(zip(toks, positions)):
            lg[i, next_token(t, p)] = 1.0
        return lg

    def prefill(self, input_ids):
        ids = input_ids.tolist()
        b, T = len(ids), len(ids[0])
        cache = PagedKVCache(self.allocator)
        lcp = T
        for row in ids[1:]:
            lcp = min(lcp, next((i for i, (a, c) in enumerate(zip(ids[0], row)) if a != c), T))
        n_prefix = min(lcp, T - 1) // 16 if b > 1 else 0
        if n_prefix:
            cache.prefix = self.allocator.allocate_sequence("prefix", n_prefix * 16)
            cache.tables = [self.allocator.share_prefix(cache.prefix, n_prefix, f"seq{i}", T) for i in range(b)]
        else:
            cache.tables = [self.allocator.allocate_sequence(f"seq{i}", T) for i in range(b)]
        cache.n_shared_blocks = n_prefix
        self.calls.append(("prefill", b, n_prefix))
        return self._logits([r[-1] for r in ids], [T - 1] * b), cache

    def decode(self, token_ids, cache=None):
        toks = token_ids[:, -1].tolist()
        assert len(toks) == len(cache.tables)
        pos = []
        for t in cache.tables:
            pos.append(t.num_tokens)
            self.allocator.append_token(t)
        lead = [t.block_ids()[:cache.n_shared_blocks] for t in cache.tables]
        assert all(x == lead[0] for x in lead)  # the kernel's shared-prefix contract
        self.calls.append(("decode", len(toks), cache.n_shared_blocks))
        return self._logits(toks, pos), cache

    def sample(self, logits, temperature=1.0, top_k=0, top_p=0.0):
        return logits.argmax(-1)[:, None]


def _req(i, prompt, n, **kw):
    return Request(request_id=f"r{i}", prompt="", prompt_ids=list(prompt), max_new_tokens=n, **kw)


def test_streams_match_and_decode_is_batched():
    be = FakeBackend(num_blocks=256)
    sch = BatchedScheduler(be, max_batch_size=4)
    reqs = [_req(i, [(i * 13 + j) % V for j in range(5 + 7 * i)], 6 + 3 * i) for i in range(7)]
    for r in reqs:
        sch.add_request(r)
    done = sch.run_until_complete()
    assert sorted(r.request_id for r in done) == sorted(r.request_id for r in reqs)
    for r in reqs:
        assert r.status == RequestStatus.COMPLETED
        assert r.generated_token_ids == stream(r.prompt_ids, r.max_new_tokens), r.request_id
    assert max(sch.decode_batch_sizes) == 4
    assert be.allocator.get_num_free_blocks() == 256
    assert sch.get_profile_breakdown()["total_steps"] == sch.profiling_stats["total_steps"] > 0


def test_priority_order_and_eos():
    be = FakeBackend(num_blocks=256)
    prompt = [5, 6, 7]
    eos = stream(prompt, 4)[2]  # the third generated token of this prompt
    sch = BatchedScheduler(be, max_batch_size=1, eos_token_id=eos)
    low = _req(0, [1, 2], 3, priority=0)
    high = _req(1, prompt, 50, priority=5)
    sch.add_request(low)
    sch.add_request(high)
    first = sch.step()
    assert high.status == RequestStatus.RUNNING and low.status == RequestStatus.PENDING
    assert not first
    sch.run_until_complete()
    assert high.generated_token_ids == stream(prompt, 3)  # stopped at EOS
    assert low.generated_token_ids == stream([1, 2], 3)
    assert low.start_time >= high.finish_time


def test_admission_waits_for_kv_blocks():
    # each request needs ceil((20 + 28) / 16) = 3 blocks; 7 blocks admit two at a time
    be = FakeBackend(num_blocks=7)
    sch = BatchedScheduler(be, max_batch_size=4)
    reqs = [_req(i, [(3 * i + j) % V for j in range(20)], 28) for i in range(5)]
    for r in reqs:
        sch.add_request(r)
    sch.run_until_complete()
    assert max(sch.decode_batch_sizes) == 2
    for r in reqs:
        assert r.generated_token_ids == stream(r.prompt_ids, 28)
    assert be.allocator.get_num_free_blocks() == 7


def test_shared_prefix_blocks_reach_the_kernel():
    be = FakeBackend(num_blocks=64)
    sch = BatchedScheduler(be, max_batch_size=4)
    shared = [(7 * j) % V for j in range(40)]  # 2 whole blocks shared, prompts of equal length
    reqs = [_req(i, shared + [i, i + 1], 10) for i in range(3)]
    for r in reqs:
        sch.add_request(r)
    sch.run_until_complete()
    dec = [c for c in be.calls if c[0] == "decode"]
    assert be.calls[0] == ("prefill", 3, 2)
    assert all(n == 2 for _, b, n in dec if b == 3)
    for r in reqs:
        assert r.generated_token_ids == stream(r.prompt_ids, 10)
    assert be.allocator.get_num_free_blocks() == 64


def test_rejects_requests_that_cannot_fit():
    be = FakeBackend(num_blocks=4, max_blocks=32)
    sch = BatchedScheduler(be, max_batch_size=2)
    with pytest.raises(ValueError):
        sch.add_request(_req(0, [1] * 60, 10))   # 5 blocks > 4
    with pytest.raises(ValueError):
        sch.add_request(_req(1, [], 3))
    with pytest.raises(ValueError):
        BatchedScheduler(be, max_batch_size=9)


def test_cancelled_requests_are_skipped():
    be = FakeBackend()
    sch = BatchedScheduler(be, max_batch_size=2)
    a, b = _req(0, [1, 2, 3], 4), _req(1, [4, 5], 4)
    sch.add_request(a)
    sch.add_request(b)
    a.status = RequestStatus.CANCELLED
    sch.run_until_complete()
    assert a.generated_token_ids == [] and b.generated_token_ids == stream([4, 5], 4)

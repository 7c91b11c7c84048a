"""Chunked prefill (``DecodeEngine.prefill``: many prompt positions per pass, every linear on all those
tokens in one tcgen05 launch, causal attention per prompt on the paged kernel) against the position-at-a-time
prefill through the decode step, on the same seeded models and allocator order: the logits after the
prompt, the K/V written to the pool, and teacher-forced decode logits afterwards agree within the bf16
tolerance (the two paths group the same arithmetic into different launches: split-K and attention split
plans differ, so sums may differ in their last bits). Covers batches with a shared prompt prefix,
prompts continued through a returned cache, chunk sizes that do and do not divide the prompt, and the
three families."""

import numpy as np
import pytest
import torch

from tests._hf_models import TINY, make_hf_model, prompt_ids

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2e-2


def _close(got, want, what):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance, max err {err.max():.3e}"


def _backend(model, chunk):
    from microgen_b200.backends import B200QuantizedBackend
    be = B200QuantizedBackend(max_batch=4, max_seq_len=160, free_list_seed=5, prefill_chunk=chunk)
    be.load_model("tiny", model_instance=model)
    return be


def _prompts(V, shared_len, tail, b):
    shared = prompt_ids(V, shared_len, seed=3)
    return [shared + prompt_ids(V, tail, seed=30 + i) for i in range(b)]


def _pool_rows(be, cache):
    """K and V of every written position of every sequence, per layer: [layers, 2, tokens, hkv, d]."""
    eng = be.engine
    out = []
    for l in range(len(eng.w.layers)):
        ks, vs = [], []
        for t in cache.tables:
            for p in range(t.num_tokens):
                blk = t.physical_blocks[p // 16].block_id
                ks.append(eng.pool.k[l][blk, :, p % 16].float())
                vs.append(eng.pool.v[l][blk, :, p % 16].float())
        out.append(torch.stack([torch.stack(ks), torch.stack(vs)]))
    return torch.stack(out).cpu().numpy()


@pytest.mark.parametrize("family", ["llama", "qwen2", "gpt2"])
@pytest.mark.parametrize("chunk", [1, 7, 64])
def test_chunked_prefill_matches_stepwise(family, chunk):
    shape = TINY[family]
    model, _ = make_hf_model(shape, seed=0)
    prompts = _prompts(shape["vocab"], 37, 14, 4)  # 2 shared whole blocks, 51 tokens each
    ref, new = _backend(model, 0), _backend(model, chunk)
    lg0, c0 = ref.prefill(torch.tensor(prompts))
    lg1, c1 = new.prefill(torch.tensor(prompts))
    assert [t.block_ids() for t in c0.tables] == [t.block_ids() for t in c1.tables]
    assert c0.n_shared_blocks == c1.n_shared_blocks == 2
    _close(lg1.cpu().numpy(), lg0.cpu().numpy(), "prompt logits")
    _close(_pool_rows(new, c1), _pool_rows(ref, c0), "K/V pool")
    tok = ref.sample(lg0)
    for step in range(6):
        lg0, c0 = ref.decode(tok, cache=c0)
        lg1, c1 = new.decode(tok, cache=c1)
        _close(lg1.cpu().numpy(), lg0.cpu().numpy(), f"decode step {step}")
        tok = ref.sample(lg0)


@pytest.mark.parametrize("chunk", [16, 64])
def test_chunked_prefill_continues_a_cache(chunk):
    """A prompt prefilled in two calls (the second through the returned cache) equals one stepwise call."""
    shape = TINY["llama"]
    model, _ = make_hf_model(shape, seed=1)
    prompts = _prompts(shape["vocab"], 0, 70, 2)
    ref, new = _backend(model, 0), _backend(model, chunk)
    lg0, c0 = ref.prefill(torch.tensor(prompts))
    _, c1 = new.prefill(torch.tensor([p[:23] for p in prompts]))
    lg1, c1 = new.prefill(torch.tensor([p[23:] for p in prompts]), cache=c1)
    _close(lg1.cpu().numpy(), lg0.cpu().numpy(), "prompt logits")
    _close(_pool_rows(new, c1), _pool_rows(ref, c0), "K/V pool")


def test_chunked_prefill_single_prompt_and_greedy_token():
    """Batch 1, a prompt longer than one chunk: logits and the device greedy token of the last position."""
    shape = TINY["qwen2"]
    model, _ = make_hf_model(shape, seed=2)
    prompt = [prompt_ids(shape["vocab"], 100, seed=9)]
    ref, new = _backend(model, 0), _backend(model, 32)
    lg0, _ = ref.prefill(torch.tensor(prompt))
    lg1, _ = new.prefill(torch.tensor(prompt))
    _close(lg1.cpu().numpy(), lg0.cpu().numpy(), "prompt logits")
    assert new.sample(lg1).item() == int(np.argmax(lg1.cpu().numpy()[0]))


@pytest.mark.parametrize("chunk", [0, 64])
def test_prefix_cache_reuses_blocks_across_prefills(chunk):
    """``prefix_cache_capacity``: a prefill caches its prompt's whole leading blocks; a later prefill whose
    prompt starts with them shares those blocks (no recompute) and gives the logits and decode steps of a
    backend without the cache. The first request's cache is freed before the later prefills and other
    blocks are allocated in between, so the shared blocks survive only through the prefix cache's own
    references."""
    shape = TINY["llama"]
    model, _ = make_hf_model(shape, seed=4)
    V = shape["vocab"]
    from microgen_b200.backends import B200QuantizedBackend
    be = B200QuantizedBackend(max_batch=4, max_seq_len=160, free_list_seed=5, prefill_chunk=chunk,
                              prefix_cache_capacity=8)
    be.load_model("tiny", model_instance=model)
    ref = _backend(model, chunk)
    s = prompt_ids(V, 48, seed=11)                          # three whole blocks
    _, c1 = be.prefill(torch.tensor([s + prompt_ids(V, 5, seed=12)]))
    cached = c1.tables[0].block_ids()[:3]
    c1.free()
    _, other = be.prefill(torch.tensor([prompt_ids(V, 70, seed=13)] * 2))  # takes the freed private blocks
    for prompts in ([s + prompt_ids(V, 20, seed=14)], [s + prompt_ids(V, 12, seed=15), s + prompt_ids(V, 12, seed=16)]):
        lg1, c2 = be.prefill(torch.tensor(prompts))
        lg0, c0 = ref.prefill(torch.tensor(prompts))
        assert c2.reused_prefix_tokens == 48
        assert all(t.block_ids()[:3] == cached for t in c2.tables)
        _close(lg1.cpu().numpy(), lg0.cpu().numpy(), "prompt logits")
        tok = ref.sample(lg0)
        for step in range(4):
            lg0, c0 = ref.decode(tok, cache=c0)
            lg1, c2 = be.decode(tok, cache=c2)
            _close(lg1.cpu().numpy(), lg0.cpu().numpy(), f"decode step {step}")
            tok = ref.sample(lg0)
        c0.free()
        c2.free()
    other.free()

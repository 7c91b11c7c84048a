"""Batched continuous-batching scheduler on the GPU: requests of different lengths, priorities and shared
prompt prefixes decode together through ``BatchedScheduler`` on the B200 backend (one graph-replayed
decode step per scheduler step for all running requests, ragged contexts). Each request's greedy stream
is then replayed alone at batch 1, teacher-forced with the scheduler's tokens: the logits must give the
same argmax wherever the top-1 / top-2 margin is clear of the bf16 tolerance (batch composition changes
the attention split plan, so only near-ties may flip)."""

import numpy as np
import pytest
import torch

from tests._hf_models import TINY, make_hf_model, prompt_ids

pytestmark = pytest.mark.gpu


def _replay(be, prompt, tokens):
    """Logits of each position of ``tokens`` when fed one by one after ``prompt`` (batch 1)."""
    logits, cache = be.prefill(torch.tensor([prompt]))
    out = [logits.float().cpu().numpy()[0]]
    for t in tokens[:-1]:
        logits, cache = be.decode(torch.tensor([[t]], device="cuda"), cache=cache)
        out.append(logits.float().cpu().numpy()[0])
    cache.free()
    return np.stack(out)


@pytest.mark.parametrize("family", ["llama", "gpt2"])
def test_scheduler_streams_match_batch1(family):
    from microgen_b200.backends import B200QuantizedBackend
    from microgen_b200.scheduler import BatchedScheduler, Request, RequestStatus
    shape = TINY[family]
    model, _ = make_hf_model(shape, seed=0)
    be = B200QuantizedBackend(max_batch=4, max_seq_len=128, free_list_seed=3)
    be.load_model("tiny", model_instance=model)
    V = shape["vocab"]
    shared = prompt_ids(V, 32, seed=11)
    prompts = [shared + prompt_ids(V, 5, seed=40 + i) for i in range(3)]       # equal length, 2 shared blocks
    prompts += [prompt_ids(V, n, seed=60 + n) for n in (3, 17, 29, 9)]
    reqs = [Request(request_id=f"r{i}", prompt="", prompt_ids=p, max_new_tokens=6 + (5 * i) % 17,
                    priority=i % 3, temperature=0.0) for i, p in enumerate(prompts)]
    sampled = Request(request_id="s", prompt="", prompt_ids=prompt_ids(V, 12, seed=99), max_new_tokens=10,
                      temperature=0.8, top_k=5)
    sch = BatchedScheduler(be, max_batch_size=4)
    for r in reqs + [sampled]:
        sch.add_request(r)
    free0 = be.allocator.get_num_free_blocks()
    done = sch.run_until_complete()
    assert len(done) == len(reqs) + 1
    assert be.allocator.get_num_free_blocks() == free0
    assert max(sch.decode_batch_sizes) == 4
    assert len(sampled.generated_token_ids) == 10 and all(0 <= t < V for t in sampled.generated_token_ids)
    clear_steps = agree = 0
    for r in reqs:
        assert r.status == RequestStatus.COMPLETED and len(r.generated_token_ids) == r.max_new_tokens
        lg = _replay(be, r.prompt_ids, r.generated_token_ids)
        tol = 1e-2 + 2e-2 * np.abs(lg)
        top2 = np.sort(lg, axis=-1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * tol.max(axis=-1)
        got = np.array(r.generated_token_ids)
        assert (np.argmax(lg, axis=-1) == got)[clear].all(), r.request_id
        clear_steps += clear.sum()
        agree += (np.argmax(lg, axis=-1) == got).sum()
    assert clear_steps > 0.3 * sum(r.max_new_tokens for r in reqs)
    assert be.allocator.get_num_free_blocks() == free0

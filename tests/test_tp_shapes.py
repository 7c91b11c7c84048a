"""Per-rank shapes of the Llama-3.2-3B-shaped workload at TP = 1, 2, 4 and 8 (one layer at the real width,
a small vocabulary), as ``WeightLoader`` produces them on the CPU: head-aligned column shards, input-split
row shards, 64-row gate/up groups, the vocab split, and the constraints the kernels put on them (K a
multiple of 16 for every linear, SwiGLU gate/up rows a multiple of 128, the fused reduce's row width, the
attention kernel's GQA group). The bench's scaling run uses these shapes on every rank."""

import pytest
import torch

from microgen_b200 import model_spec as MS
from microgen_b200.engine import WeightLoader, vocab_bounds
from microgen_b200.synthetic import SyntheticState


def _fast_quant(w):
    s = (w.abs().amax(dim=1) / 127.0).clamp_min(1e-8)
    return torch.round(w / s[:, None]).clamp(-128, 127).to(torch.int8), s


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_llama3b_rank_shapes_meet_kernel_constraints(world):
    spec = MS.ModelSpec(**dict(MS.LLAMA_3B, layers=1, vocab=1003))
    state = SyntheticState(spec, seed=0, device="cpu")
    D, H, I = spec.head_dim, spec.hidden, spec.inter
    hq, hkv = spec.heads // world, spec.kv_heads // world
    assert hq * world == spec.heads and hkv * world == spec.kv_heads and hq // hkv <= 16
    lm_rows = 0
    for rank in range(world):
        w = WeightLoader(spec, "cpu", rank, world, pack=False, quantize=_fast_quant,
                         vocab_parallel=world > 1).load(state)
        L = w.layers[0]
        assert tuple(L.qkv_q.shape) == ((hq + 2 * hkv) * D, H) and L.qkv_s.shape[0] == (hq + 2 * hkv) * D
        assert tuple(L.o_q.shape) == (H, hq * D) and L.o_s.shape[0] == H
        assert tuple(L.gu_q.shape) == (2 * I // world, H) and L.gu_q.shape[0] % 128 == 0
        assert tuple(L.d_q.shape) == (H, I // world) and L.d_s.shape[0] == H
        for q in (L.qkv_q, L.o_q, L.gu_q, L.d_q, w.lm_q):
            assert q.shape[1] % 16 == 0 and q.dtype == torch.int8
        a, e = vocab_bounds(spec.vocab, world)[rank] if world > 1 else (0, spec.vocab)
        assert w.lm_q.shape[0] == e - a and w.lm_offset == a
        lm_rows += w.lm_q.shape[0]
    assert lm_rows == spec.vocab
    assert H % 4 == 0 and H <= 4 * 1024 * 2  # the fused reduce: one float4 per thread, at most 1024 x 2 per row

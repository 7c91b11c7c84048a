"""Paged INT8 KV (the paged form of ``KVCacheState(quantize_kv=True)``, ``microgen/runtime/kv_cache.py:30-40,
114-120``) on the GPU.

* ``mg_rope_kv_append_kv8``: codes and scales bit-exact against the oracle quantizer (itself pinned to the
  reference's ``_quantize_tensor``), on the reference's own edge vectors and on seeded vectors; with RoPE, the
  rotated K vectors quantized to within one code of the oracle (the rotation's fp32 rounding may differ);
* ``mg_paged_decode_attn_kv8``: against SDPA over the reference's stored INT8 cache, and against the float64
  oracle over dequantized pools — ragged last blocks whose unused slots hold NaN scales, GQA groups 1..16,
  head_dim 32/64/128, shared prefixes, splits;
* the backend with ``quantize_kv=True``: prefill + decode of a tiny Llama against the reference's greedy
  stream decoded with an INT8 cache (logits within the contract's tolerance plus the INT8 difference of the
  step's own token, which the reference attends to before quantizing it; tokens equal wherever the
  reference's top-1 margin is clear of that tolerance).
"""

import os

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.model import rope_cos_sin

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATOL, RTOL = 1e-2, 2e-2


def K():
    from microgen_b200 import kernels
    return kernels


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def close(got, want, rtol=RTOL, atol=ATOL):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance, max err {err.max():.3e}"


def _append(qkv, pos, table, slots, hq, hkv, d, nblk):
    kp = torch.zeros((nblk, hkv, 16, d), dtype=torch.int8, device="cuda")
    vp = torch.zeros_like(kp)
    ks = torch.zeros((nblk, hkv, 16), dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    qo = K().rope_kv_append(dev(qkv), None if pos is None else dev(pos), None if table is None else dev(table),
                            dev(slots), hq, hkv, d, kp, vp, k_scales=ks, v_scales=vs)
    return qo.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), ks.cpu().numpy(), vs.cpu().numpy()


def test_kv8_append_matches_reference_quantizer():
    """The reference's edge vectors and seeded ones as V (and, without RoPE, K) vectors: bit-exact."""
    d = np.load(os.path.join(G, "kv8_cases.npz"))
    x = d["quant_x"]                       # [64 vectors, 64]
    n, D = x.shape
    hq, hkv = 2, 1
    rng = np.random.default_rng(4)
    qkv = np.zeros((n, (hq + 2 * hkv) * D), np.float32)
    qkv[:, :hq * D] = rng.standard_normal((n, hq * D))
    qkv[:, hq * D:(hq + 1) * D] = x[::-1]  # K: the same vectors in reverse order
    qkv[:, (hq + 1) * D:] = x              # V
    slots = rng.permutation(8 * 16)[:n].astype(np.int32)
    qo, kp, vp, ks, vs = _append(qkv, None, None, slots, hq, hkv, D, 8)
    for i in range(n):
        blk, off = slots[i] // 16, slots[i] % 16
        assert np.array_equal(vp[blk, 0, off], d["quant_q"][i]), i
        assert ks[blk, 0, off].view(np.uint32) == d["quant_s"][n - 1 - i].view(np.uint32)
        assert vs[blk, 0, off].view(np.uint32) == d["quant_s"][i].view(np.uint32)
        assert np.array_equal(kp[blk, 0, off], d["quant_q"][n - 1 - i])
    np.testing.assert_array_equal(qo.reshape(n, -1), qkv[:, :hq * D])


@pytest.mark.parametrize("hq,hkv,d", [(24, 8, 128), (14, 2, 64), (4, 4, 32)])
def test_kv8_append_with_rope(hq, hkv, d):
    rng = np.random.default_rng(hq + d)
    b, theta, max_pos, nblk = 6, 500000.0, 4096, 40
    qkv = (rng.standard_normal((b, (hq + 2 * hkv) * d)) * 2.0).astype(np.float32)
    pos = np.array([0, 1, 17, 1000, 4095, 33], np.int32)
    table = np.stack([np.concatenate([rope_cos_sin(p, d, theta)[0][: d // 2], rope_cos_sin(p, d, theta)[1][: d // 2]])
                      for p in range(max_pos)]).astype(np.float32)
    slots = np.array([3 * 16, 7 * 16 + 5, 39 * 16 + 15, 0, 22 * 16 + 9, 5 * 16 + 1], np.int32)
    qo, kp, vp, ks, vs = _append(qkv, pos, table, slots, hq, hkv, d, nblk)
    diffs = 0
    for i in range(b):
        c, s = rope_cos_sin(int(pos[i]), d, theta)
        heads = qkv[i].reshape(hq + 2 * hkv, d)
        rot = lambda x: (x.astype(np.float64) * c + np.concatenate([-x[d // 2:], x[: d // 2]]) * s).astype(np.float32)
        blk, off = slots[i] // 16, slots[i] % 16
        for hh in range(hkv):
            kq, kss = oatt.quantize_kv_vectors(rot(heads[hq + hh]))
            dk = np.abs(kp[blk, hh, off].astype(np.int32) - kq.astype(np.int32))
            assert dk.max() <= 1
            diffs += int((dk > 0).sum())
            assert abs(ks[blk, hh, off] - kss) <= 1e-6 * kss
            vq, vss = oatt.quantize_kv_vectors(heads[hq + hkv + hh])
            assert np.array_equal(vp[blk, hh, off], vq)
            assert vs[blk, hh, off].view(np.uint32) == vss.view(np.uint32)
    assert diffs <= b * hkv * d // 50  # only rounding-boundary codes may differ


def _kv8_case(b, hq, hkv, d, ctx, n_shared=0, extra_blocks=8, seed=0):
    rng = np.random.default_rng(seed)
    max_blocks = max((c + 15) // 16 for c in ctx)
    need = n_shared + sum((c + 15) // 16 - n_shared for c in ctx)
    nblk = need + extra_blocks
    perm = rng.permutation(nblk).astype(np.int32)
    tables = np.zeros((b, max_blocks), np.int32)
    tables[:, :n_shared] = perm[:n_shared]
    nxt = n_shared
    for i, c in enumerate(ctx):
        nb = (c + 15) // 16
        tables[i, n_shared:nb] = perm[nxt:nxt + nb - n_shared]
        nxt += nb - n_shared
    kq, ks = oatt.quantize_kv_vectors(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32))
    vq, vs = oatt.quantize_kv_vectors(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32))
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    return q, kq, vq, ks, vs, tables, np.array(ctx, np.int32)


def _run_kv8(q, kq, vq, ks, vs, tables, ctx, n_shared):
    d = q.shape[-1]
    out = K().paged_decode_attn(dev(q), dev(kq), dev(vq), dev(tables), dev(ctx), 1.0 / np.sqrt(d),
                                n_shared_blocks=n_shared, k_scales=dev(ks), v_scales=dev(vs))
    return out.float().cpu().numpy().reshape(q.shape)


def test_kv8_attention_vs_reference_fixture():
    d = np.load(os.path.join(G, "kv8_cases.npz"))
    got = _run_kv8(d["attn_q"], d["attn_kpool"], d["attn_vpool"], d["attn_kscale"], d["attn_vscale"],
                   d["attn_tables"], d["attn_ctx"], 0)
    close(got, d["attn_out"])


@pytest.mark.parametrize("b,hq,hkv,d,ctx,n_shared", [
    (1, 32, 8, 128, [1], 0),
    (3, 8, 2, 64, [15, 16, 17], 0),
    (4, 24, 8, 128, [100, 260, 33, 512], 0),
    (2, 14, 2, 64, [1000, 2047], 0),
    (16, 32, 8, 128, [1024 + 37 * i for i in range(16)], 0),
    (5, 24, 8, 128, [64 * 16 + 5 * i + 1 for i in range(5)], 64),
    (8, 32, 8, 128, [9 * 16 + i for i in range(8)], 9),
    (3, 12, 12, 64, [40, 48, 100], 2),
    (2, 16, 1, 128, [300, 17], 1),
    (4, 8, 8, 32, [70, 3, 33, 16], 0),
])
def test_kv8_attention_vs_oracle(b, hq, hkv, d, ctx, n_shared):
    q, kq, vq, ks, vs, tables, ctxa = _kv8_case(b, hq, hkv, d, ctx, n_shared, seed=b * 5 + hq)
    got = _run_kv8(q, kq, vq, ks, vs, tables, ctxa, n_shared)
    want = oatt.paged_decode_attention_kv8(q, kq, vq, ks, vs, tables, ctxa, 1.0 / np.sqrt(d))
    close(got, want)


@pytest.mark.parametrize("n_shared", [0, 2])
def test_kv8_attention_ignores_stale_slots(n_shared):
    """Slots past a sequence's length hold stale codes and NaN scales; they must not reach the output."""
    ctx = [37, 16 * 5 + 1, 200, 16 * 3]
    q, kq, vq, ks, vs, tables, ctxa = _kv8_case(4, 24, 8, 128, ctx, n_shared, seed=11)
    want = oatt.paged_decode_attention_kv8(q, kq, vq, ks, vs, tables, ctxa, 1.0 / np.sqrt(128))
    for i, c in enumerate(ctxa):
        if c % 16:
            last = tables[i, (c - 1) // 16]
            ks[last, :, c % 16:] = np.nan
            vs[last, :, c % 16:] = np.nan
            kq[last, :, c % 16:] = 127
            vq[last, :, c % 16:] = -128
    got = _run_kv8(q, kq, vq, ks, vs, tables, ctxa, n_shared)
    assert np.isfinite(got).all()
    close(got, want)


def test_kv8_shared_prefix_equals_unshared():
    q, kq, vq, ks, vs, tables, ctxa = _kv8_case(6, 24, 8, 128, [640 + 16 * i + 3 for i in range(6)], 40, seed=3)
    a = _run_kv8(q, kq, vq, ks, vs, tables, ctxa, 40)
    b_ = _run_kv8(q, kq, vq, ks, vs, tables, ctxa, 0)
    close(a, b_, rtol=1e-2, atol=5e-3)


@pytest.mark.parametrize("graph", [False, True])
def test_backend_quantize_kv_matches_reference_stream(graph):
    import json
    from microgen_b200.backends import B200QuantizedBackend
    from tests._hf_models import make_hf_model
    d = np.load(os.path.join(G, "kv8_cases.npz"))
    shape = json.loads(str(d["model_shape"]))
    model, _ = make_hf_model(shape, seed=0)
    be = B200QuantizedBackend(max_batch=2, max_seq_len=128, use_cuda_graph=graph, quantize_kv=True)
    be.load_model("tiny", model_instance=model)
    assert be.engine.pool.k.dtype == torch.int8
    ref_tok, ref_lg = d["model_tokens"], d["model_logits"]
    logits, cache = be.prefill(torch.tensor([d["model_prompt"].tolist()]))
    got_lg, got_tok = [], []
    for i in range(len(ref_tok)):
        got_tok.append(int(be.sample(logits)[0, 0]))
        if i < len(ref_lg):
            got_lg.append(logits[0].float().cpu().numpy())
        # teacher-forced with the reference's token, so a near-tie flip cannot derail the comparison
        logits, cache = be.decode(torch.tensor([[int(ref_tok[i])]], device="cuda"), cache=cache)
    close(np.stack(got_lg), ref_lg, rtol=4e-2, atol=4e-2)
    lg = np.stack(got_lg)
    top2 = np.sort(ref_lg, axis=-1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 2 * (4e-2 + 4e-2 * np.abs(ref_lg).max(axis=-1))
    assert (np.array(got_tok[:len(ref_lg)]) == ref_tok[:len(ref_lg)])[clear].all()
    assert np.mean(np.array(got_tok) == ref_tok) > 0.8

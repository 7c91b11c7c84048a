"""Kernel parity on the GPU: every C-ABI kernel against the CPU oracle and the
reference's own fixtures (tests/golden/). Tolerance for bf16-activation outputs
is the contract's: |got - want| <= 1e-2 + 2e-2 * |want| against an fp64
dequantize-then-matmul / SDPA oracle fed the same bf16-rounded inputs."""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import linear as olin
from oracle.model import rope_cos_sin
from oracle.quant import quantize_rows_i8 as oq

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
RTOL, ATOL = 2e-2, 1e-2


def K():
    from microgen_b200 import kernels
    return kernels


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def bf16_np(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def close(got, want, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


# ------------------------------------------------------------------ quantizer (bit-exact)
@pytest.mark.parametrize("case", ["seeded", "edge", "wide", "ragged"])
def test_quantize_matches_reference_fixture(case):
    d = np.load(os.path.join(G, "quant_cases.npz"))
    q, s = K().quantize_rows_i8(dev(d[f"{case}_w"]))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), d[f"{case}_q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), d[f"{case}_s"].astype(np.float32).view(np.uint32))


def test_quantize_full_size_digest():
    meta = json.load(open(os.path.join(G, "quant_digest.json")))
    g = torch.Generator().manual_seed(3)
    w = torch.randn(3072, 3072, generator=g, dtype=torch.float32) * 0.02
    q, s = K().quantize_rows_i8(w.cuda())
    h = hashlib.sha256()
    h.update(q.cpu().numpy().tobytes())
    h.update(s.cpu().numpy().astype(np.float32).tobytes())
    assert h.hexdigest() == meta["codes_scales_sha256"]


@pytest.mark.parametrize("shape", [(1, 16), (7, 48), (300, 4096), (128, 8192)])
def test_quantize_random_vs_oracle(shape):
    rng = np.random.default_rng(shape[0])
    w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w[0, : shape[1] // 2] = 0
    q, s = K().quantize_rows_i8(dev(w))
    qo, so = oq(w)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


# ------------------------------------------------------------------ INT8 linear
def _mk_linear(m, k, n, seed, bias=True):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    q, s = oq(w)
    x = bf16_np(rng.standard_normal((m, k), dtype=np.float32))
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32) if bias else None
    return x, q, s, b


@pytest.mark.parametrize("algo", ["simt", "tc"])
@pytest.mark.parametrize("m,k,n", [(1, 256, 384), (5, 96, 40), (16, 896, 1152), (32, 3072, 1024), (33, 448, 896),
                                   (100, 1024, 640), (256, 512, 256), (300, 256, 136)])
def test_linear_store_bf16_vs_oracle(algo, m, k, n):
    x, q, s, b = _mk_linear(m, k, n, seed=m + k + n)
    y = K().i8_linear(dev(x, torch.bfloat16), dev(q), dev(s), dev(b), algo=algo)
    want = olin.i8_linear(x, q, s, b)
    close(y.float().cpu().numpy(), want)


@pytest.mark.parametrize("split", [1, 2, 3, 4, 5, 8])
def test_linear_tc_split_k_deterministic_and_close(split):
    x, q, s, b = _mk_linear(32, 3072, 768, seed=4)
    y = K().i8_linear(dev(x, torch.bfloat16), dev(q), dev(s), dev(b), epilogue=K().EPI_STORE_F32, algo="tc",
                      split_k=split)
    want = olin.i8_linear(x, q, s, b)
    close(y.cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    y2 = K().i8_linear(dev(x, torch.bfloat16), dev(q), dev(s), dev(b), epilogue=K().EPI_STORE_F32, algo="tc",
                       split_k=split)
    assert torch.equal(y, y2)


@pytest.mark.parametrize("m,split", [(16, 8), (9, 4), (32, 2), (20, 8), (32, 1), (64, 4)])
def test_linear_tc_split_reduction_epilogues(m, split):
    """Split-K reductions (power-of-two splits run the batched reduction, others the per-column one)
    with the residual-add and SwiGLU epilogues."""
    k_ = K()
    k, n = 2048, 256
    x, q, s, b = _mk_linear(m, k, n, seed=m * 10 + split)
    want = olin.i8_linear(x, q, s, b)
    xd, qd, sd, bd = dev(x, torch.bfloat16), dev(q), dev(s), dev(b)
    base = np.random.default_rng(split).standard_normal((m, n)).astype(np.float32)
    acc = dev(base)
    k_.i8_linear(xd, qd, sd, bd, y=acc, epilogue=k_.EPI_ADD_F32, algo="tc", split_k=split)
    close(acc.cpu().numpy(), base + want, rtol=1e-4, atol=1e-4)
    sw = k_.i8_linear(xd, qd, sd, bd, epilogue=k_.EPI_SWIGLU_BF16, algo="tc", split_k=split)
    wr = want.reshape(m, n // 128, 2, 64)
    gate, up = wr[:, :, 0, :].reshape(m, -1), wr[:, :, 1, :].reshape(m, -1)
    close(sw.float().cpu().numpy(), gate / (1 + np.exp(-gate)) * up)


@pytest.mark.parametrize("algo", ["simt", "tc"])
def test_linear_epilogues(algo):
    k_ = K()
    m, k, n = 24, 512, 256
    x, q, s, b = _mk_linear(m, k, n, seed=9)
    want = olin.i8_linear(x, q, s, b)
    xd, qd, sd, bd = dev(x, torch.bfloat16), dev(q), dev(s), dev(b)
    y = k_.i8_linear(xd, qd, sd, bd, epilogue=k_.EPI_STORE_F32, algo=algo)
    close(y.cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    base = np.random.default_rng(1).standard_normal((m, n)).astype(np.float32)
    acc = dev(base)
    k_.i8_linear(xd, qd, sd, bd, y=acc, epilogue=k_.EPI_ADD_F32, algo=algo)
    close(acc.cpu().numpy(), base + want, rtol=1e-4, atol=1e-4)
    g = k_.i8_linear(xd, qd, sd, bd, epilogue=k_.EPI_GELU_BF16, algo=algo)
    gelu = 0.5 * want * (1 + np.tanh(np.sqrt(2 / np.pi) * (want + 0.044715 * want ** 3)))
    close(g.float().cpu().numpy(), gelu)
    # SwiGLU: rows interleaved in groups of 64 gate rows + 64 up rows
    sw = k_.i8_linear(xd, qd, sd, bd, epilogue=k_.EPI_SWIGLU_BF16, algo=algo)
    wr = want.reshape(m, n // 128, 2, 64)
    gate, up = wr[:, :, 0, :].reshape(m, -1), wr[:, :, 1, :].reshape(m, -1)
    close(sw.float().cpu().numpy(), gate / (1 + np.exp(-gate)) * up)


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_linear_vs_reference_fixture(tag):
    d = np.load(os.path.join(G, "linear_cases.npz"))
    x = d[f"{tag}_x"]
    k = x.shape[1]
    if k % 16:
        pytest.skip("kernel needs k % 16 == 0")
    y = K().i8_linear(dev(x).to(torch.bfloat16), dev(d[f"{tag}_q"]), dev(d[f"{tag}_s"]), dev(d[f"{tag}_b"]),
                      epilogue=K().EPI_STORE_F32)
    # reference ran fp32 activations; ours are bf16-rounded: contract tolerance
    close(y.cpu().numpy(), d[f"{tag}_y"])


# ------------------------------------------------------------------ norms, rope, argmax
def test_rmsnorm_and_layernorm():
    rng = np.random.default_rng(3)
    h = rng.standard_normal((7, 3072)).astype(np.float32) * 3
    w = rng.standard_normal(3072).astype(np.float32)
    bb = rng.standard_normal(3072).astype(np.float32)
    x = K().rmsnorm(dev(h), dev(w), 1e-5).float().cpu().numpy()
    want = w * (h / np.sqrt((h.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-5))
    close(x, want, rtol=1e-2, atol=1e-3)
    x = K().layernorm(dev(h), dev(w), dev(bb), 1e-5).float().cpu().numpy()
    hd = h.astype(np.float64)
    mu = hd.mean(-1, keepdims=True)
    want = (hd - mu) / np.sqrt(((hd - mu) ** 2).mean(-1, keepdims=True) + 1e-5) * w + bb
    close(x, want, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("hq,hkv,d", [(24, 8, 128), (7, 1, 64), (12, 12, 64)])
def test_rope_kv_append(hq, hkv, d):
    k_ = K()
    rng = np.random.default_rng(hq)
    b, theta, max_pos = 5, 500000.0, 4096
    qkv = rng.standard_normal((b, (hq + 2 * hkv) * d)).astype(np.float32)
    pos = np.array([0, 1, 17, 1000, 4095], np.int32)
    table = np.stack([np.concatenate([rope_cos_sin(p, d, theta)[0][: d // 2], rope_cos_sin(p, d, theta)[1][: d // 2]])
                      for p in range(max_pos)]).astype(np.float32)
    nblk = 40
    slots = np.array([3 * 16 + 0, 7 * 16 + 5, 39 * 16 + 15, 0, 22 * 16 + 9], np.int32)
    kp = torch.zeros((nblk, hkv, 16, d), dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    qo = k_.rope_kv_append(dev(qkv), dev(pos), dev(table), dev(slots), hq, hkv, d, kp, vp)
    qo, kpn, vpn = qo.cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy()
    for i in range(b):
        c, s = rope_cos_sin(int(pos[i]), d, theta)
        heads = qkv[i].reshape(hq + 2 * hkv, d).astype(np.float64)
        rot = lambda x: x * c + np.concatenate([-x[d // 2:], x[: d // 2]]) * s
        for hh in range(hq):
            close(qo[i, hh], rot(heads[hh]), rtol=1e-5, atol=1e-5)
        blk, off = slots[i] // 16, slots[i] % 16
        for hh in range(hkv):
            close(kpn[blk, hh, off], rot(heads[hq + hh]), rtol=1e-2, atol=1e-2)
            close(vpn[blk, hh, off], heads[hq + hkv + hh], rtol=1e-2, atol=1e-2)


def test_argmax_first_max_index():
    """torch.argmax's answer (numpy's argmax agrees): the first maximal index; NaN counts as larger than
    every number, so a row with NaNs gives its first NaN; a row of -inf gives 0."""
    rng = np.random.default_rng(5)
    lg = rng.standard_normal((11, 128256)).astype(np.float32)
    lg[1, 77] = lg[1, 1000] = 50.0     # tie -> first index
    lg[2, :] = 0.0
    lg[3, -1] = 99.0
    lg[4, 5] = lg[4, 100000] = 60.0    # tie across the row's chunks
    lg[5, 128255] = 70.0               # last element
    lg[6, 90000] = np.nan              # a NaN after the row's maximum
    lg[6, 10] = 80.0
    lg[7, 70001] = lg[7, 3] = np.nan   # NaNs in two chunks: the first one
    lg[8, :] = np.nan
    lg[9, :] = -np.inf
    lg[10, 128255] = np.nan            # the last element, float4 path
    out = K().argmax_rows(dev(lg)).cpu().numpy()
    assert out.tolist() == np.argmax(lg, axis=1).tolist()
    assert out.tolist() == torch.from_numpy(lg).argmax(1).tolist()


@pytest.mark.parametrize("n,ld", [(5, 5), (31, 33), (1000, 1003), (50257, 50257), (50257, 50260)])
def test_argmax_short_and_unaligned_rows(n, ld):
    """Rows shorter than the split, and rows whose stride breaks 16-byte alignment (scalar path)."""
    rng = np.random.default_rng(n)
    full = rng.standard_normal((9, ld)).astype(np.float32)
    full[0, n - 1] = 40.0
    full[1, 0] = 40.0
    full[2, :n] = 1.0
    full[3, n // 2] = np.nan
    full[3, n - 1] = np.nan
    full[4, :n] = -np.inf
    lgd = dev(full)[:, :n]
    out = K().argmax_rows(lgd).cpu().numpy()
    assert out.tolist() == np.argmax(full[:, :n], axis=1).tolist()


# ------------------------------------------------------------------ paged attention
def _paged_case(b, hq, hkv, d, ctx, n_shared=0, extra_blocks=8, seed=0):
    rng = np.random.default_rng(seed)
    max_blocks = max((c + 15) // 16 for c in ctx)
    need = n_shared + sum((c + 15) // 16 - n_shared for c in ctx)
    nblk = need + extra_blocks
    perm = rng.permutation(nblk).astype(np.int32)
    tables = np.zeros((b, max_blocks), np.int32)
    shared = perm[:n_shared]
    nxt = n_shared
    for i, c in enumerate(ctx):
        nb = (c + 15) // 16
        tables[i, :n_shared] = shared
        tables[i, n_shared:nb] = perm[nxt:nxt + nb - n_shared]
        nxt += nb - n_shared
    kp = bf16_np(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32))
    vp = bf16_np(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32))
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    return q, kp, vp, tables, np.array(ctx, np.int32)


def _run_attn(q, kp, vp, tables, ctx, n_shared):
    d = q.shape[-1]
    out = K().paged_decode_attn(dev(q), dev(kp, torch.bfloat16), dev(vp, torch.bfloat16), dev(tables), dev(ctx),
                                1.0 / np.sqrt(d), n_shared_blocks=n_shared)
    return out.float().cpu().numpy().reshape(q.shape)


@pytest.mark.parametrize("tag", ["gqa", "mha", "llama"])
def test_attention_vs_reference_fixture(tag):
    d = np.load(os.path.join(G, "attn_cases.npz"))
    q = d[f"{tag}_q"]
    kp, vp = bf16_np(d[f"{tag}_kpool"]), bf16_np(d[f"{tag}_vpool"])
    got = _run_attn(q, kp, vp, d[f"{tag}_tables"], d[f"{tag}_ctx"], 0)
    close(got, d[f"{tag}_out"])


@pytest.mark.parametrize("b,hq,hkv,d,ctx,n_shared", [
    (1, 32, 8, 128, [1], 0),
    (3, 8, 2, 64, [15, 16, 17], 0),
    (4, 24, 8, 128, [100, 260, 33, 512], 0),
    (2, 14, 2, 64, [1000, 2047], 0),
    (16, 32, 8, 128, [2048 + 37 * i for i in range(16)], 0),
    (5, 24, 8, 128, [64 * 16 + 5 * i + 1 for i in range(5)], 64),
    (8, 32, 8, 128, [9 * 16 + i for i in range(8)], 9),
    (3, 12, 12, 64, [40, 48, 100], 2),
    (2, 16, 1, 128, [300, 17], 1),
])
def test_paged_attention_vs_oracle(b, hq, hkv, d, ctx, n_shared):
    q, kp, vp, tables, ctxa = _paged_case(b, hq, hkv, d, ctx, n_shared, seed=b * 7 + hq)
    got = _run_attn(q, kp, vp, tables, ctxa, n_shared)
    want = oatt.paged_decode_attention(q, kp, vp, tables, ctxa, 1.0 / np.sqrt(d))
    close(got, want)


def test_paged_attention_shared_prefix_equals_unshared():
    q, kp, vp, tables, ctxa = _paged_case(6, 24, 8, 128, [640 + 16 * i + 3 for i in range(6)], 40, seed=3)
    a = _run_attn(q, kp, vp, tables, ctxa, 40)
    b_ = _run_attn(q, kp, vp, tables, ctxa, 0)
    close(a, b_, rtol=1e-2, atol=5e-3)


@pytest.mark.parametrize("n_shared", [0, 2])
def test_paged_attention_ignores_nan_in_unused_slots(n_shared):
    """Pool slots past a sequence's length hold whatever was there (NaN here); the partial last block
    is read whole by TMA and its unused V rows must not leak into the output."""
    ctx = [37, 16 * 5 + 1, 200, 16 * 3]
    q, kp, vp, tables, ctxa = _paged_case(4, 24, 8, 128, ctx, n_shared, seed=11)
    for i, c in enumerate(ctxa):
        if c % 16:
            last = tables[i, (c - 1) // 16]
            kp[last, :, c % 16:, :] = np.nan
            vp[last, :, c % 16:, :] = np.nan
    got = _run_attn(q, kp, vp, tables, ctxa, n_shared)
    assert np.isfinite(got).all()
    close(got, oatt.paged_decode_attention(q, kp, vp, tables, ctxa, 1.0 / np.sqrt(128)))


def test_no_device_error_recorded():
    K().check_device()


# ------------------------------------------------------------------ tile-packed weights
@pytest.mark.parametrize("n,k", [(384, 256), (200, 96), (1000, 3072), (3072, 448)])
def test_pack_layout(n, k):
    rng = np.random.default_rng(n + k)
    q = rng.integers(-128, 128, size=(n, k), dtype=np.int8)
    pw = K().pack_weights(dev(q))
    tiles, kb = (n + 127) // 128, (k + 127) // 128
    ref = np.zeros((tiles * 128, kb * 128), np.int8)
    ref[:n, :k] = q
    ref = ref.reshape(tiles, 128, kb, 128).transpose(0, 2, 1, 3).reshape(-1)
    assert np.array_equal(pw.data.cpu().numpy(), ref)


@pytest.mark.parametrize("m,k,n,split", [(1, 3072, 640, 0), (32, 3072, 1024, 0), (32, 448, 896, 3),
                                         (100, 1024, 640, 2), (256, 512, 256, 0), (7, 96, 200, 1)])
def test_packed_linear_vs_oracle_and_rowmajor(m, k, n, split):
    x, q, s, b = _mk_linear(m, k, n, seed=m * 3 + k + n)
    k_ = K()
    xd, qd, sd, bd = dev(x, torch.bfloat16), dev(q), dev(s), dev(b)
    pw = k_.pack_weights(qd)
    y = k_.i8_linear(xd, pw, sd, bd, epilogue=k_.EPI_STORE_F32, split_k=split)
    close(y.cpu().numpy(), olin.i8_linear(x, q, s, b), rtol=1e-4, atol=1e-4)
    y_rm = k_.i8_linear(xd, qd, sd, bd, epilogue=k_.EPI_STORE_F32, algo="tc", split_k=split)
    if split:
        assert torch.equal(y, y_rm)  # same tiles, same split: identical sums


def test_packed_linear_swiglu_epilogue():
    k_ = K()
    m, k, n = 32, 768, 512
    x, q, s, b = _mk_linear(m, k, n, seed=77)
    want = olin.i8_linear(x, q, s, b).reshape(m, n // 128, 2, 64)
    gate, up = want[:, :, 0, :].reshape(m, -1), want[:, :, 1, :].reshape(m, -1)
    sw = k_.i8_linear(dev(x, torch.bfloat16), k_.pack_weights(dev(q)), dev(s), dev(b), epilogue=k_.EPI_SWIGLU_BF16)
    close(sw.float().cpu().numpy(), gate / (1 + np.exp(-gate)) * up)

"""Kernel parity at the isolated-sweep shapes of the workloads (seeded inputs, GPU vs the fp64 oracle).

INT8 linear: W N(0, 0.02) quantized per output channel (bit-exact quantizer), x bf16 N(0, 1),
M in {1, 8, 32, 128, 256} x (K, N) in {(3072, 9216), (3072, 8192), (8192, 3072), (4096, 14336)}:
* the tensor-core kernel on tile-packed codes (the path the decode engine runs) and on row-major codes;
* the CUDA-core GEMV at the decode batch sizes 1 and 8;
* the row-parallel form at one rank: partial pushed through a world-1 peer-memory communicator and
  reduced onto an fp32 residual (N <= 8192, the reduce kernel's row limit).
Paged decode attention: 32 query / 8 KV heads, head_dim 128, bf16 K/V N(0, 1), ctx in {512, 8192,
32768} x batch in {1, 16, 64}, shuffled block tables, the first half of every sequence's blocks shared by
the batch. The oracle checks four sequences of each case (first, last, two seeded picks) on every head;
the pools are generated on the device and only the checked sequences' blocks are copied back.

Tolerance: |got - want| <= 1e-2 + 2e-2 * |want| (bf16 activations against fp64 dequantize-then-matmul /
SDPA of the same bf16-rounded inputs)."""

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import linear as olin

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-2, 1e-2
KN = [(3072, 9216), (3072, 8192), (8192, 3072), (4096, 14336)]
MS = [1, 8, 32, 128, 256]


def close(got, want, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


_CACHE = {}


def _linear_case(k, n):
    """Device (x bf16 [256, k], codes, scales, packed codes) and the fp64 oracle y [256, n]."""
    if (k, n) not in _CACHE:  # all four shapes stay cached (~0.3 GB of device codes)
        from microgen_b200 import kernels as K
        g = torch.Generator(device="cuda").manual_seed(k * 7 + n)
        w = torch.randn((n, k), generator=g, device="cuda").mul_(0.02)
        q, s = K.quantize_rows_i8(w)
        del w
        x = torch.randn((max(MS), k), generator=g, device="cuda").to(torch.bfloat16)
        want = olin.i8_linear(x.float().cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
        _CACHE[(k, n)] = (x, q, s, K.pack_weights(q), want)
    return _CACHE[(k, n)]


@pytest.mark.parametrize("k,n", KN)
@pytest.mark.parametrize("m", MS)
def test_c4_linear_tensor_core(k, n, m):
    from microgen_b200 import kernels as K
    x, q, s, pw, want = _linear_case(k, n)
    y = K.i8_linear(x[:m], pw, s, epilogue=K.EPI_STORE_F32)
    close(y.cpu().numpy(), want[:m])
    y_rm = K.i8_linear(x[:m], q, s, epilogue=K.EPI_STORE_BF16, algo="tc")
    close(y_rm.float().cpu().numpy(), want[:m])


@pytest.mark.parametrize("k,n", KN)
@pytest.mark.parametrize("m", [1, 8])
def test_c4_linear_simt(k, n, m):
    from microgen_b200 import kernels as K
    x, q, s, pw, want = _linear_case(k, n)
    y = K.i8_linear(x[:m], q, s, epilogue=K.EPI_STORE_F32, algo="simt")
    close(y.cpu().numpy(), want[:m])


@pytest.mark.parametrize("k,n", [kn for kn in KN if kn[1] <= 8192])
@pytest.mark.parametrize("m", [1, 32, 256])
def test_c4_row_parallel_push_reduce(k, n, m):
    from microgen_b200 import kernels as K
    x, q, s, pw, want = _linear_case(k, n)
    comm = K.Comm(0, 1, max(MS) * n, exchange=lambda mine: [mine])
    try:
        h0 = torch.randn((m, n), generator=torch.Generator(device="cuda").manual_seed(m), device="cuda")
        h = h0.clone()
        K.i8_linear_rowpar(x[:m], pw, s, comm)
        K.rowpar_reduce_norm(comm, h, None, K.NORM_NONE)
        torch.cuda.synchronize()
        close(h.cpu().numpy(), h0.cpu().numpy().astype(np.float64) + want[:m])  # partials travel as bf16
        K.check_device()
    finally:
        comm.close()


def _attn_case(ctx, b, seed, hq=32, hkv=8, d=128):
    import random
    nb = (ctx + 15) // 16
    ns = nb // 2
    nblocks = ns + b * (nb - ns)
    order = list(range(nblocks))
    random.Random(seed).shuffle(order)
    tables = np.zeros((b, nb), np.int32)
    tables[:, :ns] = order[:ns]
    for i in range(b):
        tables[i, ns:] = order[ns + i * (nb - ns):ns + (i + 1) * (nb - ns)]
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn((nblocks, hkv, 16, d), generator=g, device="cuda").to(torch.bfloat16)
    vp = torch.randn((nblocks, hkv, 16, d), generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn((b, hq, d), generator=g, device="cuda")
    return q, kp, vp, tables, ns


@pytest.mark.parametrize("ctx", [512, 8192, 32768])
@pytest.mark.parametrize("b", [1, 16, 64])
def test_c4_paged_attention_half_shared(ctx, b):
    from microgen_b200 import kernels as K
    d = 128
    q, kp, vp, tables, ns = _attn_case(ctx, b, seed=ctx + b)
    ctxs = np.full(b, ctx, np.int32)
    out = K.paged_decode_attn(q, kp, vp, torch.from_numpy(tables).cuda(), torch.from_numpy(ctxs).cuda(),
                              d ** -0.5, n_shared_blocks=ns)
    got = out.float().cpu().numpy().reshape(b, 32, d)
    rng = np.random.default_rng(ctx * b)
    rows = sorted({0, b - 1, int(rng.integers(0, b)), int(rng.integers(0, b))})
    for i in rows:
        ids = torch.from_numpy(tables[i].astype(np.int64)).cuda()
        kk = kp.index_select(0, ids).float().cpu().numpy()[None]   # [1, nb, hkv, 16, d]
        vv = vp.index_select(0, ids).float().cpu().numpy()[None]
        tab = np.arange(len(tables[i]), dtype=np.int32)[None]
        want = oatt.paged_decode_attention(q[i:i + 1].cpu().numpy(), kk[0], vv[0], tab, ctxs[i:i + 1], d ** -0.5)
        close(got[i:i + 1], want)
    K.check_device()

"""The allocation-free attention entry point against the regular one (GPU).

``mg_paged_decode_attn_noalloc`` serves callers that cannot allocate device memory themselves (a host
binding that only receives pointers from another runtime's allocator, or a serving loop that must not
take cudaMalloc's device-wide synchronisation mid-step): it runs the same paged decode attention with
its split scratch in a fixed library-owned device array. These tests call it through the C ABI with
caller-allocated inputs and outputs and compare it with ``mg_paged_decode_attn`` (the existing entry
point, given a workspace) on consecutive calls, using the attention tolerance of the other GPU tests.

The file name sorts last, so a run that stops at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 1e-2


def _case(b, hq, hkv, d, ctx, n_shared, seed):
    rng = np.random.default_rng(seed)
    max_blocks = max((c + 15) // 16 for c in ctx)
    nblk = n_shared + sum((c + 15) // 16 - n_shared for c in ctx) + 4
    perm = rng.permutation(nblk).astype(np.int32)
    tables = np.zeros((b, max_blocks), np.int32)
    tables[:, :n_shared] = perm[:n_shared]
    nxt = n_shared
    for i, c in enumerate(ctx):
        nb = (c + 15) // 16
        tables[i, n_shared:nb] = perm[nxt:nxt + nb - n_shared]
        nxt += nb - n_shared
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    kp = dev(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32)).to(torch.bfloat16)
    vp = dev(rng.standard_normal((nblk, hkv, 16, d)).astype(np.float32)).to(torch.bfloat16)
    q = dev(rng.standard_normal((b, hq, d)).astype(np.float32))
    return q, kp, vp, dev(tables), dev(np.array(ctx, np.int32)), n_shared


def _noalloc(lib, q, kp, vp, tables, ctx, n_shared, out):
    b, hq, d = q.shape
    return lib.mg_paged_decode_attn_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kp.data_ptr()), ctypes.c_void_p(vp.data_ptr()), kp.shape[0],
        ctypes.c_void_p(tables.data_ptr()), tables.shape[1], ctypes.c_void_p(ctx.data_ptr()), b, hq, kp.shape[1], d,
        n_shared, 1.0 / float(np.sqrt(d)), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _existing(q, kp, vp, tables, ctx, n_shared):
    from microgen_b200 import kernels as K
    return K.paged_decode_attn(q, kp, vp, tables, ctx, 1.0 / float(np.sqrt(q.shape[-1])), n_shared_blocks=n_shared)


def _close(got, want):
    got, want = got.float().cpu().numpy().astype(np.float64), want.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - want)
    assert not (err > ATOL + RTOL * np.abs(want)).any(), f"max err {err.max():.3e}"


def test_noalloc_matches_existing_entry_point_on_consecutive_calls():
    from microgen_b200 import _lib
    lib = _lib.load()
    cases = [
        _case(8, 24, 8, 128, [1024 + 37 * i for i in range(8)], 32, seed=1),   # shared prefix, split partials
        _case(3, 14, 2, 64, [200, 17, 1000], 0, seed=2),                        # different shape, no sharing
        _case(8, 24, 8, 128, [1024 + 37 * i for i in range(8)], 32, seed=3),   # first shape again, new data
    ]
    for q, kp, vp, tables, ctx, n_shared in cases:
        out = torch.empty((q.shape[0], q.shape[1] * q.shape[2]), dtype=torch.bfloat16, device="cuda")
        assert _noalloc(lib, q, kp, vp, tables, ctx, n_shared, out) == _lib.MG_OK
        want = _existing(q, kp, vp, tables, ctx, n_shared)
        torch.cuda.synchronize()
        _close(out, want)
    _lib.check_device(torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from microgen_b200 import _lib
    lib = _lib.load()
    # 64 sequences x 32 heads over 2048 blocks with a 1024-block shared prefix needs far more split
    # scratch than the fixed array holds: the call must refuse before launching anything.
    need = ctypes.c_size_t(0)
    assert lib.mg_paged_attn_workspace_bytes(64, 32, 8, 128, 2048, 1024, ctypes.byref(need)) == _lib.MG_OK
    assert need.value > 16 << 20
    q = torch.zeros((64, 32, 128), dtype=torch.float32, device="cuda")
    kp = torch.zeros((1, 8, 16, 128), dtype=torch.bfloat16, device="cuda")
    tables = torch.zeros((64, 2048), dtype=torch.int32, device="cuda")
    ctx = torch.ones(64, dtype=torch.int32, device="cuda")
    out = torch.empty((64, 32 * 128), dtype=torch.bfloat16, device="cuda")
    assert _noalloc(lib, q, kp, kp, tables, ctx, 1024, out) == _lib.MG_ERR_UNSUPPORTED

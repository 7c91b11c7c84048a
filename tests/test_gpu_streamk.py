"""Stream-K INT8 linear (tile-packed codes, m <= 128) against the fp64 oracle.

Shapes are chosen for the unit split: one unit (grid of one CTA), tiles spread over many CTAs (the
finisher adds several partials), tiles wholly inside a CTA, ragged N (a partial last 128-row tile) and
ragged K (a partial last K block), at every MMA width (16, 32, 64, 128 tokens). Every epilogue is checked,
results are bit-identical from run to run (partials are added in a fixed CTA order), the flags of the
workspace are zero again after each launch (the next launch may reuse it), and the row-parallel push at
one rank equals the plain linear added onto the residual."""

import numpy as np
import pytest
import torch

from oracle import linear as olin
from oracle.quant import quantize_rows_i8 as oq

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-2, 1e-2


def K():
    from microgen_b200 import kernels
    return kernels


def close(got, want, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


def _case(m, k, n, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    q, s = oq(w)
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(torch.bfloat16)
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    want = olin.i8_linear(x.float().numpy(), q, s, b)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return x.cuda(), K().pack_weights(d(q)), d(s), d(b), want


def _flags_zero(ws, m, k, n):
    """The flag words lead the workspace, one per CTA of the launch's grid (SMs x CTAs per SM, at most one
    CTA per two units): every flag the kernel raised has been cleared again."""
    torch.cuda.synchronize()
    mp = 16 if m <= 16 else 32 if m <= 32 else 64 if m <= 64 else 128
    units = -(-n // 128) * -(-k // 128)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    grid = min(sms * (2 if mp <= 32 else 1), max(1, units // 2))
    return int(ws[:grid * 4].view(torch.int32).abs().sum().item()) == 0


SHAPES = [(128, 128), (2048, 256), (3072, 3072), (3072, 1024), (8192, 768), (448, 200), (96, 640), (3072, 16384)]


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 17, 32, 33, 64, 100, 128])
def test_streamk_store_f32_vs_oracle_and_deterministic(m, k, n):
    k_ = K()
    x, pw, s, b, want = _case(m, k, n, seed=m * 31 + k + n)
    ws = k_.sk_workspace(m, x.device)
    y = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_STORE_F32, workspace=ws)
    close(y.cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    assert _flags_zero(ws, m, k, n)
    y2 = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_STORE_F32, workspace=ws)
    assert torch.equal(y, y2)
    k_.check_device()


@pytest.mark.parametrize("m", [8, 32, 128])
def test_streamk_epilogues(m):
    k_ = K()
    k, n = 2048, 512
    x, pw, s, b, want = _case(m, k, n, seed=m)
    ws = k_.sk_workspace(m, x.device)
    y = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_STORE_BF16, workspace=ws)
    close(y.float().cpu().numpy(), want)
    base = np.random.default_rng(m).standard_normal((m, n)).astype(np.float32)
    acc = torch.from_numpy(base).cuda()
    k_.i8_linear(x, pw, s, b, y=acc, epilogue=k_.EPI_ADD_F32, workspace=ws)
    close(acc.cpu().numpy(), base + want, rtol=1e-4, atol=1e-4)
    g = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_GELU_BF16, workspace=ws)
    close(g.float().cpu().numpy(), 0.5 * want * (1 + np.tanh(np.sqrt(2 / np.pi) * (want + 0.044715 * want ** 3))))
    sw = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_SWIGLU_BF16, workspace=ws)
    wr = want.reshape(m, n // 128, 2, 64)
    gate, up = wr[:, :, 0, :].reshape(m, -1), wr[:, :, 1, :].reshape(m, -1)
    close(sw.float().cpu().numpy(), gate / (1 + np.exp(-gate)) * up)
    assert _flags_zero(ws, m, k, n)
    k_.check_device()


def test_streamk_large_m_falls_back_to_cluster_kernel():
    k_ = K()
    x, pw, s, b, want = _case(200, 1024, 384, seed=5)
    ws = k_.sk_workspace(128, x.device)
    y = k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_STORE_F32, workspace=ws)
    close(y.cpu().numpy(), want, rtol=1e-4, atol=1e-4)


def test_streamk_workspace_too_small_is_rejected():
    k_ = K()
    x, pw, s, b, _ = _case(32, 3072, 3072, seed=6)
    small = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError):
        k_.i8_linear(x, pw, s, b, epilogue=k_.EPI_STORE_F32, workspace=small)


@pytest.mark.parametrize("m", [1, 32, 128])
def test_streamk_row_parallel_push_world1(m):
    k_ = K()
    k, n = 3072, 3072
    x, pw, s, b, want = _case(m, k, n, seed=m + 3)
    ws = k_.sk_workspace(m, x.device)
    comm = k_.Comm(0, 1, m * n, exchange=lambda mine: [mine])
    try:
        h0 = np.random.default_rng(m).standard_normal((m, n)).astype(np.float32)
        h = torch.from_numpy(h0).cuda()
        for _ in range(2):  # both receive sets
            h.copy_(torch.from_numpy(h0))
            k_.i8_linear_rowpar(x, pw, s, comm, workspace=ws)
            k_.rowpar_reduce_norm(comm, h, b, k_.NORM_NONE)
            torch.cuda.synchronize()
            close(h.cpu().numpy(), h0 + want)  # partials travel as bf16
        assert _flags_zero(ws, m, k, n)
        k_.check_device()
    finally:
        comm.close()

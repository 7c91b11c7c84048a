"""Fused row-parallel all-reduce on one GPU (the multi-GPU path is tests/test_gpu_tp.py).

* world 1: the row-parallel push + reduce(+norm) equals ``h + x·(q·s)ᵀ + bias`` and the RMSNorm /
  LayerNorm of it, against the fp64 oracle (partials travel as bf16: the contract's bf16 tolerance);
* a missing peer: a world-2 communicator whose second rank never pushes — the reduce kernel's
  bounded wait gives up after about a second, records MG_ERR_TIMEOUT, and the host raises
  TimeoutError; the context stays usable (a later world-1 reduce still works);
* the vocab-parallel greedy argmax (``mg_vocab_argmax``) at world 1 equals the local argmax kernel on
  rows with exact ties, -inf and NaN entries, interleaved with row-parallel pushes of the same epoch
  sequence; with a peer that never publishes it times out the same way.
"""

import time

import numpy as np
import pytest
import torch

from oracle import linear as olin
from oracle.quant import quantize_rows_i8

pytestmark = pytest.mark.gpu


def _case(m, k, n, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    q, s = quantize_rows_i8(w)
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(torch.bfloat16)
    h0 = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32) * np.float32(0.1)
    g = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    gb = (0.1 * rng.standard_normal(n)).astype(np.float32)
    return x, q, s, h0, bias, g, gb


def _close(got, want, rtol, atol):
    err = np.abs(np.asarray(got, np.float64) - want)
    assert not (err > atol + rtol * np.abs(want)).any(), f"max err {err.max():.3e}"


@pytest.mark.parametrize("norm", [0, 1, 2])
def test_world1_push_reduce_norm(norm):
    from microgen_b200 import kernels as K
    m, k, n = 24, 1024, 768
    x, q, s, h0, bias, g, gb = _case(m, k, n, seed=norm)
    comm = K.Comm(0, 1, m * n, exchange=lambda mine: [mine])
    try:
        d = lambda a: torch.from_numpy(a).cuda()
        h = d(h0.copy())
        pw = K.pack_weights(d(q))
        for rep in range(2):  # the second push uses the other receive set
            h.copy_(d(h0))
            K.i8_linear_rowpar(x.cuda(), pw, d(s), comm)
            xo = K.rowpar_reduce_norm(comm, h, d(bias), norm, d(g), d(gb), 1e-5)
            torch.cuda.synchronize()
            want_h = h0 + olin.i8_linear(x.float().numpy(), q, s, bias)
            _close(h.cpu().numpy(), want_h, 2e-2, 1e-2)  # partials travel as bf16
            if norm == 1:
                want_x = g * (want_h / np.sqrt((want_h ** 2).mean(-1, keepdims=True) + 1e-5))
                _close(xo.float().cpu().numpy(), want_x, 2e-2, 1e-2)
            elif norm == 2:
                mu = want_h.mean(-1, keepdims=True)
                want_x = (want_h - mu) / np.sqrt(((want_h - mu) ** 2).mean(-1, keepdims=True) + 1e-5) * g + gb
                _close(xo.float().cpu().numpy(), want_x, 2e-2, 1e-2)
        K.check_device()
    finally:
        comm.close()


def test_missing_peer_times_out_and_context_survives():
    from microgen_b200 import kernels as K
    m, k, n = 4, 256, 256
    x, q, s, h0, bias, g, gb = _case(m, k, n, seed=9)
    d = lambda a: torch.from_numpy(a).cuda()
    # rank 0 of a world of 2 whose rank-1 slot maps to itself: nothing ever pushes as rank 1
    comm = K.Comm(0, 2, m * n, exchange=lambda mine: [mine, mine])
    try:
        h = d(h0.copy())
        K.i8_linear_rowpar(x.cuda(), K.pack_weights(d(q)), d(s), comm)
        t0 = time.time()
        K.rowpar_reduce_norm(comm, h, d(bias), 1, d(g), None, 1e-5)
        with pytest.raises(TimeoutError):
            K.check_device()
        assert 0.5 < time.time() - t0 < 30
    finally:
        comm.close()
    test_world1_push_reduce_norm(1)  # the context is still healthy


def test_decode_raises_when_a_peer_never_pushes():
    """The serving path surfaces a peer timeout: a TP decode step whose row-parallel reduces wait on a rank
    that never pushes (a world-2 communicator whose second rank maps to this process) ends in TimeoutError
    from ``decode`` rather than returning logits built from missing partials."""
    from microgen_b200 import kernels as K
    from microgen_b200.backends import B200QuantizedBackend
    from tests._hf_models import TINY, make_hf_model
    model, _ = make_hf_model(TINY["llama"], seed=0)
    be = B200QuantizedBackend(max_batch=1, max_seq_len=64, use_cuda_graph=False)
    be.load_model("tiny", model_instance=model)
    logits, cache = be.prefill(torch.tensor([[1, 2, 3]]))
    K.check_device()
    comm = K.Comm(0, 2, be.engine.max_batch * be.spec.hidden, exchange=lambda mine: [mine, mine])
    be.engine.comm = comm
    try:
        with pytest.raises(TimeoutError):
            be.decode(be.sample(logits), cache=cache)
    finally:
        be.engine.comm = None
        torch.cuda.synchronize()
        comm.close()
    test_world1_push_reduce_norm(1)  # the context is still healthy


def _vocab_logits(m, n, seed):
    g = torch.Generator().manual_seed(seed)
    lg = torch.randint(-4, 5, (m, n), generator=g).float()  # small integers: exact ties everywhere
    lg[1] = float("-inf")
    lg[2, ::5] = float("nan")
    lg[3] = float("nan")
    return lg.cuda()


def test_world1_vocab_argmax_matches_local_argmax():
    from microgen_b200 import kernels as K
    m, k, n = 8, 256, 256
    x, q, s, h0, bias, g, gb = _case(m, k, n, seed=3)
    d = lambda a: torch.from_numpy(a).cuda()
    comm = K.Comm(0, 1, m * n, exchange=lambda mine: [mine])
    try:
        h = d(h0.copy())
        pw = K.pack_weights(d(q))
        for rep in range(3):  # pushes and argmax exchanges share one epoch sequence and both sets
            K.i8_linear_rowpar(x.cuda(), pw, d(s), comm)
            K.rowpar_reduce_norm(comm, h, d(bias), 0)
            lg = _vocab_logits(m, 1000 + rep, seed=rep)
            want = K.argmax_rows(lg).cpu()
            assert torch.equal(want, lg.cpu().argmax(1).to(want.dtype))  # torch.argmax, NaN rows included
            got = K.vocab_argmax(comm, lg, 0).cpu()
            assert torch.equal(got, want), (got, want)
            # a column slice with a row stride > its width, as the engine's shard buffer is
            wide = torch.full((m, 1200), 7.0, device="cuda")
            wide[:, :1000] = lg[:, :1000]
            got2 = K.vocab_argmax(comm, wide[:, :1000], 0).cpu()
            assert torch.equal(got2, K.argmax_rows(lg[:, :1000]).cpu())
        K.check_device()
    finally:
        comm.close()


def test_vocab_argmax_missing_peer_times_out():
    from microgen_b200 import kernels as K
    comm = K.Comm(0, 2, 4096, exchange=lambda mine: [mine, mine])
    try:
        t0 = time.time()
        K.vocab_argmax(comm, _vocab_logits(4, 300, seed=1), 0)
        with pytest.raises(TimeoutError):
            K.check_device()
        assert 0.5 < time.time() - t0 < 30
    finally:
        comm.close()
    test_world1_vocab_argmax_matches_local_argmax()  # the context is still healthy

"""The persistent decode-layer kernel (mg_decode_block) against the kernel-per-op decode step.

Both paths compute the same arithmetic — INT8 codes x bf16 activations with fp32 accumulation, the same
bf16 rounding points, the same norms, RoPE and paged K/V slots — so a whole decode step through
``B200QuantizedBackend`` must give the same logits within the contract tolerance
(|err| <= 1e-2 + 2e-2 |ref|) and the same greedy tokens, step after step (teacher-forced with the
kernel-per-op path's own tokens so one flipped near-tie cannot derail the comparison). The block path is
also bit-reproducible: its split-K partials are added in a fixed order."""

import json
import os

import numpy as np
import pytest
import torch

from microgen_b200 import kernels as K

pytestmark = pytest.mark.gpu
RTOL, ATOL = 2e-2, 1e-2

# a Llama-3.2-3B-wide slice (two layers, smaller vocabulary) at batch 32 with a shared prefix
LLAMA_3B_SLICE = dict(family="llama", hidden=3072, layers=2, heads=24, kv_heads=8, head_dim=128, inter=8192,
                      vocab=8192, eps=1e-5, rope_theta=500000.0)
QWEN_05B_SLICE = dict(family="qwen2", hidden=896, layers=2, heads=14, kv_heads=2, head_dim=64, inter=4864,
                      vocab=4096, eps=1e-6, rope_theta=1000000.0, tie=True, qkv_bias=True)
GPT2_SLICE = dict(family="gpt2", hidden=768, layers=2, heads=12, kv_heads=12, head_dim=64, inter=3072,
                  vocab=4096, eps=1e-5, max_pos=1024, tie=True, qkv_bias=True, mlp_bias=True)


def _backends(shape, monkeypatch, batch, seq):
    from microgen_b200.backends import B200QuantizedBackend
    from microgen_b200.model_spec import spec_from_hf_config
    from tests._hf_models import seeded_state_for_shape
    cfg, state = seeded_state_for_shape(shape, seed=0)
    spec = spec_from_hf_config(cfg)
    out = []
    for block in ("0", "1"):
        monkeypatch.setenv("MG_BLOCK", block)
        be = B200QuantizedBackend(max_batch=batch, max_seq_len=seq, free_list_seed=7)
        be.load_state(spec, state)
        out.append(be)
    monkeypatch.delenv("MG_BLOCK")
    assert out[0].engine.block_args is None and out[1].engine.block_args is not None
    return out


def _close(got, want, what, atol=ATOL):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + RTOL * np.abs(want)
    if bad.any() and bad.ndim == 2:
        rows, cols = np.nonzero(bad)
        print(f"{what}: bad rows {np.unique(rows).tolist()[:40]}; bad 128-column tiles "
              f"{np.unique(cols // 128).tolist()[:40]}; count per tile {np.bincount(cols // 128).tolist()}")
    assert not bad.any(), f"{what}: {bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


def _prompts(vocab, batch, length, shared, seed):
    g = np.random.default_rng(seed)
    head = g.integers(0, vocab, shared)
    return torch.tensor(np.stack([np.concatenate([head, g.integers(0, vocab, length - shared)])
                                  for _ in range(batch)]))


@pytest.mark.parametrize("shape,batch,shared", [
    ("tiny_llama", 4, 16), ("tiny_qwen2", 3, 0), ("tiny_gpt2", 2, 0),
    ("llama_3b_slice", 32, 32), ("qwen_05b_slice", 16, 0), ("gpt2_slice", 8, 0)])
def test_block_step_matches_kernel_per_op(shape, batch, shared, monkeypatch):
    from tests._hf_models import TINY
    shapes = {"tiny_llama": TINY["llama"], "tiny_qwen2": TINY["qwen2"], "tiny_gpt2": TINY["gpt2"],
              "llama_3b_slice": LLAMA_3B_SLICE, "qwen_05b_slice": QWEN_05B_SLICE, "gpt2_slice": GPT2_SLICE}
    s = shapes[shape]
    # The two paths add the split-K partials of each linear in different orders, so at the workload widths
    # a bf16 activation now and then rounds to the neighbouring value (1 ulp = 0.4 %); over two layers that
    # moves logits by up to ~0.025. The logit check therefore uses the model-level bound of the full-shape
    # tests (4x the per-kernel 1e-2); every phase is held to the per-kernel bound by
    # test_block_phases_vs_float64.
    atol = ATOL if s["hidden"] <= 256 else 4 * ATOL
    ref, blk = _backends(s, monkeypatch, batch, 96)
    prompts = _prompts(s["vocab"], batch, 40, shared, seed=11)
    lr, cr = ref.prefill(prompts)
    lb, cb = blk.prefill(prompts)
    for step in range(12):
        try:
            K.check_device()
        except TimeoutError:
            d = K.decode_block_diag()
            prog = [(c, d[32 + 4 * c] & 0xffff, d[32 + 4 * c] >> 16, d[33 + 4 * c], d[34 + 4 * c] & 0xffff,
                     d[34 + 4 * c] >> 16, d[35 + 4 * c] & 0xffff, (d[35 + 4 * c] >> 16) & 0x7fff,
                     d[35 + 4 * c] >> 31) for c in range(148)]
            print("progress (cta, x loads, w loads, converted, mma units, mma segs, epi segs, epi stage, "
                  "epi waiting):")
            for row in prog:
                print(row)
            raise AssertionError(f"{shape} step {step}: device wait gave up; diag {d[:32]}")
        _close(lb.float().cpu().numpy(), lr.float().cpu().numpy(), f"{shape} step {step}", atol=atol)
        tok = ref.sample(lr)
        lr, cr = ref.decode(tok, cache=cr)
        lb, cb = blk.decode(tok, cache=cb)
    K.check_device()
    cr.free()
    cb.free()


def test_block_step_is_bit_reproducible(monkeypatch):
    ref, blk = _backends(LLAMA_3B_SLICE, monkeypatch, 32, 96)
    del ref
    prompts = _prompts(LLAMA_3B_SLICE["vocab"], 32, 40, 32, seed=3)
    runs = []
    for _ in range(2):
        logits, cache = blk.prefill(prompts)
        seq = [logits.float().cpu().numpy()]
        for _ in range(4):
            logits, cache = blk.decode(blk.sample(logits), cache=cache)
            seq.append(logits.float().cpu().numpy())
        cache.free()
        runs.append(np.stack(seq))
    assert np.array_equal(runs[0], runs[1])


def test_block_launch_count(monkeypatch):
    """One launch per layer boundary: embed + (layers + 1) blocks + layers attentions (+ combine kernels)
    + lm_head + argmax, against ~8 launches per layer for the kernel-per-op step."""
    from microgen_b200 import _lib
    from tests._hf_models import TINY
    ref, blk = _backends(TINY["llama"], monkeypatch, 2, 64)
    prompts = _prompts(TINY["llama"]["vocab"], 2, 20, 0, seed=1)
    counts = []
    for be in (ref, blk):
        be.use_cuda_graph = False
        logits, cache = be.prefill(prompts)
        n0 = _lib.LAUNCHES[0]
        be.decode(be.sample(logits), cache=cache)
        counts.append(_lib.LAUNCHES[0] - n0)
        cache.free()
    L = TINY["llama"]["layers"]
    assert counts[1] <= 1 + (L + 1) + 2 * L + 2 + 1, counts  # (+1: the greedy sample's argmax)
    assert counts[1] < counts[0], counts


def test_block_args_rejected():
    """Argument errors come back as MG_ERR_INVALID_ARG / MG_ERR_UNSUPPORTED before any launch."""
    from microgen_b200 import _lib
    a = K.BlockArgs()
    with pytest.raises(_lib.MGError):
        K.block_workspace_bytes(a)  # no phase enabled
    a.flags = K.BLK_N1
    a.m, a.hidden, a.norm = 40, 256, K.NORM_RMS
    with pytest.raises(_lib.MGError):
        K.block_workspace_bytes(a)  # more tokens than one launch holds


# ---- one launch, phase by phase, against a float64 restatement -------------------------------------
def _rope_table(D, theta, max_pos):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))
    ang = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], 1).contiguous()


class _Layer:
    """Random INT8 weights of one decoder layer (codes quantized on the device), packed for the kernel,
    with float64 dequantized copies for the restatement."""

    def __init__(self, H, hq, hkv, D, inter, family, g):
        from microgen_b200.engine import _interleave_gate_up
        dev = torch.device("cuda")
        self.H, self.hq, self.hkv, self.D, self.family = H, hq, hkv, D, family
        w = lambda n, k: (torch.randn((n, k), generator=g) * 0.02).to(dev)
        b = lambda n: (torch.randn((n,), generator=g) * 0.1).to(dev)
        nq = (hq + 2 * hkv) * D

        def quant(t):
            q, s = K.quantize_rows_i8(t)
            return q, s, (q.double() * s.double()[:, None]).cpu().numpy()

        self.qkv_q, self.qkv_s, self.Wqkv = quant(w(nq, H))
        self.o_q, self.o_s, self.Wo = quant(w(H, hq * D))
        self.d_q, self.d_s, self.Wd = quant(w(H, inter))
        self.qkv_b, self.o_b, self.d_b = b(nq), b(H), b(H)
        if family == "gpt2":
            self.gu_q, self.gu_s, self.Wgu = quant(w(inter, H))
            self.gu_b = b(inter)
        else:
            gq, gs, _ = quant(w(inter, H))
            uq, us, _ = quant(w(inter, H))
            self.gu_q, self.gu_s, gb = _interleave_gate_up(gq, gs, uq, us, b(inter), b(inter))
            self.gu_b = gb
            self.Wgu = (self.gu_q.double() * self.gu_s.double()[:, None]).cpu().numpy()
        self.n1_w, self.n2_w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(dev), \
            (1.0 + 0.1 * torch.randn(H, generator=g)).to(dev)
        self.n1_b, self.n2_b = (b(H), b(H)) if family == "gpt2" else (None, None)
        self.packed = {n: K.pack_weights(getattr(self, n + "_q")) for n in ("qkv", "o", "gu", "d")}


def _np(t):
    return t.detach().double().cpu().numpy()


def _norm64(h, w, b, family, eps=1e-5):
    if family == "gpt2":
        mu = h.mean(-1, keepdims=True)
        var = ((h - mu) ** 2).mean(-1, keepdims=True)
        return (h - mu) / np.sqrt(var + eps) * w + b
    return w * (h / np.sqrt((h * h).mean(-1, keepdims=True) + eps))


@pytest.mark.parametrize("family,H,hq,hkv,D,inter,m", [
    ("llama", 3072, 24, 8, 128, 8192, 32),    # the Llama-3.2-3B layer, batch 32
    ("qwen2", 896, 7, 1, 64, 2432, 16),       # a Qwen2.5-0.5B rank at TP=2 (QKV ends in a partial tile)
    ("gpt2", 768, 12, 12, 64, 3072, 8),       # a GPT-2-small layer: LayerNorm, GELU, every bias
    ("llama", 256, 4, 2, 32, 192, 3),         # fewer units than SMs; down's K ends mid block
])
def test_block_phases_vs_float64(family, H, hq, hkv, D, inter, m):
    from microgen_b200 import _lib
    torch.cuda.set_device(0)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(H + m)
    L = _Layer(H, hq, hkv, D, inter, family, g)
    nblk, max_pos = 16, 256
    act_cols = inter
    h0 = torch.randn((m, H), generator=g).to(dev)
    attn = torch.randn((m, hq * D), generator=g).to(dev).to(torch.bfloat16)
    x2 = torch.zeros((m, H), dtype=torch.bfloat16, device=dev)
    x1 = torch.zeros((m, H), dtype=torch.bfloat16, device=dev)
    act = torch.zeros((m, act_cols), dtype=torch.bfloat16, device=dev)
    q_out = torch.zeros((m, hq, D), dtype=torch.float32, device=dev)
    kp = torch.zeros((nblk, hkv, 16, D), dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    pos = torch.randint(0, max_pos, (m,), generator=g, dtype=torch.int32).to(dev)
    slots = torch.from_numpy(np.random.default_rng(m).permutation(nblk * 16)[:m].astype(np.int32)).to(dev)
    cs = _rope_table(D, 10000.0, max_pos).to(dev) if family != "gpt2" else None
    ptr = lambda t: 0 if t is None else t.data_ptr()

    def args(flags, h):
        a = K.BlockArgs()
        a.m, a.flags, a.hidden, a.hq, a.hkv, a.head_dim = m, flags, H, hq, hkv, D
        a.norm = K.NORM_LAYER if family == "gpt2" else K.NORM_RMS
        a.mlp = K.EPI_GELU_BF16 if family == "gpt2" else K.EPI_SWIGLU_BF16
        a.eps = 1e-5
        a.o = K.block_linear(L.packed["o"], L.o_s, L.o_b)
        a.gate_up = K.block_linear(L.packed["gu"], L.gu_s, L.gu_b)
        a.down = K.block_linear(L.packed["d"], L.d_s, L.d_b)
        a.qkv = K.block_linear(L.packed["qkv"], L.qkv_s, L.qkv_b)
        a.h, a.attn, a.x2, a.act, a.x1 = ptr(h), ptr(attn), ptr(x2), ptr(act), ptr(x1)
        a.n2_w, a.n2_b, a.n1_w, a.n1_b = ptr(L.n2_w), ptr(L.n2_b), ptr(L.n1_w), ptr(L.n1_b)
        if cs is not None:
            a.cos_sin, a.max_pos = ptr(cs), max_pos
        a.positions, a.slots, a.q_out = ptr(pos), ptr(slots), ptr(q_out)
        a.k_pool, a.v_pool, a.num_blocks = ptr(kp), ptr(vp), nblk
        return a

    full = K.BLK_O | K.BLK_MLP | K.BLK_N1 | K.BLK_QKV
    ws = torch.zeros(K.block_workspace_bytes(args(full, h0)), dtype=torch.uint8, device=dev)
    tol = lambda got, want, what: _close(got, want, f"{family} H={H} m={m}: {what}")

    # o_proj alone: h += attn . Wo^T + b
    h = h0.clone()
    K.decode_block(args(K.BLK_O, h), ws)
    torch.cuda.synchronize()
    want_h = _np(h0) + _np(attn) @ L.Wo.T + _np(L.o_b)
    tol(_np(h), want_h, "o_proj residual")

    # MLP + norm1 (reads the h the previous launch left)
    h_mid = h.clone()
    K.decode_block(args(K.BLK_MLP | K.BLK_N1, h), ws)
    torch.cuda.synchronize()
    tol(_np(x2), _norm64(_np(h_mid), _np(L.n2_w), _np(L.n2_b) if L.n2_b is not None else 0, family), "norm2")
    pre = _np(x2) @ L.Wgu.T + _np(L.gu_b)
    if family == "gpt2":
        want_act = 0.5 * pre * (1 + np.tanh(0.7978845608028654 * (pre + 0.044715 * pre ** 3)))
    else:
        n_t = pre.shape[1] // 128
        gate = pre.reshape(m, n_t, 2, 64)[:, :, 0].reshape(m, -1)
        up = pre.reshape(m, n_t, 2, 64)[:, :, 1].reshape(m, -1)
        want_act = gate / (1 + np.exp(-gate)) * up
    tol(_np(act), want_act, "MLP activation")
    want_h2 = _np(h_mid) + _np(act) @ L.Wd.T + _np(L.d_b)
    tol(_np(h), want_h2, "down residual")
    tol(_np(x1), _norm64(_np(h), _np(L.n1_w), _np(L.n1_b) if L.n1_b is not None else 0, family), "norm1")

    # QKV with RoPE + KV append (reads the x1 the previous launch left; N1 off)
    K.decode_block(args(K.BLK_QKV, h), ws)
    torch.cuda.synchronize()
    qkv = _np(x1) @ L.Wqkv.T + _np(L.qkv_b)
    qkv = qkv.reshape(m, hq + 2 * hkv, D)
    if cs is not None:
        half = D // 2
        c = _np(cs)[_np(pos).astype(int)]
        cos, sin = np.concatenate([c[:, :half]] * 2, 1)[:, None], np.concatenate([c[:, half:]] * 2, 1)[:, None]
        rot = lambda x: x * cos + np.concatenate([-x[..., half:], x[..., :half]], -1) * sin
        qkv[:, :hq + hkv] = rot(qkv[:, :hq + hkv])
    tol(_np(q_out), qkv[:, :hq], "q (RoPE)")
    sl = slots.cpu().numpy()
    tol(_np(kp)[sl // 16, :, sl % 16], qkv[:, hq:hq + hkv], "K slots")
    tol(_np(vp)[sl // 16, :, sl % 16], qkv[:, hq + hkv:], "V slots")

    # all phases in one launch from the same start: the chained values above
    outs = {n: t.clone() for n, t in (("x2", x2), ("act", act), ("x1", x1), ("q", q_out), ("k", kp), ("v", vp))}
    h_all = h0.clone()
    K.decode_block(args(full, h_all), ws)
    torch.cuda.synchronize()
    tol(_np(h_all), _np(h), "one launch: residual")
    for n, t in (("x2", x2), ("act", act), ("x1", x1), ("q", q_out), ("k", kp), ("v", vp)):
        tol(_np(t), _np(outs[n]), f"one launch: {n}")
    # bit-reproducible: the same launch from the same inputs gives the same bits
    first = {n: t.clone() for n, t in (("h", h_all), ("x2", x2), ("act", act), ("x1", x1), ("q", q_out), ("k", kp))}
    h_again = h0.clone()
    K.decode_block(args(full, h_again), ws)
    torch.cuda.synchronize()
    for n, t in (("h", h_again), ("x2", x2), ("act", act), ("x1", x1), ("q", q_out), ("k", kp)):
        assert torch.equal(t, first[n]), f"{family} H={H} m={m}: {n} differs between two identical launches"
    code, info = _lib.device_error(torch.cuda.current_stream().cuda_stream)
    assert code == 0, (code, info)

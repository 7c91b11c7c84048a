"""CPU baseline of the decode step (test/bench infrastructure — the timed CPU "port").

The reference runs decode on CPU with torch as: every ``QuantizedLinear`` dequantizes its weight on each
call (``weight_int8.to(dtype) * scales``, ``microgen/backends/quantized.py:24-27``) and calls ``F.linear``;
the KV cache grows with ``torch.cat`` (``microgen/runtime/kv_cache.py:106-107``, and HF's ``DynamicCache``);
HF computes RMSNorm, RoPE and SDPA (``enable_gqa`` when no mask is given) over the grown cache. This module
restates one such Llama-family decode layer for a batch with the same torch CPU operations (fp32, torch's
intra-op threads), at the full model shape, so ``bench.py`` can time it on the host cores:
``measure_steps`` runs whole decode steps (the layer applied once per model layer, then the final norm +
lm_head + argmax); ``measure`` times single layers and the head on a bounded sample. It is checked
against the reference's own ``QuantizedPyTorchBackend.decode`` on the same cores by
``oracle/port_vs_reference_timing.py``.
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F


def _rms(h, w, eps):
    """HF ``LlamaRMSNorm`` in fp32."""
    return w * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps))


def _rand_codes(g, n, k):
    q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    s = torch.full((n, 1), 0.02 * 4 / 127, dtype=torch.float32)
    return q, s


def _qlinear(x, qs):
    """``QuantizedLinear.forward``: dequantize the whole weight, then ``F.linear``."""
    q, s = qs
    return F.linear(x, q.to(x.dtype) * s)


class LlamaLayerPort:
    """One decoder layer (RMSNorm, q/k/v, RoPE, cache append, GQA SDPA, o, RMSNorm, SwiGLU MLP)."""

    def __init__(self, hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps=1e-5, theta=500000.0, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.H, self.hq, self.hkv, self.D, self.I, self.B = hidden, heads, kv_heads, head_dim, inter, batch
        self.eps = eps
        self.wq = _rand_codes(g, heads * head_dim, hidden)
        self.wk = _rand_codes(g, kv_heads * head_dim, hidden)
        self.wv = _rand_codes(g, kv_heads * head_dim, hidden)
        self.wo = _rand_codes(g, hidden, heads * head_dim)
        self.wg = _rand_codes(g, inter, hidden)
        self.wu = _rand_codes(g, inter, hidden)
        self.wd = _rand_codes(g, hidden, inter)
        self.n1 = torch.ones(hidden)
        self.n2 = torch.ones(hidden)
        self.k = torch.randn((batch, kv_heads, ctx, head_dim), generator=g)
        self.v = torch.randn((batch, kv_heads, ctx, head_dim), generator=g)
        inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        ang = float(ctx) * inv
        self.cos = torch.cos(torch.cat([ang, ang]))
        self.sin = torch.sin(torch.cat([ang, ang]))

    def _rope(self, x):
        h = self.D // 2
        return x * self.cos + torch.cat([-x[..., h:], x[..., :h]], dim=-1) * self.sin

    @torch.no_grad()
    def step(self, h: torch.Tensor) -> torch.Tensor:
        B, D = self.B, self.D
        x = _rms(h, self.n1, self.eps)
        q = _qlinear(x, self.wq).view(B, 1, self.hq, D).transpose(1, 2)
        k = _qlinear(x, self.wk).view(B, 1, self.hkv, D).transpose(1, 2)
        v = _qlinear(x, self.wv).view(B, 1, self.hkv, D).transpose(1, 2)
        q, k = self._rope(q), self._rope(k)
        self.k = torch.cat([self.k, k], dim=2)   # the cache grows by concatenation along the sequence
        self.v = torch.cat([self.v, v], dim=2)
        att = F.scaled_dot_product_attention(q, self.k, self.v, enable_gqa=True)
        h = h + _qlinear(att.transpose(1, 2).reshape(B, self.hq * D), self.wo)
        x = _rms(h, self.n2, self.eps)
        h = h + _qlinear(F.silu(_qlinear(x, self.wg)) * _qlinear(x, self.wu), self.wd)
        # keep the cache length fixed across repeated samples
        self.k = self.k[:, :, 1:]
        self.v = self.v[:, :, 1:]
        return h


def _threads() -> int:
    return torch.get_num_threads()


def measure(hidden, heads, kv_heads, head_dim, inter, vocab, layers, batch, ctx, budget_s=20.0, eps=1e-5,
            theta=500000.0) -> dict:
    """Time the CPU port on a bounded sample; returns tokens/s for the whole step estimated
    as ``layers * t_layer + t_head`` and a description of the sample."""
    t_setup = time.perf_counter()
    layer = LlamaLayerPort(hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps, theta)
    g = torch.Generator().manual_seed(1)
    head = _rand_codes(g, vocab, hidden)
    h = torch.randn((batch, hidden), generator=g)
    layer.step(h)  # warm-up
    t_layers, n_layer = 0.0, 0
    start = time.perf_counter()
    with torch.no_grad():
        while n_layer < 2 or (time.perf_counter() - start < budget_s * 0.7 and n_layer < 64):
            t0 = time.perf_counter()
            h = layer.step(h)
            t_layers += time.perf_counter() - t0
            n_layer += 1
        t0 = time.perf_counter()
        logits = _qlinear(_rms(h, torch.ones(hidden), eps), head)
        _ = torch.argmax(logits, dim=-1)
        t_head = time.perf_counter() - t0
    t_layer = t_layers / n_layer
    step = layers * t_layer + t_head
    return {
        "tokens_per_s": batch / step,
        "step_s": step,
        "layer_s": t_layer,
        "head_s": t_head,
        "layers_timed": n_layer,
        "setup_s": start - t_setup,
        "threads": _threads(),
    }


def measure_steps(hidden, heads, kv_heads, head_dim, inter, vocab, layers, batch, ctx, budget_s=60.0,
                  max_steps=20, warmup=1, eps=1e-5, theta=500000.0) -> dict:
    """Time WHOLE decode steps of the CPU port: each step runs the decoder layer ``layers`` times (one
    layer's weights and cache, applied once per layer of the model: the same arithmetic and the same
    bytes streamed as ``layers`` distinct layers) and then the final norm + lm_head + argmax. Runs
    ``warmup`` untimed steps, then timed steps until ``budget_s`` is spent (at least one, at most
    ``max_steps``); returns the number of steps actually timed with the mean step time."""
    layer = LlamaLayerPort(hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps, theta)
    g = torch.Generator().manual_seed(1)
    head = _rand_codes(g, vocab, hidden)
    h0 = torch.randn((batch, hidden), generator=g)
    norm = torch.ones(hidden)

    @torch.no_grad()
    def step():
        h = h0
        for _ in range(layers):
            h = layer.step(h)
        return torch.argmax(_qlinear(_rms(h, norm, eps), head), dim=-1)

    for _ in range(warmup):
        step()
    times = []
    start = time.perf_counter()
    while not times or (len(times) < max_steps and time.perf_counter() - start < budget_s):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    step_s = sum(times) / len(times)
    return {"tokens_per_s": batch / step_s, "step_s": step_s, "steps": len(times), "warmup": warmup,
            "timed_s": sum(times), "threads": _threads()}

"""CPU baseline of the decode step (test/bench infrastructure — the timed CPU "port").

The reference runs decode on CPU as: every ``QuantizedLinear`` dequantizes its weight
on each call (``weight_int8.to(dtype) * scales``, ``microgen/backends/quantized.py:24-27``)
and calls ``F.linear``; ``KVCacheState.update`` grows the cache with ``torch.cat``
(``microgen/runtime/kv_cache.py:106-107``); HF computes SDPA over the grown cache.
This module restates one such Llama-family decode layer for a batch in numpy fp32
(multithreaded BLAS), at the full model shape, so ``bench.py`` can time a bounded
sample on the host cores: ``layer_seconds`` for one layer and ``head_seconds`` for the
final norm + lm_head; a whole step is ``layers * layer + head``.
"""

from __future__ import annotations

import os
import time

import numpy as np


def _rms(h, w, eps):
    return w * (h / np.sqrt(np.mean(h * h, axis=-1, keepdims=True) + eps))


def _rand_codes(rng, n, k):
    q = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    s = np.full((n,), 0.02 * 4 / 127, np.float32)
    return q, s


def _deq(q, s):
    return q.astype(np.float32) * s[:, None]


class LlamaLayerPort:
    """One decoder layer (RMSNorm, q/k/v, RoPE, cache append, GQA SDPA, o, RMSNorm, SwiGLU MLP)."""

    def __init__(self, hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps=1e-5, theta=500000.0, seed=0):
        rng = np.random.default_rng(seed)
        self.H, self.hq, self.hkv, self.D, self.I, self.B = hidden, heads, kv_heads, head_dim, inter, batch
        self.eps = eps
        self.wq = _rand_codes(rng, heads * head_dim, hidden)
        self.wk = _rand_codes(rng, kv_heads * head_dim, hidden)
        self.wv = _rand_codes(rng, kv_heads * head_dim, hidden)
        self.wo = _rand_codes(rng, hidden, heads * head_dim)
        self.wg = _rand_codes(rng, inter, hidden)
        self.wu = _rand_codes(rng, inter, hidden)
        self.wd = _rand_codes(rng, hidden, inter)
        self.n1 = np.ones(hidden, np.float32)
        self.n2 = np.ones(hidden, np.float32)
        self.k = rng.standard_normal((batch, kv_heads, ctx, head_dim), dtype=np.float32)
        self.v = rng.standard_normal((batch, kv_heads, ctx, head_dim), dtype=np.float32)
        inv = 1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)))
        ang = np.float32(ctx) * inv
        self.cos = np.cos(np.concatenate([ang, ang])).astype(np.float32)
        self.sin = np.sin(np.concatenate([ang, ang])).astype(np.float32)

    def _rope(self, x):
        h = self.D // 2
        return x * self.cos + np.concatenate([-x[..., h:], x[..., :h]], axis=-1) * self.sin

    def step(self, h: np.ndarray) -> np.ndarray:
        B, D = self.B, self.D
        x = _rms(h, self.n1, self.eps)
        q = (x @ _deq(*self.wq).T).reshape(B, self.hq, 1, D)
        k = (x @ _deq(*self.wk).T).reshape(B, self.hkv, 1, D)
        v = (x @ _deq(*self.wv).T).reshape(B, self.hkv, 1, D)
        q, k = self._rope(q), self._rope(k)
        self.k = np.concatenate([self.k, k], axis=2)   # KVCacheState.update: torch.cat along seq
        self.v = np.concatenate([self.v, v], axis=2)
        g = self.hq // self.hkv
        qg = q.reshape(B, self.hkv, g, D)
        sc = np.einsum("bhgd,bhtd->bhgt", qg, self.k) / np.float32(np.sqrt(D))
        sc = np.exp(sc - sc.max(-1, keepdims=True))
        sc /= sc.sum(-1, keepdims=True)
        att = np.einsum("bhgt,bhtd->bhgd", sc, self.v).reshape(B, self.hq * D)
        h = h + att @ _deq(*self.wo).T
        x = _rms(h, self.n2, self.eps)
        gt = x @ _deq(*self.wg).T
        up = x @ _deq(*self.wu).T
        h = h + ((gt / (1 + np.exp(-gt))) * up) @ _deq(*self.wd).T
        # keep the cache length fixed across repeated samples
        self.k = self.k[:, :, 1:]
        self.v = self.v[:, :, 1:]
        return h.astype(np.float32)


def measure(hidden, heads, kv_heads, head_dim, inter, vocab, layers, batch, ctx, budget_s=20.0, eps=1e-5,
            theta=500000.0) -> dict:
    """Time the CPU port on a bounded sample; returns tokens/s for the whole step estimated
    as ``layers * t_layer + t_head`` and a description of the sample."""
    t_setup = time.perf_counter()
    layer = LlamaLayerPort(hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps, theta)
    rng = np.random.default_rng(1)
    head = _rand_codes(rng, vocab, hidden)
    h = rng.standard_normal((batch, hidden), dtype=np.float32)
    layer.step(h)  # warm-up
    t_layers, n_layer = 0.0, 0
    start = time.perf_counter()
    while n_layer < 2 or (time.perf_counter() - start < budget_s * 0.7 and n_layer < 64):
        t0 = time.perf_counter()
        h = layer.step(h)
        t_layers += time.perf_counter() - t0
        n_layer += 1
    t0 = time.perf_counter()
    logits = _rms(h, np.ones(hidden, np.float32), eps) @ _deq(*head).T
    _ = np.argmax(logits, axis=-1)
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
        "threads": os.cpu_count() or 1,
    }


def measure_steps(hidden, heads, kv_heads, head_dim, inter, vocab, layers, batch, ctx, budget_s=60.0,
                  max_steps=20, warmup=1, eps=1e-5, theta=500000.0) -> dict:
    """Time WHOLE decode steps of the CPU port: each step runs the decoder layer ``layers`` times (one
    layer's weights and cache, applied once per layer of the model: the same arithmetic and the same
    bytes streamed as ``layers`` distinct layers) and then the final norm + lm_head + argmax. Runs
    ``warmup`` untimed steps, then timed steps until ``budget_s`` is spent (at least one, at most
    ``max_steps``); returns the number of steps actually timed with the mean step time."""
    layer = LlamaLayerPort(hidden, heads, kv_heads, head_dim, inter, batch, ctx, eps, theta)
    rng = np.random.default_rng(1)
    head = _rand_codes(rng, vocab, hidden)
    h0 = rng.standard_normal((batch, hidden), dtype=np.float32)

    def step():
        h = h0
        for _ in range(layers):
            h = layer.step(h)
        logits = _rms(h, np.ones(hidden, np.float32), eps) @ _deq(*head).T
        return np.argmax(logits, axis=-1)

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
            "timed_s": sum(times), "threads": os.cpu_count() or 1}

"""Oracle: decode attention over a paged KV pool (test infrastructure).

The reference never stores KV in pages: ``KVCacheState.update``
(``microgen/runtime/kv_cache.py:76-127``) grows a contiguous ``[B, Hkv, L, D]``
tensor with ``torch.cat`` and HF's ``sdpa_attention_forward``
(transformers 5.5.0 ``integrations/sdpa_attention.py:40-92``) computes
``softmax(q·Kᵀ·scale)·V`` with ``enable_gqa`` (query head ``g`` reads KV head
``g // (Hq/Hkv)``).  The block allocator
(``microgen/runtime/paged_kv.py:34-110``) only hands out block ids.

This oracle gathers the contiguous cache back out of a paged pool through the
block table (pool layout ``[num_blocks, Hkv, BLOCK, D]``, token ``t`` of a
sequence at block ``table[t // BLOCK]``, row ``t % BLOCK``) and then computes
exactly the SDPA decode step, in float64.
"""

from __future__ import annotations

import numpy as np

BLOCK = 16  # PhysicalBlock.block_size default, paged_kv.py:10


def gather_contiguous(pool: np.ndarray, table: np.ndarray, ctx_len: int) -> np.ndarray:
    """[Hkv, ctx_len, D] view of one sequence's cache out of a paged pool."""
    nblk = (ctx_len + BLOCK - 1) // BLOCK
    blocks = pool[np.asarray(table[:nblk], dtype=np.int64)]  # [nblk, Hkv, BLOCK, D]
    hkv, d = pool.shape[1], pool.shape[3]
    return blocks.transpose(1, 0, 2, 3).reshape(hkv, nblk * BLOCK, d)[:, :ctx_len]


def sdpa_decode(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """One query token per head: q [Hq, D], k/v [Hkv, L, D] -> [Hq, D] (float64)."""
    hq, hkv = q.shape[0], k.shape[0]
    group = hq // hkv
    out = np.empty((hq, q.shape[1]), dtype=np.float64)
    for g in range(hq):
        kh = k[g // group].astype(np.float64)
        vh = v[g // group].astype(np.float64)
        s = kh @ q[g].astype(np.float64) * scale
        if s.size == 0:
            out[g] = 0.0
            continue
        p = np.exp(s - s.max())
        out[g] = (p / p.sum()) @ vh
    return out


def paged_decode_attention(q, k_pool, v_pool, block_tables, ctx_lens, scale: float) -> np.ndarray:
    """q [B, Hq, D]; pools [num_blocks, Hkv, BLOCK, D]; tables [B, max_blocks];
    ctx_lens [B] -> [B, Hq, D] float64."""
    b = q.shape[0]
    out = np.empty(q.shape, dtype=np.float64)
    for i in range(b):
        k = gather_contiguous(k_pool, block_tables[i], int(ctx_lens[i]))
        v = gather_contiguous(v_pool, block_tables[i], int(ctx_lens[i]))
        out[i] = sdpa_decode(q[i], k, v, scale)
    return out


def quantize_kv_vectors(x):
    """Per-vector INT8 of ``KVCacheState(quantize_kv=True)`` (``microgen/runtime/kv_cache.py:30-35``,
    ``_quantize_tensor``): over the last axis, ``s = max(max|x| / 127, 1e-8)`` and
    ``code = clamp(round_half_even(x / s), -128, 127)``, in float32 as the reference computes it.
    Returns (int8 codes shaped like x, float32 scales with the last axis dropped)."""
    x = np.asarray(x, dtype=np.float32)
    s = np.maximum(np.abs(x).max(axis=-1, keepdims=True) / np.float32(127.0), np.float32(1e-8))
    s = s.astype(np.float32)
    q = np.clip(np.rint(x / s), -128, 127).astype(np.int8)
    return q, s[..., 0]


def paged_decode_attention_kv8(q, k_pool, v_pool, k_scale, v_scale, block_tables, ctx_lens,
                               scale: float) -> np.ndarray:
    """``paged_decode_attention`` over INT8 pools: K and V are the codes times their per-vector scales
    (``_dequantize_tensor``, ``kv_cache.py:38-40``), evaluated in float64. Pools int8
    ``[num_blocks, Hkv, BLOCK, D]``, scales ``[num_blocks, Hkv, BLOCK]``."""
    k = k_pool.astype(np.float64) * k_scale.astype(np.float64)[..., None]
    v = v_pool.astype(np.float64) * v_scale.astype(np.float64)[..., None]
    return paged_decode_attention(q, k, v, block_tables, ctx_lens, scale)

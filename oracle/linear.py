"""Oracle: INT8 weight-only linear and its tensor-parallel splits (test infrastructure).

* ``i8_linear`` restates ``QuantizedLinear.forward`` (``microgen/backends/quantized.py:24-27``):
  ``y = x · (q·s)ᵀ + b`` with the fp32 dequantized weight; accumulated here in
  float64 so it serves as the "truth" a bf16-activation kernel is measured against.
* ``column_shards`` / ``row_shards`` restate the split rules of
  ``ColumnParallelLinear`` (``parallel.py:12-37``: out-features split in
  ``N // world`` slices, the last rank takes the remainder) and
  ``RowParallelLinear`` (``parallel.py:40-81``: in-features split likewise, the
  partial outputs summed — the all-reduce — and the bias added once).
"""

from __future__ import annotations

import numpy as np

from .quant import dequantize_rows


def i8_linear(x: np.ndarray, q: np.ndarray, scales: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """fp64 result of x[M,K] · dequant(q,s)[N,K]ᵀ (+ bias[N])."""
    w = dequantize_rows(q, scales).astype(np.float64)
    y = np.asarray(x, dtype=np.float64) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64)
    return y


def shard_bounds(total: int, world: int) -> list[tuple[int, int]]:
    """[start, end) per rank: ``total // world`` each, the last rank takes the rest
    (``parallel.py:19-20`` and ``:47-48``)."""
    per = total // world
    return [(r * per, (r + 1) * per if r < world - 1 else total) for r in range(world)]


def column_shards(q: np.ndarray, scales: np.ndarray, bias, world: int):
    """Row slices of the FULL-matrix codes/scales: column-parallel shards."""
    out = []
    for a, b in shard_bounds(q.shape[0], world):
        out.append((q[a:b], scales[a:b], None if bias is None else bias[a:b]))
    return out


def row_shards(q: np.ndarray, scales: np.ndarray, world: int):
    """Column slices of the FULL-matrix codes; scales are per output row and so
    replicated on every rank."""
    return [(q[:, a:b], scales) for a, b in shard_bounds(q.shape[1], world)]


def column_parallel_linear(x, q, scales, bias, world: int) -> np.ndarray:
    """``ColumnParallelLinear.forward``: per-shard linear, concatenated (``parallel.py:34-37``)."""
    return np.concatenate([i8_linear(x, qs, ss, bs) for qs, ss, bs in column_shards(q, scales, bias, world)], axis=-1)


def row_parallel_linear(x, q, scales, bias, world: int) -> np.ndarray:
    """``RowParallelLinear.forward``: per-shard partial, summed, bias once (``parallel.py:65-81``)."""
    parts = []
    for (a, b), (qs, ss) in zip(shard_bounds(q.shape[1], world), row_shards(q, scales, world)):
        parts.append(i8_linear(np.asarray(x)[..., a:b], qs, ss))
    y = sum(parts)
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float64)
    return y

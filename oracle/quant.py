"""Oracle: symmetric per-output-channel INT8 quantization (test infrastructure).

Restates ``quantize_linear_layer_per_channel`` of the reference,
``microgen/backends/quantized.py:30-39``:

    max_vals = max(|W|, dim=-1, keepdim=True)          # fp32, exact
    scales   = clamp(max_vals / 127.0, min=1e-8)       # fp32 IEEE division
    q        = clamp(round(W / scales), -128, 127).int8  # round half to even

numpy float32 division is IEEE-754 correctly rounded, like torch's, and
``np.rint`` rounds half to even like ``torch.round``; the result is therefore
bit-identical to the reference (pinned against its outputs in
``tests/golden/quant_*.npz``).
"""

from __future__ import annotations

import numpy as np

SCALE_FLOOR = np.float32(1e-8)  # quantized.py:36, the Python float cast to fp32


def quantize_rows_i8(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Return (codes int8 [N,K], scales fp32 [N]) for an fp32 weight [N,K]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("weight must be 2-D [out_features, in_features]")
    maxv = np.max(np.abs(w), axis=-1, keepdims=True) if w.shape[1] else np.zeros((w.shape[0], 1), np.float32)
    scales = np.maximum(maxv / np.float32(127.0), SCALE_FLOOR).astype(np.float32)
    q = np.clip(np.rint(w / scales), -128, 127).astype(np.int8)
    return q, scales.reshape(-1)


def dequantize_rows(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 weight ``q.to(fp32) * scales`` as QuantizedLinear.forward builds it
    (``quantized.py:26``)."""
    return q.astype(np.float32) * scales.reshape(-1, 1).astype(np.float32)

"""INT8 per-channel weight quantization on the B200 (mirror of ``microgen/backends/quantized.py``).

* ``quantize_linear_layer_per_channel`` — same contract as the reference
  (``quantized.py:30-39``), computed by the bit-exact device kernel.
* ``QuantizedLinear`` — same buffers (``weight_int8`` [N,K], ``scales`` [N,1], ``bias``);
  ``forward`` runs the INT8 tensor-core linear instead of materialising the fp weight
  (``quantized.py:24-27``). Activations enter the kernel as bf16; the output has x's dtype.
* ``quantize_model`` — the reference's recursive ``nn.Linear`` swap (``quantized.py:59-73``).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import kernels as K


class QuantizedLinear(nn.Module):
    """INT8 weight-only linear: y = x · (q·s)ᵀ + b on the tensor cores."""

    def __init__(self, weight_int8: torch.Tensor, scales: torch.Tensor, bias: Optional[nn.Parameter] = None) -> None:
        super().__init__()
        self.register_buffer("weight_int8", weight_int8)
        self.register_buffer("scales", scales)
        self.bias = bias if bias is not None else None

    @property
    def in_features(self) -> int:
        return self.weight_int8.shape[1]

    @property
    def out_features(self) -> int:
        return self.weight_int8.shape[0]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        bias = None if self.bias is None else self.bias.detach().to(torch.float32).contiguous()
        y = K.i8_linear(x2, self.weight_int8, self.scales.reshape(-1), bias, epilogue=K.EPI_STORE_F32)
        return y.to(x.dtype).reshape(*shape[:-1], self.out_features)


def quantize_weight(weight: torch.Tensor, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(int8 codes [N,K], fp32 scales [N]) of a weight, on ``device`` (default: current CUDA device)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return K.quantize_rows_i8(weight.detach().to(device=dev, dtype=torch.float32).contiguous())


def quantize_linear_layer_per_channel(module: nn.Linear, device=None) -> QuantizedLinear:
    """Quantize an ``nn.Linear`` to INT8 per output channel (bit-exact with the reference)."""
    q, s = quantize_weight(module.weight, device)
    bias = None
    if module.bias is not None:
        bias = nn.Parameter(module.bias.detach().to(device=q.device, dtype=torch.float32), requires_grad=False)
    return QuantizedLinear(weight_int8=q, scales=s.reshape(-1, 1), bias=bias)


def quantize_model(model: nn.Module, device=None) -> nn.Module:
    """Swap every ``nn.Linear`` of ``model`` for a ``QuantizedLinear`` (recursive ``setattr`` walk)."""
    for name, child in list(model.named_children()):
        if isinstance(child, nn.Linear):
            setattr(model, name, quantize_linear_layer_per_channel(child, device))
        else:
            quantize_model(child, device)
    return model

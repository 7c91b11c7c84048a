"""Tensor-parallel INT8 linears (mirror of ``microgen/backends/parallel.py:12-81``) and the module walk
that installs them (``parallel.py:108-131``).

Split rules follow the reference: out-features (column) or in-features (row) split in
``N // world`` slices, the last rank taking the remainder; the row-parallel bias is
added once, after the reduction. Codes and scales come from quantizing the FULL
weight, then slicing (column: rows and scales; row: columns, scales replicated).

Two modes:
* ``group=None`` — every shard lives in this process and the forward loops over
  them (the reference's single-process simulation), each shard on the INT8 kernel;
* ``group`` given — SPMD, one process per GPU: this rank holds its shard only;
  the column output is all-gathered, the row partial all-reduced (NCCL).
The decode engine does not go through these modules: it keeps column outputs
sharded (head-local attention) and fuses the row reduction into the residual
update; these modules are the module-level drop-in surface.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import kernels as K
from .quantized import quantize_weight


def shard_bounds(total: int, world: int) -> list[tuple[int, int]]:
    """[start, end) per rank; the last rank takes the remainder (``parallel.py:19-20``, ``:47-48``)."""
    per = total // world
    return [(r * per, (r + 1) * per if r < world - 1 else total) for r in range(world)]


class _TPBase(nn.Module):
    def __init__(self, world_size: int, group) -> None:
        super().__init__()
        self.world_size = world_size
        self.group = group
        self.rank = dist.get_rank(group) if group is not None else None

    def _ranks(self):
        return range(self.world_size) if self.group is None else [self.rank]


class ColumnParallelLinear(_TPBase):
    """INT8 linear sharded along out-features; forward = per-shard linear + concat."""

    def __init__(self, full_weight: torch.Tensor, full_bias: Optional[torch.Tensor], world_size: int,
                 group=None, device=None) -> None:
        super().__init__(world_size, group)
        q, s = quantize_weight(full_weight, device)
        self.bounds = shard_bounds(q.shape[0], world_size)
        self.shards = nn.ModuleList()
        for r in self._ranks():
            a, b = self.bounds[r]
            m = nn.Module()
            m.register_buffer("weight_int8", q[a:b].contiguous())
            m.register_buffer("scales", s[a:b].contiguous())
            m.register_buffer("bias", None if full_bias is None else
                              full_bias.detach()[a:b].to(device=q.device, dtype=torch.float32).contiguous())
            self.shards.append(m)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        outs = [K.i8_linear(x2, m.weight_int8, m.scales, m.bias, epilogue=K.EPI_STORE_F32) for m in self.shards]
        if self.group is not None:
            # pad every shard to the widest (the last rank may hold a remainder), gather, trim
            sizes = [b - a for a, b in self.bounds]
            widest = max(sizes)
            local = torch.zeros((x2.shape[0], widest), dtype=torch.float32, device=x2.device)
            local[:, : sizes[self.rank]] = outs[0]
            full = [torch.empty_like(local) for _ in range(self.world_size)]
            dist.all_gather(full, local, group=self.group)
            outs = [full[r][:, : sizes[r]] for r in range(self.world_size)]
        y = torch.cat(outs, dim=-1)
        return y.to(x.dtype).reshape(*shape[:-1], y.shape[-1])


class RowParallelLinear(_TPBase):
    """INT8 linear sharded along in-features; forward = per-shard partial, sum (all-reduce), bias once."""

    def __init__(self, full_weight: torch.Tensor, full_bias: Optional[torch.Tensor], world_size: int,
                 group=None, device=None) -> None:
        super().__init__(world_size, group)
        q, s = quantize_weight(full_weight, device)
        self.bounds = shard_bounds(q.shape[1], world_size)
        self.shards = nn.ModuleList()
        for r in self._ranks():
            a, b = self.bounds[r]
            m = nn.Module()
            m.register_buffer("weight_int8", q[:, a:b].contiguous())
            m.register_buffer("scales", s)
            self.shards.append(m)
        self.bias = None
        if full_bias is not None:
            self.bias = nn.Parameter(full_bias.detach().to(device=q.device, dtype=torch.float32), requires_grad=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y = None
        for r, m in zip(self._ranks(), self.shards):
            a, b = self.bounds[r]
            xs = x2[:, a:b].to(torch.bfloat16).contiguous()
            if xs.shape[1] % 16:
                raise ValueError(f"row shard width {xs.shape[1]} must be a multiple of 16")
            part = K.i8_linear(xs, m.weight_int8, m.scales, None, epilogue=K.EPI_STORE_F32)
            y = part if y is None else y + part
        if self.group is not None:
            dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype).reshape(*shape[:-1], y.shape[-1])


# Child-name patterns of the reference's TP walk (``parallel.py:113-128``): column-parallel projections,
# then row-parallel ones. ``lm_head`` matches neither and stays as it is (the reference leaves it unsharded).
COLUMN_NAMES = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "fc1", "c_attn")
ROW_NAMES = ("o_proj", "down_proj", "fc2", "c_proj")


def apply_tensor_parallelism(model: nn.Module, world_size: int, group=None, device=None) -> nn.Module:
    """Install INT8 ``ColumnParallelLinear`` / ``RowParallelLinear`` modules in place of ``model``'s
    ``nn.Linear`` children, classified by child name as the reference's
    ``TensorParallelPyTorchBackend.apply_tensor_parallelism`` does (``parallel.py:108-131``): a name containing
    one of ``COLUMN_NAMES`` becomes column-parallel, else one containing one of ``ROW_NAMES`` becomes
    row-parallel, others are left alone; non-Linear children are walked recursively. Each replacement
    quantizes the FULL weight and keeps its shards (all of them with ``group=None``, this rank's with a
    process group). Returns ``model``."""
    if world_size < 1:
        raise ValueError("world_size must be >= 1")

    def walk(module: nn.Module) -> None:
        for name, child in list(module.named_children()):
            if isinstance(child, nn.Linear):
                low = name.lower()
                bias = child.bias.data if child.bias is not None else None
                if any(p in low for p in COLUMN_NAMES):
                    setattr(module, name, ColumnParallelLinear(child.weight.data, bias, world_size, group, device))
                elif any(p in low for p in ROW_NAMES):
                    setattr(module, name, RowParallelLinear(child.weight.data, bias, world_size, group, device))
            else:
                walk(child)

    walk(model)
    return model

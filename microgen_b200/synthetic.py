"""Seeded random-init weights of a model shape, generated on the device.

The workloads use random-init weights (every Linear / Embedding weight N(0, 0.02),
biases 0, norm weights 1). ``SyntheticState`` is a lazy mapping keyed by HF
parameter names: each matrix is drawn on the device when the loader asks for it
(so a 3B-parameter model never sits in fp32 all at once), from a generator seeded
by (seed, parameter index).
"""

from __future__ import annotations

from collections.abc import Mapping

import torch

from .model_spec import ModelSpec


def param_shapes(s: ModelSpec) -> dict:
    D = s.head_dim
    out = {}
    if s.family == "gpt2":
        out["transformer.wte.weight"] = (s.vocab, s.hidden)
        out["transformer.wpe.weight"] = (s.max_pos, s.hidden)
        for i in range(s.layers):
            p = f"transformer.h.{i}."
            out[p + "ln_1.weight"] = out[p + "ln_1.bias"] = (s.hidden,)
            out[p + "attn.c_attn.weight"] = (s.hidden, 3 * s.hidden)
            out[p + "attn.c_attn.bias"] = (3 * s.hidden,)
            out[p + "attn.c_proj.weight"] = (s.hidden, s.hidden)
            out[p + "attn.c_proj.bias"] = (s.hidden,)
            out[p + "ln_2.weight"] = out[p + "ln_2.bias"] = (s.hidden,)
            out[p + "mlp.c_fc.weight"] = (s.hidden, s.inter)
            out[p + "mlp.c_fc.bias"] = (s.inter,)
            out[p + "mlp.c_proj.weight"] = (s.inter, s.hidden)
            out[p + "mlp.c_proj.bias"] = (s.hidden,)
        out["transformer.ln_f.weight"] = out["transformer.ln_f.bias"] = (s.hidden,)
        return out
    out["model.embed_tokens.weight"] = (s.vocab, s.hidden)
    for i in range(s.layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = (s.hidden,)
        out[p + "self_attn.q_proj.weight"] = (s.heads * D, s.hidden)
        out[p + "self_attn.k_proj.weight"] = (s.kv_heads * D, s.hidden)
        out[p + "self_attn.v_proj.weight"] = (s.kv_heads * D, s.hidden)
        if s.qkv_bias:
            out[p + "self_attn.q_proj.bias"] = (s.heads * D,)
            out[p + "self_attn.k_proj.bias"] = (s.kv_heads * D,)
            out[p + "self_attn.v_proj.bias"] = (s.kv_heads * D,)
        out[p + "self_attn.o_proj.weight"] = (s.hidden, s.heads * D)
        out[p + "post_attention_layernorm.weight"] = (s.hidden,)
        out[p + "mlp.gate_proj.weight"] = (s.inter, s.hidden)
        out[p + "mlp.up_proj.weight"] = (s.inter, s.hidden)
        out[p + "mlp.down_proj.weight"] = (s.hidden, s.inter)
    out["model.norm.weight"] = (s.hidden,)
    if not s.tie:
        out["lm_head.weight"] = (s.vocab, s.hidden)
    return out


class SyntheticState(Mapping):
    """Lazy {name: fp32 tensor on ``device``}: N(0, 0.02) weights, zero biases, unit norms."""

    def __init__(self, spec: ModelSpec, seed: int = 0, device="cuda") -> None:
        self.spec, self.seed, self.device = spec, seed, torch.device(device)
        self.shapes = param_shapes(spec)
        self.index = {k: i for i, k in enumerate(self.shapes)}

    def __getitem__(self, name: str) -> torch.Tensor:
        shape = self.shapes[name]
        leaf = name.rsplit(".", 1)[0].rsplit(".", 1)[-1]
        if name.endswith("bias"):
            return torch.zeros(shape, dtype=torch.float32, device=self.device)
        if "norm" in leaf or leaf.startswith("ln_"):
            return torch.ones(shape, dtype=torch.float32, device=self.device)
        g = torch.Generator(device=self.device)
        g.manual_seed(self.seed * 1_000_003 + self.index[name])
        return torch.randn(shape, generator=g, dtype=torch.float32, device=self.device).mul_(0.02)

    def __contains__(self, name) -> bool:
        return name in self.shapes

    def __iter__(self):
        return iter(self.shapes)

    def __len__(self) -> int:
        return len(self.shapes)

"""Seeded random-init HF models shared by the golden generator and the tests.

Weights are drawn from numpy's PCG64 (platform independent), so the build
container that produced the golden fixtures and any GPU box rebuild identical
models: every Linear / Conv1D / Embedding weight N(0, 0.02) in fp32, biases 0,
norm weights 1 (the HF ``_init_weights`` recipe with a portable generator).
"""

from __future__ import annotations

import numpy as np
import torch

from microgen_b200.model_spec import hf_config

# Small shapes of the three families, sized so the CPU reference finishes in seconds.
TINY = {
    "llama": dict(family="llama", hidden=128, layers=2, heads=4, kv_heads=2, head_dim=32, inter=256,
                  vocab=512, eps=1e-5, rope_theta=500000.0),
    "qwen2": dict(family="qwen2", hidden=128, layers=2, heads=4, kv_heads=2, head_dim=32, inter=192,
                  vocab=512, eps=1e-6, rope_theta=1000000.0, tie=True, qkv_bias=True),
    "gpt2": dict(family="gpt2", hidden=128, layers=2, heads=4, kv_heads=4, head_dim=32, inter=512,
                 vocab=512, eps=1e-5, max_pos=256, tie=True, qkv_bias=True, mlp_bias=True),
}


def _seeded_params(model: torch.nn.Module, seed: int):
    """(name, numpy fp32 value) of every parameter in ``named_parameters`` order, drawn from one PCG64."""
    rng = np.random.default_rng(seed)
    for name, p in model.named_parameters():
        leaf = name.rsplit(".", 1)[0].rsplit(".", 1)[-1]
        if name.endswith("bias"):
            a = np.zeros(p.shape, np.float32)
        elif "norm" in leaf or leaf.startswith("ln_"):
            a = np.ones(p.shape, np.float32)
        else:
            a = rng.standard_normal(p.shape, dtype=np.float32)
            a *= np.float32(0.02)
        yield name, a


def seeded_state(model: torch.nn.Module, seed: int) -> dict:
    return dict(_seeded_params(model, seed))


def seeded_model(shape: dict, seed: int = 0):
    """HF model of ``shape`` (fp32, eval) with the seeded weights, filled one parameter at a time
    (no second copy of the weights is held: full-size shapes fit in host memory)."""
    from transformers import AutoModelForCausalLM
    cfg = hf_config(shape)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = AutoModelForCausalLM.from_config(cfg)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name, a in _seeded_params(model, seed):
            params[name].copy_(torch.from_numpy(a))
    return model.eval()


def seeded_state_for_shape(shape: dict, seed: int = 0) -> tuple[object, dict]:
    """(HF config, {parameter name: fp32 CPU tensor}) with exactly the values ``seeded_model`` holds,
    without building the HF model's weights (the parameter order comes from a meta-device model)."""
    from transformers import AutoModelForCausalLM
    cfg = hf_config(shape)
    cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg)
    return cfg, {name: torch.from_numpy(a) for name, a in _seeded_params(model, seed)}


def make_hf_model(shape: dict, seed: int = 0):
    """(HF model in fp32 eval mode, numpy state dict keyed by parameter name)."""
    from transformers import AutoModelForCausalLM
    cfg = hf_config(shape)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = AutoModelForCausalLM.from_config(cfg)
    state = seeded_state(model, seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            p.copy_(torch.from_numpy(state[name]))
    model.eval()
    full = {k: v.detach().numpy().copy() for k, v in model.state_dict().items()}
    return model, full


def prompt_ids(vocab: int, n: int, seed: int) -> list[int]:
    rng = np.random.default_rng(1000 + seed)
    return [int(t) for t in rng.integers(0, vocab, size=n)]

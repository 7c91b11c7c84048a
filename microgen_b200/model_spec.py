"""Model shapes on the decode path and their HF configurations.

The reference runs HF transformers models (``microgen/backends/pytorch.py:73-88``);
the backend here reads the same HF configuration and parameters. ``ModelSpec``
is the subset of a config the decode step needs. ``hf_config`` builds the HF
config of a named shape (Llama-3.2-3B, Qwen2.5-0.5B, GPT-2-small, or a small
variant of one of them for tests).
"""

from __future__ import annotations

from dataclasses import dataclass, asdict


@dataclass(frozen=True)
class ModelSpec:
    family: str              # "llama" | "qwen2" | "gpt2"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    rope_theta: float = 10000.0
    max_pos: int = 0         # GPT-2 learned positions
    tie: bool = False
    qkv_bias: bool = False   # Qwen2 q/k/v, GPT-2 everywhere
    mlp_bias: bool = False   # GPT-2

    def as_dict(self) -> dict:
        return asdict(self)


# Shapes named by the workloads (random-init, N(0, 0.02)).
LLAMA_3B = dict(family="llama", hidden=3072, layers=28, heads=24, kv_heads=8, head_dim=128, inter=8192,
                vocab=128256, eps=1e-5, rope_theta=500000.0)
QWEN_05B = dict(family="qwen2", hidden=896, layers=24, heads=14, kv_heads=2, head_dim=64, inter=4864,
                vocab=151936, eps=1e-6, rope_theta=1000000.0, tie=True, qkv_bias=True)
GPT2_SMALL = dict(family="gpt2", hidden=768, layers=12, heads=12, kv_heads=12, head_dim=64, inter=3072,
                  vocab=50257, eps=1e-5, max_pos=1024, tie=True, qkv_bias=True, mlp_bias=True)


def spec_from_hf_config(cfg) -> ModelSpec:
    """ModelSpec of a ``LlamaConfig`` / ``Qwen2Config`` / ``GPT2Config``."""
    mt = cfg.model_type
    if mt in ("llama", "qwen2"):
        heads = cfg.num_attention_heads
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // heads
        rp = getattr(cfg, "rope_parameters", None) or {}
        theta = float(rp.get("rope_theta", getattr(cfg, "rope_theta", 10000.0)))
        rtype = rp.get("rope_type", "default")
        if rtype not in ("default", None):
            raise ValueError(f"rope_type {rtype!r} is not supported by the decode kernels")
        return ModelSpec(family=mt, hidden=cfg.hidden_size, layers=cfg.num_hidden_layers, heads=heads,
                         kv_heads=cfg.num_key_value_heads, head_dim=head_dim, inter=cfg.intermediate_size,
                         vocab=cfg.vocab_size, eps=float(cfg.rms_norm_eps), rope_theta=theta,
                         tie=bool(getattr(cfg, "tie_word_embeddings", False)),
                         qkv_bias=(mt == "qwen2") or bool(getattr(cfg, "attention_bias", False)),
                         mlp_bias=bool(getattr(cfg, "mlp_bias", False)))
    if mt == "gpt2":
        inter = cfg.n_inner or 4 * cfg.n_embd
        return ModelSpec(family="gpt2", hidden=cfg.n_embd, layers=cfg.n_layer, heads=cfg.n_head,
                         kv_heads=cfg.n_head, head_dim=cfg.n_embd // cfg.n_head, inter=inter,
                         vocab=cfg.vocab_size, eps=float(cfg.layer_norm_epsilon), max_pos=cfg.n_positions,
                         tie=True, qkv_bias=True, mlp_bias=True)
    raise ValueError(f"model_type {mt!r} is not on the decode path (llama, qwen2, gpt2)")


def hf_config(shape: dict):
    """HF config object for a shape dict (keys of ModelSpec)."""
    s = dict(shape)
    fam = s["family"]
    if fam == "llama":
        from transformers import LlamaConfig
        return LlamaConfig(hidden_size=s["hidden"], intermediate_size=s["inter"], num_hidden_layers=s["layers"],
                           num_attention_heads=s["heads"], num_key_value_heads=s["kv_heads"],
                           head_dim=s["head_dim"], vocab_size=s["vocab"], rms_norm_eps=s["eps"],
                           rope_theta=s["rope_theta"], tie_word_embeddings=s.get("tie", False),
                           max_position_embeddings=131072)
    if fam == "qwen2":
        from transformers import Qwen2Config
        return Qwen2Config(hidden_size=s["hidden"], intermediate_size=s["inter"], num_hidden_layers=s["layers"],
                           num_attention_heads=s["heads"], num_key_value_heads=s["kv_heads"],
                           vocab_size=s["vocab"], rms_norm_eps=s["eps"], rope_theta=s["rope_theta"],
                           tie_word_embeddings=s.get("tie", True), max_position_embeddings=32768,
                           use_sliding_window=False)
    if fam == "gpt2":
        from transformers import GPT2Config
        return GPT2Config(n_embd=s["hidden"], n_layer=s["layers"], n_head=s["heads"], n_inner=s["inter"],
                          vocab_size=s["vocab"], n_positions=s["max_pos"], layer_norm_epsilon=s["eps"],
                          activation_function="gelu_new", resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)
    raise ValueError(fam)

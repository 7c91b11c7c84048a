"""Oracle: one decode step of the model families on the path (test infrastructure).

Restates, in numpy, the forward the reference runs inside ``backend.decode``
(``microgen/backends/pytorch.py:118-142``) for HF transformers 5.5.0 models, with
every projection replaced by the reference's INT8 ``QuantizedLinear``
(``microgen/backends/quantized.py:24-39``):

* Llama / Qwen2 (``modeling_llama.py`` / ``modeling_qwen2.py``): RMSNorm
  (fp32, ``w * h * rsqrt(mean(h²) + eps)``), q/k/v projections (Qwen2 with bias),
  default RoPE (``inv_freq = 1 / theta^(2i/D)``, rotate-half), GQA SDPA,
  o_proj, RMSNorm, ``down(silu(gate(x)) * up(x))``, final norm, lm_head.
* GPT-2 (``modeling_gpt2.py``): token + learned position embeddings, LayerNorm,
  ``c_attn`` (Conv1D, weight stored ``[in, out]``), MHA SDPA, ``c_proj``,
  LayerNorm, ``c_fc`` → gelu_new → ``mlp.c_proj``, ``ln_f``, tied lm_head.
  The reference's quantizer skips Conv1D (it is not an ``nn.Linear``); the
  oracle quantizes ``Conv1D.weight.T`` with the same per-channel formula.

Weights are a dict of numpy fp32 arrays keyed by the HF parameter names.
The state per sequence is a contiguous per-layer K/V list, like ``KVCacheState``.
Everything is computed in float64 from the fp32 masters and the int8 codes.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .quant import quantize_rows_i8, dequantize_rows


@dataclass
class Spec:
    family: str            # "llama" | "qwen2" | "gpt2"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    rope_theta: float = 10000.0
    max_pos: int = 0
    tie: bool = False


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """``1 / theta ** (arange(0, D, 2) / D)`` in fp32 (``modeling_rope_utils`` default rope)."""
    e = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    return (np.float32(1.0) / (np.float32(theta) ** e)).astype(np.float32)


def rope_cos_sin(pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    freqs = (np.float32(pos) * rope_inv_freq(head_dim, theta)).astype(np.float32)  # fp32 product, as HF
    emb = np.concatenate([freqs, freqs]).astype(np.float64)
    return np.cos(emb), np.sin(emb)


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def rms_norm(h, w, eps):
    var = np.mean(h * h, axis=-1, keepdims=True)
    return w * (h / np.sqrt(var + eps))


def layer_norm(h, w, b, eps):
    mu = np.mean(h, axis=-1, keepdims=True)
    var = np.mean((h - mu) ** 2, axis=-1, keepdims=True)
    return (h - mu) / np.sqrt(var + eps) * w + b


def gelu_new(x):
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def silu(x):
    return x / (1.0 + np.exp(-x))


@dataclass
class QLinear:
    w: np.ndarray          # dequantized fp32 weight [N, K] as float64
    b: np.ndarray | None

    def __call__(self, x):
        y = x @ self.w.T
        return y if self.b is None else y + self.b


def _qlin(w_out_in: np.ndarray, b=None) -> QLinear:
    q, s = quantize_rows_i8(w_out_in)
    return QLinear(dequantize_rows(q, s).astype(np.float64), None if b is None else b.astype(np.float64))


@dataclass
class OracleModel:
    spec: Spec
    wts: dict
    lin: dict = field(default_factory=dict)

    def __post_init__(self):
        s, w = self.spec, self.wts
        if s.family in ("llama", "qwen2"):
            for i in range(s.layers):
                p = f"model.layers.{i}."
                for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                    self.lin[p + n] = _qlin(w[p + f"self_attn.{n}.weight"], w.get(p + f"self_attn.{n}.bias"))
                for n in ("gate_proj", "up_proj", "down_proj"):
                    self.lin[p + n] = _qlin(w[p + f"mlp.{n}.weight"])
            head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
            self.lin["lm_head"] = _qlin(head)
        else:
            for i in range(s.layers):
                p = f"transformer.h.{i}."
                for n in ("attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj"):
                    self.lin[p + n] = _qlin(w[p + n + ".weight"].T, w[p + n + ".bias"])
            self.lin["lm_head"] = _qlin(w["transformer.wte.weight"])

    def new_cache(self):
        return [([], []) for _ in range(self.spec.layers)]

    def step(self, token: int, pos: int, cache) -> np.ndarray:
        """Process one token of one sequence at position ``pos``; append its K/V to
        ``cache``; return the fp64 logits [V]."""
        s, w = self.spec, self.wts
        f64 = lambda a: np.asarray(a, dtype=np.float64)
        D, Hq, Hkv = s.head_dim, s.heads, s.kv_heads
        scale = 1.0 / np.sqrt(D)
        if s.family == "gpt2":
            h = f64(w["transformer.wte.weight"][token]) + f64(w["transformer.wpe.weight"][pos])
        else:
            h = f64(w["model.embed_tokens.weight"][token])
            cos, sin = rope_cos_sin(pos, D, s.rope_theta)
        for i in range(s.layers):
            if s.family == "gpt2":
                p = f"transformer.h.{i}."
                x = layer_norm(h, f64(w[p + "ln_1.weight"]), f64(w[p + "ln_1.bias"]), s.eps)
                qkv = self.lin[p + "attn.c_attn"](x)
                q, k, v = np.split(qkv, 3)
            else:
                p = f"model.layers.{i}."
                x = rms_norm(h, f64(w[p + "input_layernorm.weight"]), s.eps)
                q, k, v = (self.lin[p + n](x) for n in ("q_proj", "k_proj", "v_proj"))
            q = q.reshape(Hq, D)
            k = k.reshape(Hkv, D)
            v = v.reshape(Hkv, D)
            if s.family != "gpt2":
                q = q * cos + rotate_half(q) * sin
                k = k * cos + rotate_half(k) * sin
            cache[i][0].append(k)
            cache[i][1].append(v)
            K = np.stack(cache[i][0], axis=1)   # [Hkv, L, D]
            V = np.stack(cache[i][1], axis=1)
            att = np.empty((Hq, D))
            grp = Hq // Hkv
            for g in range(Hq):
                sc = K[g // grp] @ q[g] * scale
                pr = np.exp(sc - sc.max())
                att[g] = (pr / pr.sum()) @ V[g // grp]
            att = att.reshape(-1)
            if s.family == "gpt2":
                h = h + self.lin[p + "attn.c_proj"](att)
                x = layer_norm(h, f64(w[p + "ln_2.weight"]), f64(w[p + "ln_2.bias"]), s.eps)
                h = h + self.lin[p + "mlp.c_proj"](gelu_new(self.lin[p + "mlp.c_fc"](x)))
            else:
                h = h + self.lin[p + "o_proj"](att)
                x = rms_norm(h, f64(w[p + "post_attention_layernorm.weight"]), s.eps)
                h = h + self.lin[p + "down_proj"](silu(self.lin[p + "gate_proj"](x)) * self.lin[p + "up_proj"](x))
        if s.family == "gpt2":
            x = layer_norm(h, f64(w["transformer.ln_f.weight"]), f64(w["transformer.ln_f.bias"]), s.eps)
        else:
            x = rms_norm(h, f64(w["model.norm.weight"]), s.eps)
        return self.lin["lm_head"](x)

    def greedy(self, prompt: list[int], n_new: int) -> tuple[list[int], list[np.ndarray]]:
        """Greedy stream of one sequence (``torch.argmax``: first maximal index)."""
        cache = self.new_cache()
        logits = None
        for t, tok in enumerate(prompt):
            logits = self.step(int(tok), t, cache)
        out, all_logits = [], []
        pos = len(prompt)
        for _ in range(n_new):
            nxt = int(np.argmax(logits))
            out.append(nxt)
            all_logits.append(logits)
            logits = self.step(nxt, pos, cache)
            pos += 1
        return out, all_logits

"""How far bf16 activations alone move the logits of the full-shape models (test infrastructure).

The B200 path computes every linear from INT8 codes and bf16 activations with fp32 accumulation, keeps
the residual stream in fp32 and stores K/V in bf16; the reference's ``QuantizedPyTorchBackend`` does
the same arithmetic on the same dequantized weights in fp32 throughout. This script replays the prefill
of each ``full_<shape>.npz`` fixture on the CPU twice — in fp32, and with the B200 path's bf16 rounding
points (norm outputs, the attention output and the MLP activation entering a linear, K and V) emulated —
and compares both with the reference's own logits stored in the fixture. The fp32 replay checks the
replay itself (its gap to the fixture is ~1e-5); the bf16 replay measures the rounding's effect, which
``tests/test_gpu_full_models.py`` uses to scale its model-level logit tolerance. Writes
``full_<shape>_bf16.json``:

    python tests/golden/bf16_sensitivity.py [gpt2_small qwen_05b llama_3b]
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.quant import quantize_rows_i8  # noqa: E402
from tests._hf_models import seeded_state_for_shape  # noqa: E402


def _deq(w: torch.Tensor) -> torch.Tensor:
    q, s = quantize_rows_i8(np.ascontiguousarray(w.numpy(), dtype=np.float32))
    return torch.from_numpy(q.astype(np.float32) * s[:, None])


def replay(shape: dict, st: dict, dq, prompts: torch.Tensor, bf16: bool) -> torch.Tensor:
    """Logits [B, V] after the prompts (causal prefill), fp32 or with bf16 rounding points. ``st``: the
    seeded parameters; ``dq(name, transpose)``: the dequantized INT8 weight of a parameter."""
    r = (lambda t: t.to(torch.bfloat16).float()) if bf16 else (lambda t: t)
    fam, L = shape["family"], shape["layers"]
    H, hq, hkv, D = shape["hidden"], shape["heads"], shape["kv_heads"], shape["head_dim"]
    eps = shape["eps"]
    B, T = prompts.shape
    mask = torch.full((T, T), float("-inf")).triu(1)
    g = lambda k: st.get(k)

    def lin(x, w, b=None):
        y = x @ w.T
        return y if b is None else y + b

    def norm(h, w, b):
        if fam == "gpt2":
            mu = h.mean(-1, keepdim=True)
            var = (h - mu).pow(2).mean(-1, keepdim=True)
            return (h - mu) * torch.rsqrt(var + eps) * w + b
        return w * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps))

    def attend(q, k, v):  # [B, T, heads*D] each
        q = q.view(B, T, hq, D).transpose(1, 2)
        k = k.view(B, T, hkv, D).transpose(1, 2)
        v = v.view(B, T, hkv, D).transpose(1, 2)
        if fam != "gpt2":
            theta = shape["rope_theta"]
            inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
            ang = torch.arange(T).float()[:, None] * inv[None, :]
            cos, sin = torch.cat([ang.cos()] * 2, 1), torch.cat([ang.sin()] * 2, 1)
            rot = lambda x: x * cos + torch.cat([-x[..., D // 2:], x[..., :D // 2]], -1) * sin
            q, k = rot(q), rot(k)
        k, v = r(k).repeat_interleave(hq // hkv, 1), r(v).repeat_interleave(hq // hkv, 1)
        a = torch.softmax(q @ k.transpose(-1, -2) / D ** 0.5 + mask, -1) @ v
        return a.transpose(1, 2).reshape(B, T, hq * D)

    if fam == "gpt2":
        h = g("transformer.wte.weight")[prompts] + g("transformer.wpe.weight")[:T][None]
    else:
        h = g("model.embed_tokens.weight")[prompts].clone()
    for i in range(L):
        if fam == "gpt2":
            p = f"transformer.h.{i}."
            wqkv = dq(p + "attn.c_attn.weight", True)
            x = r(norm(h, g(p + "ln_1.weight"), g(p + "ln_1.bias")))
            qkv = lin(x, wqkv, g(p + "attn.c_attn.bias"))
            a = attend(*qkv.split(H, -1))
            h = h + lin(r(a), dq(p + "attn.c_proj.weight", True), g(p + "attn.c_proj.bias"))
            x = r(norm(h, g(p + "ln_2.weight"), g(p + "ln_2.bias")))
            u = lin(x, dq(p + "mlp.c_fc.weight", True), g(p + "mlp.c_fc.bias"))
            act = r(0.5 * u * (1.0 + torch.tanh((2.0 / np.pi) ** 0.5 * (u + 0.044715 * u ** 3))))
            h = h + lin(act, dq(p + "mlp.c_proj.weight", True), g(p + "mlp.c_proj.bias"))
        else:
            p = f"model.layers.{i}."
            x = r(norm(h, g(p + "input_layernorm.weight"), None))
            q, k, v = (lin(x, dq(p + f"self_attn.{n}_proj.weight"), g(p + f"self_attn.{n}_proj.bias"))
                       for n in "qkv")
            h = h + lin(r(attend(q, k, v)), dq(p + "self_attn.o_proj.weight"))
            x = r(norm(h, g(p + "post_attention_layernorm.weight"), None))
            gt = lin(x, dq(p + "mlp.gate_proj.weight"))
            up = lin(x, dq(p + "mlp.up_proj.weight"))
            h = h + lin(r(torch.nn.functional.silu(gt) * up), dq(p + "mlp.down_proj.weight"))
    hl = h[:, -1]
    if fam == "gpt2":
        x = r(norm(hl, g("transformer.ln_f.weight"), g("transformer.ln_f.bias")))
        head = "transformer.wte.weight"
    else:
        x = r(norm(hl, g("model.norm.weight"), None))
        head = "lm_head.weight" if g("lm_head.weight") is not None else "model.embed_tokens.weight"
    return x @ dq(head).T


def main(names):
    torch.set_num_threads(os.cpu_count() or 8)
    for name in names:
        d = np.load(os.path.join(HERE, f"full_{name}.npz"))
        shape = json.loads(str(d["shape"]))
        prompts = torch.tensor(d["prompts"])
        idx = torch.from_numpy(d["logit_idx"])
        want = d["logit_val"][:, 0]
        out = {"shape": name, "sampled_logits": int(want.size)}
        _, st = seeded_state_for_shape(shape, seed=0)
        cache = {}

        def dq(pname, transpose=False):
            if pname not in cache:
                w = st[pname].t().contiguous() if transpose else st[pname]
                cache[pname] = _deq(w)
            return cache[pname]

        with torch.no_grad():
            for mode in ("fp32", "bf16"):
                got = replay(shape, st, dq, prompts, mode == "bf16")[:, idx].numpy()
                err = np.abs(got.astype(np.float64) - want)
                out[f"{mode}_max_dev"] = float(err.max())
                out[f"{mode}_mean_dev"] = float(err.mean())
                print(name, mode, out[f"{mode}_max_dev"], out[f"{mode}_mean_dev"], flush=True)
        with open(os.path.join(HERE, f"full_{name}_bf16.json"), "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1:] or ["gpt2_small", "qwen_05b", "llama_3b"])

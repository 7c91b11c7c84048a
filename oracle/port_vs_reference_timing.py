"""Times the CPU port (``cpu_baseline.measure_steps``) against the reference's own decode, on the same cores.

Test / bench infrastructure, run where the reference checkout is importable (``MICROGEN_REFERENCE``); it
validates the port that ``bench.py`` times as the CPU baseline and the reference arm. It builds a
Llama-3.2-3B-shaped ``LlamaForCausalLM`` with fewer layers (random init), loads it into the reference's
``QuantizedPyTorchBackend`` (every ``nn.Linear``, lm_head included, becomes a ``QuantizedLinear`` that
dequantizes its weight on each call, ``microgen/backends/quantized.py:24-27, 41-73``), fills a
``DynamicCache`` with ``ctx`` random K/V positions per layer (the reference's own prefill would also
materialise logits for every prompt position, 38 GB at this size) and times ``backend.decode``
(``microgen/backends/pytorch.py:118-142``: one HF forward over the cache, which grows by ``torch.cat``) at
batch ``B``. It then times whole steps of the numpy port at the same shape, layer count, batch and context.
Prints one JSON line with both step times and their ratio.

    MICROGEN_REFERENCE=<checkout> python oracle/port_vs_reference_timing.py [--layers 2] [--steps 3]
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))

LLAMA_3B = dict(hidden=3072, heads=24, kv_heads=8, head_dim=128, inter=8192, vocab=128256, eps=1e-5,
                theta=500000.0)


def reference_step_s(layers: int, batch: int, ctx: int, steps: int) -> float:
    import torch
    from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM
    from microgen.backends.quantized import QuantizedPyTorchBackend
    s = LLAMA_3B
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=s["hidden"], intermediate_size=s["inter"], num_hidden_layers=layers,
                      num_attention_heads=s["heads"], num_key_value_heads=s["kv_heads"], head_dim=s["head_dim"],
                      vocab_size=s["vocab"], rms_norm_eps=s["eps"], max_position_embeddings=ctx + steps + 8,
                      rope_parameters={"rope_theta": s["theta"], "rope_type": "default"},
                      tie_word_embeddings=True)
    model = LlamaForCausalLM(cfg).eval()
    be = QuantizedPyTorchBackend()
    be.load_model("llama-3.2-3b-shape", model_instance=model)
    cache = DynamicCache()
    for layer in range(layers):
        kv = (batch, s["kv_heads"], ctx, s["head_dim"])
        cache.update(torch.randn(kv), torch.randn(kv), layer)
    tok = torch.randint(0, s["vocab"], (batch, 1))
    logits, cache = be.decode(tok, cache=cache)  # warm-up
    times = []
    for _ in range(steps):
        tok = be.sample(logits, temperature=0.0)
        t0 = time.perf_counter()
        logits, cache = be.decode(tok, cache=cache)
        times.append(time.perf_counter() - t0)
    return sum(times) / len(times)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=2304)
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args()
    ref = os.environ.get("MICROGEN_REFERENCE")
    if not ref:
        sys.exit("set MICROGEN_REFERENCE to the MicroGen checkout")
    sys.path.insert(0, ref)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch
    from oracle.cpu_baseline import measure_steps
    ref_s = reference_step_s(args.layers, args.batch, args.ctx, args.steps)
    s = LLAMA_3B
    port = measure_steps(s["hidden"], s["heads"], s["kv_heads"], s["head_dim"], s["inter"], s["vocab"],
                         args.layers, args.batch, args.ctx, budget_s=1e9, max_steps=args.steps, warmup=1,
                         eps=s["eps"], theta=s["theta"])
    print(json.dumps({"shape": "Llama-3.2-3B", "layers": args.layers, "batch": args.batch, "ctx": args.ctx,
                      "steps": args.steps, "torch_threads": torch.get_num_threads(), "cores": os.cpu_count(),
                      "reference_ms_per_step": round(1e3 * ref_s, 1),
                      "port_ms_per_step": round(1e3 * port["step_s"], 1),
                      "port_over_reference": round(port["step_s"] / ref_s, 3)}), flush=True)


if __name__ == "__main__":
    main()

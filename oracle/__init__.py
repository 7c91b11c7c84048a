"""CPU oracle for the decode-step hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the reference (MicroGen) for
the path the CUDA library accelerates:

* ``quant``     — per-output-channel INT8 weight quantization
                  (``microgen/backends/quantized.py:30-39``), bit-exact contract.
* ``linear``    — the INT8 weight-only linear, dequantize-then-matmul
                  (``microgen/backends/quantized.py:24-27``) and the column/row
                  tensor-parallel splits (``microgen/backends/parallel.py:12-81``).
* ``attention`` — decode attention over a paged KV pool: gather through the block
                  table, then softmax(q·Kᵀ·scale)·V with GQA head mapping, the
                  computation HF's ``sdpa_attention_forward`` performs on the
                  contiguous cache the reference grows with ``torch.cat``
                  (``microgen/runtime/kv_cache.py:76-127``).
* ``model``     — one decode step of the three model families on the path
                  (Llama / Qwen2 / GPT-2 shapes), restating the forward of
                  transformers 5.5.0 (``modeling_llama.py``, ``modeling_qwen2.py``,
                  ``modeling_gpt2.py``) with the quantized linears swapped in.
* ``cpu_baseline`` — not a checker: the reference's CPU decode step restated with
                  the same torch CPU operations it runs, for timing only
                  (``port_vs_reference_timing.py`` compares it with the reference).

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
fixtures under ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
importing and running the reference itself (and transformers 5.5.0) in the
build container.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker / the timed CPU
baseline. The product path (``microgen_b200``) never imports it.
"""

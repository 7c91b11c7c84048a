"""Generate the golden fixtures under tests/golden/ by running the REFERENCE itself.

Run where the reference checkout and transformers 5.5.0 are importable;
``MICROGEN_REFERENCE`` must point at the checkout::

    MICROGEN_REFERENCE=<checkout> python tests/golden/make_golden.py          # small fixtures
    MICROGEN_REFERENCE=<checkout> python tests/golden/make_golden.py --full   # full-shape streams

Every array written here is an output of the reference's own code:

* ``quant_cases.npz``   — ``quantize_linear_layer_per_channel``
  (``microgen/backends/quantized.py:30-39``) on seeded and edge-case matrices;
  ``quant_digest.json`` — sha256 of codes+scales for a full Llama-3.2-3B-shaped
  q_proj (3072×3072, N(0, 0.02)), too large to store.
* ``linear_cases.npz``  — ``QuantizedLinear.forward`` (``quantized.py:24-27``)
  and ``ColumnParallelLinear`` / ``RowParallelLinear`` (``parallel.py:12-81``)
  on the dequantized weights, world sizes 2 and 3 (uneven split).
* ``attn_cases.npz``    — decode attention as the reference computes it:
  ``KVCacheState.update`` (``runtime/kv_cache.py:76-127``) then HF
  ``sdpa_attention_forward``; block tables drawn from the reference
  ``PagedKVCacheAllocator`` (``runtime/paged_kv.py``) after a seeded shuffle of its
  free list, and the paged pools filled from the contiguous cache.
* ``alloc_trace.json``  — block ids the reference allocator hands out for a
  scripted allocate / append / free sequence.
* ``model_<family>.npz``— a greedy stream of 64 tokens and the logits of its
  first steps from ``QuantizedPyTorchBackend`` (``quantized.py:41-73``)
  ``prefill``/``decode`` on seeded tiny Llama / Qwen2 / GPT-2 models. For GPT-2
  the Conv1D projections are first rewrapped as ``nn.Linear`` (weight =
  ``Conv1D.weight.T``), because the reference quantizer only swaps ``nn.Linear``.
* ``kv8_cases.npz`` (``--kv8``) — INT8 KV (``KVCacheState(quantize_kv=True)``): the per-vector
  quantizer, SDPA over the stored INT8 cache, and a tiny-Llama greedy stream with that cache.
* ``full_<shape>.npz`` (``--full``) — the same greedy stream at the full model
  shapes of the workloads (GPT-2-small, Qwen2.5-0.5B, Llama-3.2-3B; every layer,
  the full vocabulary) for a batch of two prompts: 64 greedy tokens per sequence,
  the reference's top-1 minus top-2 logit margin at every step, and a sample of
  the logits of the first steps (a fixed strided index set plus each row's top 16).
"""

from __future__ import annotations

import hashlib
import json
import os
import random
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("MICROGEN_REFERENCE")
if not REF:
    sys.exit("set MICROGEN_REFERENCE to the MicroGen checkout whose code produces the fixtures")
sys.path.insert(0, REF)
sys.path.insert(0, ROOT)  # this repository's ``tests`` package wins over the reference's

from microgen.backends.quantized import (QuantizedPyTorchBackend,  # noqa: E402
                                         quantize_linear_layer_per_channel)
from microgen.backends.parallel import ColumnParallelLinear, RowParallelLinear  # noqa: E402
from microgen.runtime.kv_cache import KVCacheState  # noqa: E402
from microgen.runtime.paged_kv import PagedKVCacheAllocator  # noqa: E402
from transformers.integrations.sdpa_attention import sdpa_attention_forward  # noqa: E402

from tests._hf_models import TINY, make_hf_model, prompt_ids  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def ref_quantize(w: np.ndarray):
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(w))
    ql = quantize_linear_layer_per_channel(lin)
    return ql, ql.weight_int8.numpy().copy(), ql.scales.numpy().reshape(-1).copy()


def edge_matrix() -> np.ndarray:
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((8, 48), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w[0] = 0.0                                                  # all-zero row: scale clamps to 1e-8
    w[1] = 0.0
    w[1, :9] = np.array([127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5], np.float32)  # exact ties (scale 1)
    w[2] = np.float32(1e-9) * np.arange(48, dtype=np.float32)  # tiny row: scale floor
    w[3] = 0.0
    w[3, 5] = -3.0                                              # single negative extreme
    w[4] *= np.float32(1e6)                                     # large magnitudes
    w[5] = np.float32(1e-7)                                     # constant row below the floor*127
    w[6, ::2] = -w[6, 1::2]                                     # symmetric pairs
    w[7] = np.linspace(-1, 1, 48, dtype=np.float32)
    return w


def make_quant():
    cases = {}
    rng = np.random.default_rng(1)
    mats = {
        "seeded": (rng.standard_normal((64, 96), dtype=np.float32) * np.float32(0.02)).astype(np.float32),
        "edge": edge_matrix(),
        "wide": (rng.standard_normal((5, 4096), dtype=np.float32) * np.float32(0.02)).astype(np.float32),
        "ragged": (rng.standard_normal((3, 16), dtype=np.float32)).astype(np.float32),
    }
    for name, w in mats.items():
        _, q, s = ref_quantize(w)
        cases[f"{name}_w"], cases[f"{name}_q"], cases[f"{name}_s"] = w, q, s
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **cases)

    # Size-independent property for the full-size matrix: digest of the reference's output.
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(3072, 3072, generator=g, dtype=torch.float32) * 0.02)
    lin = torch.nn.Linear(3072, 3072, bias=False)
    with torch.no_grad():
        lin.weight.copy_(w)
    ql = quantize_linear_layer_per_channel(lin)
    h = hashlib.sha256()
    h.update(ql.weight_int8.numpy().tobytes())
    h.update(ql.scales.numpy().astype(np.float32).tobytes())
    wd = hashlib.sha256(w.numpy().tobytes()).hexdigest()
    with open(os.path.join(HERE, "quant_digest.json"), "w") as f:
        json.dump({"generator": "torch.Generator().manual_seed(3); randn(3072,3072)*0.02 fp32",
                   "weight_sha256": wd, "codes_scales_sha256": h.hexdigest(),
                   "code_hist_minus127_0_127": [int((ql.weight_int8 == -127).sum()), int((ql.weight_int8 == 0).sum()),
                                                int((ql.weight_int8 == 127).sum())]}, f, indent=1)


def make_linear():
    out = {}
    rng = np.random.default_rng(2)
    for tag, (M, K, N) in {"a": (5, 96, 40), "b": (1, 64, 33), "c": (8, 160, 72)}.items():
        w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        b = (rng.standard_normal(N, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        x = rng.standard_normal((M, K), dtype=np.float32)
        lin = torch.nn.Linear(K, N)
        with torch.no_grad():
            lin.weight.copy_(torch.from_numpy(w))
            lin.bias.copy_(torch.from_numpy(b))
        ql = quantize_linear_layer_per_channel(lin)
        xt = torch.from_numpy(x)
        with torch.no_grad():
            y = ql(xt).numpy()
            wdq = (ql.weight_int8.float() * ql.scales).clone()
            res = {}
            for world in (2, 3):
                col = ColumnParallelLinear(wdq, lin.bias.data, world)
                row = RowParallelLinear(wdq, lin.bias.data, world)
                res[f"col{world}"] = col(xt).numpy()
                res[f"row{world}"] = row(xt).numpy()
        out.update({f"{tag}_x": x, f"{tag}_w": w, f"{tag}_b": b, f"{tag}_q": ql.weight_int8.numpy(),
                    f"{tag}_s": ql.scales.numpy().reshape(-1), f"{tag}_y": y})
        out.update({f"{tag}_{k}": v for k, v in res.items()})
    np.savez_compressed(os.path.join(HERE, "linear_cases.npz"), **out)


class _Attn(torch.nn.Module):
    def __init__(self, groups):
        super().__init__()
        self.num_key_value_groups = groups
        self.is_causal = True


def make_attn():
    out = {}
    cases = {
        "gqa": dict(B=3, Hq=8, Hkv=2, D=64, ctx=[1, 17, 40], blocks=16, seed=11),
        "mha": dict(B=2, Hq=4, Hkv=4, D=32, ctx=[16, 33], blocks=8, seed=12),
        "llama": dict(B=2, Hq=24, Hkv=8, D=128, ctx=[50, 128], blocks=16, seed=13),
    }
    for tag, c in cases.items():
        B, Hq, Hkv, D, ctx = c["B"], c["Hq"], c["Hkv"], c["D"], c["ctx"]
        rng = np.random.default_rng(c["seed"])
        L = max(ctx)
        q = rng.standard_normal((B, Hq, D), dtype=np.float32)
        k = rng.standard_normal((B, Hkv, L, D), dtype=np.float32)
        v = rng.standard_normal((B, Hkv, L, D), dtype=np.float32)
        alloc = PagedKVCacheAllocator(num_blocks=c["blocks"] * B, block_size=16)
        random.Random(c["seed"]).shuffle(alloc._free_blocks)
        maxb = (L + 15) // 16
        tables = np.zeros((B, maxb), np.int32)
        kpool = np.zeros((alloc.num_blocks, Hkv, 16, D), np.float32)
        vpool = np.zeros_like(kpool)
        outs = np.zeros((B, Hq, D), np.float32)
        for b in range(B):
            bt = alloc.allocate_sequence(f"s{b}", ctx[b])
            ids = [blk.block_id for blk in bt.physical_blocks]
            tables[b, :len(ids)] = ids
            for t in range(ctx[b]):
                kpool[ids[t // 16], :, t % 16] = k[b, :, t]
                vpool[ids[t // 16], :, t % 16] = v[b, :, t]
            # reference: contiguous cache grown by KVCacheState.update, then HF SDPA for one query token
            cache = KVCacheState(max_seq_len=4096)
            kk = torch.from_numpy(k[b:b + 1, :, :ctx[b]])
            vv = torch.from_numpy(v[b:b + 1, :, :ctx[b]])
            split = max(1, ctx[b] // 2)
            cache.update(kk[:, :, :split], vv[:, :, :split], 0)
            kc, vc = cache.update(kk[:, :, split:], vv[:, :, split:], 0) if ctx[b] > split else (kk, vv)
            qq = torch.from_numpy(q[b:b + 1, :, None, :])
            o, _ = sdpa_attention_forward(_Attn(Hq // Hkv), qq, kc, vc, None, scaling=1.0 / np.sqrt(D))
            outs[b] = o[0, 0].numpy()
        out.update({f"{tag}_q": q, f"{tag}_kpool": kpool, f"{tag}_vpool": vpool, f"{tag}_tables": tables,
                    f"{tag}_ctx": np.array(ctx, np.int32), f"{tag}_out": outs})
    np.savez_compressed(os.path.join(HERE, "attn_cases.npz"), **out)


def make_alloc_trace():
    a = PagedKVCacheAllocator(num_blocks=12, block_size=16)
    trace = []
    t1 = a.allocate_sequence("a", 35)
    trace.append(("alloc", "a", 35, [b.block_id for b in t1.physical_blocks]))
    t2 = a.allocate_sequence("b", 16)
    trace.append(("alloc", "b", 16, [b.block_id for b in t2.physical_blocks]))
    for _ in range(13):
        a.append_token(t1)
    trace.append(("append13", "a", t1.num_tokens, [b.block_id for b in t1.physical_blocks]))
    a.append_token(t2)
    trace.append(("append1", "b", t2.num_tokens, [b.block_id for b in t2.physical_blocks]))
    a.free_sequence(t1)
    trace.append(("free", "a", a.get_num_free_blocks(), [b.block_id for b in a._free_blocks]))
    t3 = a.allocate_sequence("c", 70)
    trace.append(("alloc", "c", 70, [b.block_id for b in t3.physical_blocks]))
    t4 = a.allocate_sequence("d", 0)
    trace.append(("alloc", "d", 0, [b.block_id for b in t4.physical_blocks]))
    err = None
    try:
        a.allocate_sequence("e", 16 * 20)
    except MemoryError as e:
        err = str(e)
    trace.append(("oom", "e", 320, err))
    with open(os.path.join(HERE, "alloc_trace.json"), "w") as f:
        json.dump(trace, f, indent=1)


def make_prefix_trace():
    """Scripted insert / match / evict / get sequence on the reference's PrefixKVCache (capacity 3); each
    stored state is a label, so the trace records which entry every lookup returns."""
    from microgen.caching.prefix_cache import PrefixKVCache, compute_token_hash
    pc = PrefixKVCache(max_capacity=3)
    seqs = {"a": list(range(1, 33)), "b": list(range(1, 17)), "c": [7] * 16 + [9] * 16, "d": list(range(1, 49)),
            "e": [3] * 16}
    trace = []
    keys = {}

    def match(ids):
        m = pc.match_prefix(ids)
        return None if m is None else [m[0], m[1]]

    for lab in ("a", "b", "c"):
        keys[lab] = pc.insert(seqs[lab], lab)
        trace.append(["insert", lab, keys[lab], pc.size])
    for probe in (list(range(1, 41)), list(range(1, 21)), [7] * 16 + [9] * 20, [2, 3], list(range(1, 16)), []):
        trace.append(["match", probe, match(probe)])
    keys["d"] = pc.insert(seqs["d"], "d")           # evicts "a" (oldest)
    trace.append(["insert", "d", keys["d"], pc.size])
    trace.append(["get", "a", pc.get(keys["a"])])
    trace.append(["get", "b", pc.get(keys["b"])])
    trace.append(["match", list(range(1, 41)), match(list(range(1, 41)))])
    trace.append(["match", list(range(1, 60)), match(list(range(1, 60)))])
    keys["b2"] = pc.insert(seqs["b"], "b2")        # re-insert of a present key: no eviction
    trace.append(["insert", "b2", keys["b2"], pc.size])
    keys["e"] = pc.insert(seqs["e"], "e")           # evicts "b" (the oldest remaining insertion)
    trace.append(["insert", "e", keys["e"], pc.size])
    trace.append(["match", list(range(1, 20)), match(list(range(1, 20)))])
    trace.append(["hash", [1, 2, 3], compute_token_hash([1, 2, 3])])
    with open(os.path.join(HERE, "prefix_trace.json"), "w") as f:
        json.dump({"seqs": seqs, "trace": trace}, f, indent=0)


def _conv1d_to_linear(model):
    from transformers.pytorch_utils import Conv1D

    def walk(mod):
        for name, ch in list(mod.named_children()):
            if isinstance(ch, Conv1D):
                lin = torch.nn.Linear(ch.weight.shape[0], ch.weight.shape[1])
                with torch.no_grad():
                    lin.weight.copy_(ch.weight.t())
                    lin.bias.copy_(ch.bias)
                setattr(mod, name, lin)
            else:
                walk(ch)
    walk(model)


def make_models(n_prompt=16, n_new=64, n_logits=8):
    for fam, shape in TINY.items():
        model, state = make_hf_model(shape, seed=0)
        if fam == "gpt2":
            _conv1d_to_linear(model)
        be = QuantizedPyTorchBackend(quant_type="int8")
        be.load_model(f"tiny-{fam}", model_instance=model)
        prompt = prompt_ids(shape["vocab"], n_prompt, seed=0)
        ids = torch.tensor([prompt], dtype=torch.long)
        logits, cache = be.prefill(ids, cache=KVCacheState(max_seq_len=1024))
        toks, lg = [], []
        for i in range(n_new):
            tok = torch.argmax(logits, dim=-1, keepdim=True)
            toks.append(int(tok.item()))
            if i < n_logits:
                lg.append(logits[0].numpy().copy())
            logits, cache = be.decode(tok, cache=cache)
        np.savez_compressed(os.path.join(HERE, f"model_{fam}.npz"), prompt=np.array(prompt, np.int64),
                            tokens=np.array(toks, np.int64), logits=np.stack(lg).astype(np.float32),
                            shape=json.dumps(shape))


def make_kv8(n_prompt=16, n_new=32, n_logits=8):
    """INT8 KV (``KVCacheState(quantize_kv=True)``, ``runtime/kv_cache.py:30-40, 114-120``): the reference's
    per-vector quantizer on seeded and edge-case vectors; its stored codes and scales after two updates with
    the SDPA decode output over their dequantization; and a tiny-Llama greedy stream decoded with an INT8
    cache (``QuantizedPyTorchBackend``)."""
    from microgen.runtime.kv_cache import _dequantize_tensor, _quantize_tensor
    out = {}
    rng = np.random.default_rng(21)
    x = rng.standard_normal((64, 64), dtype=np.float32) * np.float32(3.0)
    x[0] = 0.0                                        # the 1e-8 scale floor
    x[1] = np.linspace(-1.0, 1.0, 64, dtype=np.float32)
    x[2, :] = 0.5
    x[2, 0] = 127.0                                   # exact .5 quotients: round half to even
    x[3] = 1e-12                                      # tiny vector: floor scale, codes clamp at 127
    q, sc = _quantize_tensor(torch.from_numpy(x))
    out.update(quant_x=x, quant_q=q.numpy(), quant_s=sc.numpy()[:, 0])
    # attention over the stored INT8 cache of the reference
    B, Hq, Hkv, D, ctx = 2, 12, 4, 64, [37, 80]
    L = max(ctx)
    q_ = rng.standard_normal((B, Hq, D), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, L, D), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, L, D), dtype=np.float32)
    alloc = PagedKVCacheAllocator(num_blocks=16 * B, block_size=16)
    random.Random(22).shuffle(alloc._free_blocks)
    maxb = (L + 15) // 16
    tables = np.zeros((B, maxb), np.int32)
    kpool = np.zeros((alloc.num_blocks, Hkv, 16, D), np.int8)
    vpool = np.zeros_like(kpool)
    kscale = np.zeros((alloc.num_blocks, Hkv, 16), np.float32)
    vscale = np.zeros_like(kscale)
    outs = np.zeros((B, Hq, D), np.float32)
    for b in range(B):
        cache = KVCacheState(max_seq_len=4096, quantize_kv=True)
        kk = torch.from_numpy(k[b:b + 1, :, :ctx[b]])
        vv = torch.from_numpy(v[b:b + 1, :, :ctx[b]])
        split = ctx[b] // 2
        cache.update(kk[:, :, :split], vv[:, :, :split], 0)
        cache.update(kk[:, :, split:], vv[:, :, split:], 0)
        kc, vc = cache.key_cache[0], cache.value_cache[0]          # int8 [1, Hkv, ctx, D]
        ks, vs = cache.key_scales[0], cache.value_scales[0]        # fp32 [1, Hkv, ctx, 1]
        bt = alloc.allocate_sequence(f"s{b}", ctx[b])
        ids = [blk.block_id for blk in bt.physical_blocks]
        tables[b, :len(ids)] = ids
        for t in range(ctx[b]):
            kpool[ids[t // 16], :, t % 16] = kc[0, :, t].numpy()
            vpool[ids[t // 16], :, t % 16] = vc[0, :, t].numpy()
            kscale[ids[t // 16], :, t % 16] = ks[0, :, t, 0].numpy()
            vscale[ids[t // 16], :, t % 16] = vs[0, :, t, 0].numpy()
        kd = _dequantize_tensor(kc, ks, torch.float32)
        vd = _dequantize_tensor(vc, vs, torch.float32)
        qq = torch.from_numpy(q_[b:b + 1, :, None, :])
        o, _ = sdpa_attention_forward(_Attn(Hq // Hkv), qq, kd, vd, None, scaling=1.0 / np.sqrt(D))
        outs[b] = o[0, 0].numpy()
    out.update(attn_q=q_, attn_kpool=kpool, attn_vpool=vpool, attn_kscale=kscale, attn_vscale=vscale,
               attn_tables=tables, attn_ctx=np.array(ctx, np.int32), attn_out=outs)
    # tiny Llama greedy stream with an INT8 KV cache
    shape = TINY["llama"]
    model, _ = make_hf_model(shape, seed=0)
    be = QuantizedPyTorchBackend(quant_type="int8")
    be.load_model("tiny-llama", model_instance=model)
    prompt = prompt_ids(shape["vocab"], n_prompt, seed=0)
    logits, cache = be.prefill(torch.tensor([prompt], dtype=torch.long),
                               cache=KVCacheState(max_seq_len=1024, quantize_kv=True))
    toks, lg = [], []
    for i in range(n_new):
        tok = torch.argmax(logits, dim=-1, keepdim=True)
        toks.append(int(tok.item()))
        if i < n_logits:
            lg.append(logits[0].numpy().copy())
        logits, cache = be.decode(tok, cache=cache)
    out.update(model_prompt=np.array(prompt, np.int64), model_tokens=np.array(toks, np.int64),
               model_logits=np.stack(lg).astype(np.float32), model_shape=json.dumps(shape))
    np.savez_compressed(os.path.join(HERE, "kv8_cases.npz"), **out)


# Full-shape greedy streams: batch of two prompts of FULL_PROMPT ids; the Llama-3.2-3B shape shares
# its first FULL_SHARED ids across the batch (the shared-prefix workload), the others share nothing.
FULL_PROMPT, FULL_SHARED, FULL_NEW, FULL_LOGIT_STEPS, FULL_STRIDE, FULL_TOPK = 40, 32, 64, 4, 61, 16


def full_prompts(vocab: int, shared: int) -> list[list[int]]:
    head = prompt_ids(vocab, shared, seed=50) if shared else []
    return [head + prompt_ids(vocab, FULL_PROMPT - shared, seed=51 + i) for i in range(2)]


def make_full_models(names=("GPT2_SMALL", "QWEN_05B", "LLAMA_3B")):
    import gc
    import time
    from microgen_b200 import model_spec as MS
    from tests._hf_models import seeded_model
    for name in names:
        t0 = time.time()
        shape = dict(getattr(MS, name))
        shared = FULL_SHARED if name == "LLAMA_3B" else 0
        model = seeded_model(shape, seed=0)
        if shape["family"] == "gpt2":
            _conv1d_to_linear(model)
        be = QuantizedPyTorchBackend(quant_type="int8")
        be.load_model(name, model_instance=model)
        gc.collect()
        prompts = full_prompts(shape["vocab"], shared)
        ids = torch.tensor(prompts, dtype=torch.long)
        V = shape["vocab"]
        idx = np.arange(0, V, FULL_STRIDE, dtype=np.int64)
        toks, margins, vals, top_i, top_v = [], [], [], [], []
        with torch.no_grad():
            logits, cache = be.prefill(ids, cache=KVCacheState(max_seq_len=4096))
            for i in range(FULL_NEW):
                lg = logits.float()
                tok = torch.argmax(lg, dim=-1, keepdim=True)
                t2 = torch.topk(lg, 2, dim=-1).values
                toks.append(tok[:, 0].numpy().copy())
                margins.append((t2[:, 0] - t2[:, 1]).numpy().copy())
                if i < FULL_LOGIT_STEPS:
                    vals.append(lg[:, idx].numpy().copy())
                    tk = torch.topk(lg, FULL_TOPK, dim=-1)
                    top_i.append(tk.indices.numpy().copy())
                    top_v.append(tk.values.numpy().copy())
                logits, cache = be.decode(tok, cache=cache)
        np.savez_compressed(
            os.path.join(HERE, f"full_{name.lower()}.npz"), prompts=np.array(prompts, np.int64),
            shared=np.int64(shared), tokens=np.stack(toks, 1).astype(np.int64),
            margins=np.stack(margins, 1).astype(np.float32), logit_idx=idx,
            logit_val=np.stack(vals, 1).astype(np.float32), top_idx=np.stack(top_i, 1).astype(np.int64),
            top_val=np.stack(top_v, 1).astype(np.float32), shape=json.dumps(shape))
        print(f"{name}: {time.time() - t0:.0f} s; min margin {np.min(np.stack(margins)):.4f}", flush=True)
        del be, model, cache, logits
        gc.collect()


if __name__ == "__main__":
    if "--kv8" in sys.argv:
        make_kv8()
        sys.exit(0)
    if "--full" in sys.argv:
        make_full_models([a for a in sys.argv[1:] if a != "--full"] or ("GPT2_SMALL", "QWEN_05B", "LLAMA_3B"))
        sys.exit(0)
    make_quant()
    make_linear()
    make_attn()
    make_alloc_trace()
    make_prefix_trace()
    make_models()
    print("golden fixtures written to", HERE)

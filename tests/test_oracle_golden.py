"""Pin the CPU oracle against fixtures produced by the reference itself (CPU only)."""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import linear as olin
from oracle import model as omodel
from oracle.quant import quantize_rows_i8

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _npz(name):
    return np.load(os.path.join(G, name))


@pytest.mark.parametrize("case", ["seeded", "edge", "wide", "ragged"])
def test_quant_oracle_bit_exact(case):
    d = _npz("quant_cases.npz")
    q, s = quantize_rows_i8(d[f"{case}_w"])
    assert np.array_equal(q, d[f"{case}_q"])
    assert np.array_equal(s.view(np.uint32), d[f"{case}_s"].astype(np.float32).view(np.uint32))


def test_quant_oracle_full_size_digest():
    import torch
    meta = json.load(open(os.path.join(G, "quant_digest.json")))
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(3072, 3072, generator=g, dtype=torch.float32) * 0.02).numpy()
    assert hashlib.sha256(w.tobytes()).hexdigest() == meta["weight_sha256"]
    q, s = quantize_rows_i8(w)
    h = hashlib.sha256()
    h.update(q.tobytes())
    h.update(s.astype(np.float32).tobytes())
    assert h.hexdigest() == meta["codes_scales_sha256"]


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_linear_oracle_matches_reference(tag):
    d = _npz("linear_cases.npz")
    x, q, s, b = d[f"{tag}_x"], d[f"{tag}_q"], d[f"{tag}_s"], d[f"{tag}_b"]
    y = olin.i8_linear(x, q, s, b)
    np.testing.assert_allclose(y, d[f"{tag}_y"], rtol=1e-5, atol=1e-5)
    for world in (2, 3):
        np.testing.assert_allclose(olin.column_parallel_linear(x, q, s, b, world), d[f"{tag}_col{world}"],
                                   rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(olin.row_parallel_linear(x, q, s, b, world), d[f"{tag}_row{world}"],
                                   rtol=1e-5, atol=1e-5)


def test_shard_bounds_remainder_to_last_rank():
    assert olin.shard_bounds(10, 3) == [(0, 3), (3, 6), (6, 10)]
    assert olin.shard_bounds(8, 2) == [(0, 4), (4, 8)]


@pytest.mark.parametrize("tag", ["gqa", "mha", "llama"])
def test_attention_oracle_matches_reference(tag):
    d = _npz("attn_cases.npz")
    D = d[f"{tag}_q"].shape[-1]
    out = oatt.paged_decode_attention(d[f"{tag}_q"], d[f"{tag}_kpool"], d[f"{tag}_vpool"], d[f"{tag}_tables"],
                                      d[f"{tag}_ctx"], 1.0 / np.sqrt(D))
    np.testing.assert_allclose(out, d[f"{tag}_out"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("family", ["llama", "qwen2", "gpt2"])
def test_model_oracle_greedy_matches_reference(family):
    from tests._hf_models import make_hf_model
    from microgen_b200.model_spec import spec_from_hf_config
    d = _npz(f"model_{family}.npz")
    shape = json.loads(str(d["shape"]))
    model, state = make_hf_model(shape, seed=0)
    sp = spec_from_hf_config(model.config)
    spec = omodel.Spec(**{k: getattr(sp, k) for k in omodel.Spec.__dataclass_fields__})
    om = omodel.OracleModel(spec, state)
    n = 24
    toks, logits = om.greedy([int(t) for t in d["prompt"]], n)
    assert toks == [int(t) for t in d["tokens"][:n]]
    for i in range(min(len(logits), d["logits"].shape[0])):
        np.testing.assert_allclose(logits[i], d["logits"][i], rtol=1e-3, atol=2e-4)


def test_kv8_quantizer_oracle_bit_exact():
    """The INT8-KV per-vector quantizer restated in the oracle equals the reference's ``_quantize_tensor``
    (zero vectors on the 1e-8 floor, exact .5 quotients rounded half to even, tiny vectors clamped)."""
    d = _npz("kv8_cases.npz")
    q, s = oatt.quantize_kv_vectors(d["quant_x"])
    assert np.array_equal(q, d["quant_q"])
    assert np.array_equal(s.view(np.uint32), d["quant_s"].view(np.uint32))


def test_kv8_attention_oracle_matches_reference():
    """SDPA over the reference's stored INT8 cache (its codes and scales, dequantized) = the oracle over the
    same codes and scales placed in paged pools."""
    d = _npz("kv8_cases.npz")
    D = d["attn_q"].shape[-1]
    got = oatt.paged_decode_attention_kv8(d["attn_q"], d["attn_kpool"], d["attn_vpool"], d["attn_kscale"],
                                          d["attn_vscale"], d["attn_tables"], d["attn_ctx"], 1.0 / np.sqrt(D))
    np.testing.assert_allclose(got, d["attn_out"], rtol=1e-5, atol=1e-5)

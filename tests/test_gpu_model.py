"""Whole decode steps on the GPU through the backend API, against the reference's
greedy streams / logits (tests/golden/model_*.npz) and the CPU oracle model."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import model as omodel
from tests._hf_models import TINY, make_hf_model, prompt_ids

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
RTOL, ATOL = 2e-2, 1e-2


def backend(**kw):
    from microgen_b200.backends import B200QuantizedBackend
    kw.setdefault("max_batch", 8)
    kw.setdefault("max_seq_len", 256)
    return B200QuantizedBackend(**kw)


def close(got, want, rtol=RTOL, atol=ATOL):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


@pytest.mark.parametrize("family", ["llama", "qwen2", "gpt2"])
@pytest.mark.parametrize("graph", [True, False])
def test_greedy_stream_matches_reference(family, graph):
    d = np.load(os.path.join(G, f"model_{family}.npz"))
    shape = json.loads(str(d["shape"]))
    model, _ = make_hf_model(shape, seed=0)
    be = backend(use_cuda_graph=graph)
    be.load_model(f"tiny-{family}", model_instance=model)
    ids = torch.tensor([d["prompt"].tolist()])
    logits, cache = be.prefill(ids)
    toks, lgs = [], []
    for i in range(64):
        tok = be.sample(logits)
        toks.append(int(tok.item()))
        if i < d["logits"].shape[0]:
            lgs.append(logits[0].float().cpu().numpy())
        logits, cache = be.decode(tok, cache=cache)
    # logits of the first steps against the reference's fp32 path
    for i, lg in enumerate(lgs):
        close(lg, d["logits"][i])
    assert toks == d["tokens"].tolist()


def _oracle(family):
    model, state = make_hf_model(TINY[family], seed=0)
    from microgen_b200.model_spec import spec_from_hf_config
    sp = spec_from_hf_config(model.config)
    spec = omodel.Spec(**{k: getattr(sp, k) for k in omodel.Spec.__dataclass_fields__})
    return model, omodel.OracleModel(spec, state)


@pytest.mark.parametrize("family", ["llama", "qwen2", "gpt2"])
def test_batched_shared_prefix_decode_vs_oracle(family):
    model, om = _oracle(family)
    vocab = TINY[family]["vocab"]
    shared = prompt_ids(vocab, 32, seed=5)
    prompts = [shared + prompt_ids(vocab, 7, seed=10 + i) for i in range(4)]
    be = backend(free_list_seed=3)
    be.load_model("tiny", model_instance=model)
    logits, cache = be.prefill(torch.tensor(prompts))
    assert cache.n_shared_blocks == 2
    got = [logits.float().cpu().numpy()]
    nxt = [[int(t) for t in np.argmax(got[0], axis=1)]]
    for _ in range(5):
        logits, cache = be.decode(torch.tensor(nxt[-1])[:, None], cache=cache)
        got.append(logits.float().cpu().numpy())
        nxt.append([int(t) for t in np.argmax(got[-1], axis=1)])
    for i, p in enumerate(prompts):
        c = om.new_cache()
        lg = None
        for t, tok in enumerate(p):
            lg = om.step(tok, t, c)
        close(got[0][i], lg)
        pos = len(p)
        for s in range(5):
            lg = om.step(nxt[s][i], pos, c)
            pos += 1
            close(got[s + 1][i], lg)
    blocks_before = be.allocator.get_num_free_blocks()
    cache.free()
    assert be.allocator.get_num_free_blocks() > blocks_before
    assert be.allocator.get_num_allocated_blocks() == 0


def test_quantized_linear_module_and_tp_modules_match_full():
    from microgen_b200.backends import (ColumnParallelLinear, RowParallelLinear,
                                        quantize_linear_layer_per_channel)
    torch.manual_seed(0)
    lin = torch.nn.Linear(96, 80)
    x = torch.randn(2, 3, 96)
    ql = quantize_linear_layer_per_channel(lin)
    y = ql(x.cuda())
    assert y.shape == (2, 3, 80)
    from oracle.linear import i8_linear
    from oracle.quant import quantize_rows_i8
    q, s = quantize_rows_i8(lin.weight.detach().numpy())
    xb = x.to(torch.bfloat16).float().numpy().reshape(-1, 96)
    want = i8_linear(xb, q, s, lin.bias.detach().numpy()).reshape(2, 3, 80)
    close(y.cpu().numpy(), want)
    for world in (2, 3):
        col = ColumnParallelLinear(lin.weight, lin.bias, world)
        close(col(x.cuda()).cpu().numpy(), want, rtol=1e-4, atol=1e-4)
    lin2 = torch.nn.Linear(96, 40)
    row = RowParallelLinear(lin2.weight, lin2.bias, 2)
    q2, s2 = quantize_rows_i8(lin2.weight.detach().numpy())
    want2 = i8_linear(xb, q2, s2, lin2.bias.detach().numpy()).reshape(2, 3, 40)
    close(row(x.cuda()).cpu().numpy(), want2, rtol=1e-4, atol=1e-4)


def test_memory_usage_and_errors():
    from microgen_b200.backends import B200QuantizedBackend
    be = B200QuantizedBackend(max_batch=2, max_seq_len=64)
    with pytest.raises(RuntimeError):
        be.prefill(torch.tensor([[1, 2, 3]]))
    model, _ = make_hf_model(TINY["llama"], seed=0)
    be.load_model("tiny", model_instance=model)
    info = be.get_memory_usage()
    assert info["is_quantized"] and info["quant_type"] == "int8" and info["weight_bytes"] > 0
    with pytest.raises(ValueError):
        be.prefill(torch.ones((3, 4), dtype=torch.long))   # batch > max_batch
    logits, cache = be.prefill(torch.tensor([[1, 2, 3]]))
    with pytest.raises(ValueError):
        for _ in range(80):  # past max_seq_len
            logits, cache = be.decode(torch.tensor([[1]]), cache=cache)


def _hf_last_logits(model, prompt):
    with torch.no_grad():
        out = model(input_ids=torch.tensor([prompt], device="cuda"), use_cache=False)
    return out.logits[0, -1].float().cpu().numpy()


def _oracle_last_logits(family, prompt):
    _, om = _oracle(family)
    c = om.new_cache()
    lg = None
    for t, tok in enumerate(prompt):
        lg = om.step(tok, t, c)
    return lg


@pytest.mark.parametrize("family", ["llama", "qwen2"])
def test_quantize_model_swaps_every_linear(family):
    """quantize_model (quantized.py:59-73): every nn.Linear of an HF model becomes a QuantizedLinear on the
    INT8 kernel; the model's own forward then matches the oracle's INT8 model."""
    from microgen_b200.backends import QuantizedLinear, quantize_model
    model, _ = make_hf_model(TINY[family], seed=0)
    model = model.cuda()
    n_linear = sum(isinstance(m, torch.nn.Linear) for m in model.modules())
    quantize_model(model)
    assert not any(isinstance(m, torch.nn.Linear) for m in model.modules())
    assert sum(isinstance(m, QuantizedLinear) for m in model.modules()) == n_linear
    prompt = prompt_ids(TINY[family]["vocab"], 12, seed=4)
    close(_hf_last_logits(model, prompt), _oracle_last_logits(family, prompt))


@pytest.mark.parametrize("world", [2, 4])
def test_apply_tensor_parallelism_walk(world):
    """apply_tensor_parallelism (parallel.py:108-131): q/k/v/gate/up become INT8 column-parallel and o/down
    row-parallel by child name, lm_head is left alone; with lm_head then quantized, the HF forward matches the
    oracle's INT8 model."""
    from microgen_b200.backends import (ColumnParallelLinear, RowParallelLinear, apply_tensor_parallelism,
                                        quantize_model)
    model, _ = make_hf_model(TINY["llama"], seed=0)
    model = model.cuda()
    apply_tensor_parallelism(model, world)
    layer = model.model.layers[0]
    for n in ("q_proj", "k_proj", "v_proj"):
        assert isinstance(getattr(layer.self_attn, n), ColumnParallelLinear)
    assert isinstance(layer.self_attn.o_proj, RowParallelLinear)
    assert isinstance(layer.mlp.gate_proj, ColumnParallelLinear) and isinstance(layer.mlp.up_proj,
                                                                                   ColumnParallelLinear)
    assert isinstance(layer.mlp.down_proj, RowParallelLinear)
    assert isinstance(model.lm_head, torch.nn.Linear)  # unmatched: stays as it is
    assert len(layer.self_attn.q_proj.shards) == world
    quantize_model(model)  # lm_head -> INT8, as in the oracle model
    prompt = prompt_ids(TINY["llama"]["vocab"], 12, seed=6)
    close(_hf_last_logits(model, prompt), _oracle_last_logits("llama", prompt))

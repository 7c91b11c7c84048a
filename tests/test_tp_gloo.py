"""Tensor-parallel host logic on CPU with world-size-2 and -4 ``gloo`` process groups (no GPU).

* the row-parallel reduction protocol (``row_parallel_residual``): rank 0 adds its partial into the
  residual, the others store theirs, one sum all-reduce — must equal ``h + Σ partials + bias``, the
  reference's ``RowParallelLinear`` (``parallel.py:65-81``) added to the residual;
* the sharded weight loader: every rank's column shards (Q/K/V by whole heads, gate/up by 64-row
  groups) and row shards (o/down by input columns, scales replicated) reassemble the world-size-1
  codes exactly (codes from the oracle quantizer, as the device kernel produces them).
"""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world, *args):
    port = _port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(fn, args=(world, port, d) + args, nprocs=world, join=True)
        return [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]


def _init(rank, world, port):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))


def _protocol_worker(rank, world, port, outdir):
    from microgen_b200.engine import row_parallel_residual
    from microgen_b200 import kernels as K
    _init(rank, world, port)
    g = torch.Generator().manual_seed(0)
    h0 = torch.randn(4, 16, generator=g)
    parts = [torch.randn(4, 16, generator=g) for _ in range(world)]
    bias = torch.randn(16, generator=g)
    h = h0.clone()

    def launch(y, epi):
        p = parts[rank] + (bias if rank == 0 else 0.0)
        if epi == K.EPI_ADD_F32:
            y.add_(p)
        else:
            y.copy_(p)

    row_parallel_residual(h, launch, rank, world, dist.group.WORLD)
    torch.save({"h": h, "want": h0 + sum(parts) + bias}, os.path.join(outdir, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_residual_protocol(world):
    for r in _run(_protocol_worker, world):
        torch.testing.assert_close(r["h"], r["want"], rtol=1e-6, atol=1e-6)


def _oracle_quantize(w: torch.Tensor):
    from oracle.quant import quantize_rows_i8
    q, s = quantize_rows_i8(w.numpy())
    return torch.from_numpy(q), torch.from_numpy(s)


def _shape(world):
    from tests._hf_models import TINY
    # world 4 needs 4 | kv heads and 64-row gate/up groups per rank: 8/4 heads, inter 256
    return dict(TINY["llama"]) if world <= 2 else dict(TINY["llama"], heads=8, kv_heads=4)


def _load(rank, world, shape):
    from microgen_b200.engine import WeightLoader
    from microgen_b200.model_spec import spec_from_hf_config
    from tests._hf_models import make_hf_model
    model, _ = make_hf_model(shape, seed=0)
    spec = spec_from_hf_config(model.config)
    state = {k: v.detach() for k, v in model.state_dict().items()}
    w = WeightLoader(spec, "cpu", rank, world, pack=False, quantize=_oracle_quantize).load(state)
    return spec, w


def _shard_worker(rank, world, port, outdir):
    _init(rank, world, port)
    spec, w = _load(rank, world, _shape(world))
    L = w.layers[0]
    torch.save({"qkv_q": L.qkv_q, "qkv_s": L.qkv_s, "o_q": L.o_q, "o_s": L.o_s, "gu_q": L.gu_q, "gu_s": L.gu_s,
                "d_q": L.d_q, "d_s": L.d_s, "lm_q": w.lm_q}, os.path.join(outdir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _deinterleave(q):
    """Gate/up-interleaved rows (64 gate rows then the 64 matching up rows per group) -> (gate, up)."""
    g = q.view(-1, 2, 64, *q.shape[1:])
    return g[:, 0].reshape(-1, *q.shape[1:]), g[:, 1].reshape(-1, *q.shape[1:])


@pytest.mark.parametrize("world", [2, 4])
def test_tp_shards_reassemble_tp1_codes(world):
    spec, full = _load(0, 1, _shape(world))
    shards = _run(_shard_worker, world)
    D, hq, hkv = spec.head_dim, spec.heads, spec.kv_heads
    F = full.layers[0]
    qn, kn = hq * D, hkv * D
    # column-parallel q/k/v: each rank holds hq/W query heads then hkv/W k heads then hkv/W v heads
    per_q, per_k = qn // world, kn // world
    for part, (a, n) in enumerate([(0, qn), (qn, kn), (qn + kn, kn)]):
        per = per_q if part == 0 else per_k
        off = 0 if part == 0 else (per_q if part == 1 else per_q + per_k)
        got = torch.cat([s["qkv_q"][off:off + per] for s in shards])
        assert torch.equal(got, F.qkv_q[a:a + n])
        got_s = torch.cat([s["qkv_s"][off:off + per] for s in shards])
        assert torch.equal(got_s, F.qkv_s[a:a + n])
    # row-parallel o/down: input columns split, scales replicated
    assert torch.equal(torch.cat([s["o_q"] for s in shards], dim=1), F.o_q)
    assert torch.equal(torch.cat([s["d_q"] for s in shards], dim=1), F.d_q)
    for s in shards:
        assert torch.equal(s["o_s"], F.o_s) and torch.equal(s["d_s"], F.d_s)
        assert torch.equal(s["lm_q"], full.lm_q)  # lm_head replicated, as in the reference
    # gate/up: interleaved per rank; de-interleaved rank shards concatenate to the full gate / up
    fg, fu = _deinterleave(F.gu_q)
    rg = [_deinterleave(s["gu_q"]) for s in shards]
    assert torch.equal(torch.cat([g for g, _ in rg]), fg)
    assert torch.equal(torch.cat([u for _, u in rg]), fu)


# ---- vocab-parallel lm_head -----------------------------------------------------------------------
def _vocab_shard_worker(rank, world, port, outdir):
    from microgen_b200.engine import WeightLoader
    from microgen_b200.model_spec import spec_from_hf_config
    from tests._hf_models import make_hf_model
    _init(rank, world, port)
    model, _ = make_hf_model(_shape(world), seed=0)
    spec = spec_from_hf_config(model.config)
    state = {k: v.detach() for k, v in model.state_dict().items()}
    w = WeightLoader(spec, "cpu", rank, world, pack=False, quantize=_oracle_quantize,
                     vocab_parallel=True).load(state)
    torch.save({"lm_q": w.lm_q, "lm_s": w.lm_s, "off": w.lm_offset, "vp": w.vocab_parallel},
               os.path.join(outdir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_vocab_parallel_head_rows_reassemble(world):
    """Each rank keeps lm_head rows [offset, offset + n) by the reference's split rule; in rank order the
    shards are the world-size-1 codes and scales."""
    from microgen_b200.engine import vocab_bounds
    spec, full = _load(0, 1, _shape(world))
    shards = _run(_vocab_shard_worker, world)
    bounds = vocab_bounds(spec.vocab, world)
    for s, (a, e) in zip(shards, bounds):
        assert s["vp"] and s["off"] == a and s["lm_q"].shape[0] == e - a
    assert torch.equal(torch.cat([s["lm_q"] for s in shards]), full.lm_q)
    assert torch.equal(torch.cat([s["lm_s"] for s in shards]), full.lm_s)


def test_vocab_bounds_split_rule():
    from microgen_b200.engine import vocab_bounds
    assert vocab_bounds(128256, 8) == [(r * 16032, (r + 1) * 16032) for r in range(8)]
    assert vocab_bounds(50257, 2) == [(0, 25128), (25128, 50257)]   # remainder on the last rank
    assert vocab_bounds(10, 3) == [(0, 3), (3, 6), (6, 10)]


def _merge_worker(rank, world, port, outdir, vocab, seed):
    from microgen_b200.engine import merge_vocab_argmax, vocab_bounds
    _init(rank, world, port)
    g = torch.Generator().manual_seed(seed)
    b = 6
    full = torch.randint(-3, 4, (b, vocab), generator=g).float()  # small integers: many exact ties
    full[1] = float("-inf")                        # no finite value: torch.argmax gives 0
    full[2, :] = 0.0
    full[2, vocab - 1] = 5.0                       # the maximum in the last rank's shard
    full[3, :] = float("nan")                      # NaN is larger than every number: the first NaN
    full[4, ::3] = float("nan")
    full[5, :] = 1.0
    full[5, vocab - 2] = float("nan")              # the only NaN, in the last rank's shard
    a, e = vocab_bounds(vocab, world)[rank]
    shard = full[:, a:e]
    li = shard.argmax(1)                           # local first maximal column, as the argmax kernel
    val = shard.gather(1, li[:, None])[:, 0]
    got = merge_vocab_argmax(val, (li + a).to(torch.int32), world, dist.group.WORLD)
    torch.save({"got": got, "full": full}, os.path.join(outdir, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,vocab", [(2, 37), (3, 50), (4, 64)])
def test_merge_vocab_argmax_matches_full_argmax(world, vocab):
    """The NCCL-path merge of per-rank (max, global index) pairs equals torch.argmax over the whole row:
    ties across shards go to the first index, -inf rows to 0, a row with NaNs to its first NaN."""
    outs = _run(_merge_worker, world, vocab, 5)
    full = outs[0]["full"]
    want = full.argmax(1).to(torch.int32)
    assert want[5] == vocab - 2 and want[3] == 0
    for o in outs:
        assert torch.equal(o["got"], want), (o["got"], want)

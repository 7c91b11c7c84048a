"""Tensor parallelism across real GPUs (needs >= 2): TP=2 decode through B200TensorParallelBackend,
one process per GPU, against TP=1 on the same seeded model, with the row-parallel reduction either fused
(partials pushed into peer memory by the linear's epilogue, reduced by the next norm kernel) or over NCCL. TP=2 is teacher-forced with the
TP=1 greedy stream: logits must agree within the bf16 tolerance at every step, and the argmax must agree
wherever TP=1's top-1/top-2 margin exceeds that tolerance (TP sums the row-parallel partials in another
order, so only near-ties may flip). Skipped when fewer than two GPUs are visible."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = dict(family="llama", hidden=512, layers=2, heads=8, kv_heads=4, head_dim=64, inter=1024, vocab=1024,
             eps=1e-5, rope_theta=500000.0)
N_NEW = 24
PG_TIMEOUT = datetime.timedelta(seconds=120)  # ranks that wait on a dead peer end with an error


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(be, prompts, forced=None):
    """Greedy decode (or, with ``forced``, feed those tokens); returns (tokens, logits per step, the
    backend's greedy token per step). The greedy token comes from the step's device argmax (distributed
    over the vocab shards at TP > 1); it must be the first maximal index of the returned logits."""
    logits, cache = be.prefill(torch.tensor(prompts))
    toks, lgs, greedy = [], [logits.float().cpu().numpy()], []
    for i in range(N_NEW + 1):
        gt = be.sample(logits)
        greedy.append(gt[:, 0].cpu().tolist())
        if i == N_NEW:
            break
        t = gt if forced is None else torch.tensor(forced[i], device="cuda")[:, None]
        toks.append(t[:, 0].cpu().tolist())
        logits, cache = be.decode(t, cache=cache)
        lgs.append(logits.float().cpu().numpy())
    lgs = np.stack(lgs)
    assert greedy == np.argmax(lgs, axis=-1).tolist()
    return toks, lgs, greedy


def _prompts(shape=SHAPE):
    from tests._hf_models import prompt_ids
    shared = prompt_ids(shape["vocab"], 32, seed=7)
    return [shared + prompt_ids(shape["vocab"], 9, seed=20 + i) for i in range(4)]


def _worker(rank, world, port, outdir, graph, forced, fused, shape=SHAPE, block=False):
    import torch.distributed as dist
    os.environ["MG_FUSED_AR"] = "1" if fused else "0"
    os.environ["MG_BLOCK"] = "1" if block else "0"
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from microgen_b200.backends import B200TensorParallelBackend
    from tests._hf_models import make_hf_model
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=PG_TIMEOUT)
    model, _ = make_hf_model(shape, seed=0)
    be = B200TensorParallelBackend(world_size=world, group=dist.group.WORLD, max_batch=4, max_seq_len=128,
                                   use_cuda_graph=graph, free_list_seed=1)
    be.load_model("tiny", model_instance=model)
    out = _decode(be, _prompts(shape), forced)
    assert (be.engine.comm is not None) == fused
    assert (be.engine.block_args is not None) == block
    assert be.engine.vocab_parallel and be.engine.vocab_local < shape["vocab"]
    be.engine.release_graphs()
    torch.save(out, os.path.join(outdir, f"r{rank}.pt"))
    torch.cuda.synchronize()
    dist.barrier()
    be.engine.close()
    dist.barrier()
    dist.destroy_process_group()


# an odd vocabulary: the last rank's lm_head shard is one row longer
ODD_VOCAB = dict(SHAPE, vocab=1001)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fused,graph,shape,block", [
    (True, False, SHAPE, False), (True, True, SHAPE, False), (False, False, SHAPE, False),
    (False, True, SHAPE, False), (True, True, ODD_VOCAB, False), (False, True, ODD_VOCAB, False),
    (True, True, SHAPE, True)],
    ids=["fused_push-eager", "fused_push-graph", "nccl-eager", "nccl-graph", "fused_push-graph-vocab1001",
         "nccl-graph-vocab1001", "persistent-layer-graph"])
def test_tp2_matches_tp1(graph, fused, shape, block):
    """TP=2 with a vocab-parallel lm_head (each rank streams half of it; the greedy token is merged
    across ranks on the device) against TP=1; the last case runs every layer's linears, norms and
    RoPE / K/V append through the persistent layer kernel, whose row-parallel outputs go to the peers
    from its epilogue and are reduced inside the same launch."""
    import torch.multiprocessing as mp
    from microgen_b200.backends import B200QuantizedBackend
    from tests._hf_models import make_hf_model
    model, _ = make_hf_model(shape, seed=0)
    be = B200QuantizedBackend(max_batch=4, max_seq_len=128, free_list_seed=1, use_cuda_graph=graph)
    be.load_model("tiny", model_instance=model)
    ref_toks, ref_lg, _ = _decode(be, _prompts(shape))
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d, graph, ref_toks, fused, shape, block), nprocs=2, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(2)]
    tol = 1e-2 + 2e-2 * np.abs(ref_lg)
    top2 = np.sort(ref_lg, axis=-1)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 2 * tol.max(axis=-1)
    assert np.array_equal(outs[0][1], outs[1][1])  # every rank returns the same gathered logits
    for toks, lg, _ in outs:
        assert toks == ref_toks  # teacher-forced inputs
        err = np.abs(lg - ref_lg)
        assert not (err > tol).any(), f"max err {err.max():.3e}"
        agree = np.argmax(lg, axis=-1) == np.argmax(ref_lg, axis=-1)
        assert agree[clear].all()
        assert clear.mean() > 0.3  # enough clear-margin steps for the argmax check to mean something


# 16 query / 8 KV heads of 32: whole heads and 64-row gate/up groups on every rank up to TP=8
SHAPE_W = dict(family="llama", hidden=512, layers=2, heads=16, kv_heads=8, head_dim=32, inter=2048, vocab=1024,
               eps=1e-5, rope_theta=500000.0)


@pytest.mark.parametrize("world", [4, 8])
def test_tp_world_matches_tp1(world):
    """TP=4 and TP=8 (fused push: every rank's bf16 partial summed in rank order, so 4 or 8 roundings per
    element; vocab-parallel head) against TP=1, teacher-forced, as test_tp2_matches_tp1. Skipped without
    that many GPUs."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    from microgen_b200.backends import B200QuantizedBackend
    from tests._hf_models import make_hf_model
    model, _ = make_hf_model(SHAPE_W, seed=0)
    be = B200QuantizedBackend(max_batch=4, max_seq_len=128, free_list_seed=1)
    be.load_model("tiny", model_instance=model)
    ref_toks, ref_lg, _ = _decode(be, _prompts(SHAPE_W))
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _port(), d, True, ref_toks, True, SHAPE_W, False), nprocs=world, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(world)]
    tol = 1e-2 + 2e-2 * np.abs(ref_lg)
    top2 = np.sort(ref_lg, axis=-1)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 2 * tol.max(axis=-1)
    for toks, lg, _ in outs:
        assert np.array_equal(lg, outs[0][1])
        err = np.abs(lg - ref_lg)
        assert not (err > tol).any(), f"max err {err.max():.3e}"
        assert (np.argmax(lg, axis=-1) == np.argmax(ref_lg, axis=-1))[clear].all()
    assert clear.mean() > 0.3


def _ref_worker(rank, world, port, outdir, family):
    """TP=world over the reference's fixture model: greedy stream teacher-forced with the reference's tokens."""
    import json
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from microgen_b200.backends import B200TensorParallelBackend
    from tests._hf_models import make_hf_model
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=PG_TIMEOUT)
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"model_{family}.npz"))
    model, _ = make_hf_model(json.loads(str(d["shape"])), seed=0)
    be = B200TensorParallelBackend(world_size=world, group=dist.group.WORLD, max_batch=1, max_seq_len=128)
    be.load_model("tiny", model_instance=model)
    logits, cache = be.prefill(torch.tensor([d["prompt"].tolist()]))
    got, lgs = [], []
    for t in d["tokens"].tolist():
        got.append(int(be.sample(logits)[0, 0]))
        lgs.append(logits[0].float().cpu().numpy())
        logits, cache = be.decode(torch.tensor([[t]], device="cuda"), cache=cache)
    be.engine.release_graphs()
    torch.save((got, np.stack(lgs)), os.path.join(outdir, f"r{rank}.pt"))
    torch.cuda.synchronize()
    dist.barrier()
    be.engine.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("family", ["llama"])  # the tiny Qwen2's 192-wide MLP does not split into 64-row groups
def test_tp2_stream_matches_reference_fixture(family):
    """TP=2 (fused push, vocab-parallel head) against the reference's own greedy stream and first-step logits
    (``model_<family>.npz``, made by ``QuantizedPyTorchBackend``): teacher-forced with the reference's tokens,
    the first logits within the bf16 tolerance and the greedy token equal to the reference's wherever this
    run's top-1 / top-2 margin is clear of that tolerance (partials are summed in bf16 across ranks, so only
    near-ties may flip)."""
    import torch.multiprocessing as mp
    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"model_{family}.npz"))
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_ref_worker, args=(2, _port(), tmp, family), nprocs=2, join=True)
        outs = [torch.load(os.path.join(tmp, f"r{r}.pt"), weights_only=False) for r in range(2)]
    ref_tok, ref_lg = d["tokens"], d["logits"]
    for got, lg in outs:
        tol = 1e-2 + 2e-2 * np.abs(ref_lg)
        assert not (np.abs(lg[:len(ref_lg)] - ref_lg) > tol).any()
        top2 = np.sort(lg, axis=-1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * (1e-2 + 2e-2 * np.abs(lg).max(axis=-1))
        assert (np.array(got) == ref_tok)[clear].all()
        assert clear.mean() > 0.3  # enough clear-margin steps for the token check to mean something
    assert outs[0][0] == outs[1][0]  # every rank samples the same tokens


def _argmax_rows_world(vocab):
    """fp32 rows whose first maximal index needs both shards of a 2-way vocab split (columns [0, vocab//2)
    and [vocab//2, vocab)): ties within and across shards, -inf rows, and NaN (larger than every number
    for torch.argmax) in one shard, both, or everywhere."""
    g = torch.Generator().manual_seed(4)
    full = torch.randint(-3, 4, (8, vocab), generator=g).float()
    h = vocab // 2
    full[1] = float("-inf")
    full[2, :] = 0.0
    full[2, vocab - 1] = 3.0                  # the maximum is the last rank's last column
    full[3, 5] = 100.0
    full[3, h + 200] = float("nan")            # NaN only in the second shard beats a larger number
    full[4, h + 1] = float("nan")
    full[4, 17] = float("nan")                 # NaN in both shards: the first one
    full[5, :] = 1.0
    full[5, 10] = full[5, h + 100] = 9.0       # a tie across shards: the first index
    full[6] = float("nan")
    full[7, :] = 0.0
    full[7, h - 1] = full[7, h] = 2.0          # a tie on both sides of the shard boundary
    return full


def _vocab_argmax_worker(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from microgen_b200 import kernels as K
    from microgen_b200.engine import vocab_bounds
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=PG_TIMEOUT)
    vocab = 1001
    full = _argmax_rows_world(vocab)
    a, e = vocab_bounds(vocab, world)[rank]
    comm = K.Comm(rank, world, 8 * 256, group=dist.group.WORLD)
    got = []
    try:
        wide = torch.zeros((8, e - a + 5), device="cuda")
        wide[:, :e - a] = full[:, a:e].cuda()
        for _ in range(3):  # consecutive exchanges alternate the receive sets
            got.append(K.vocab_argmax(comm, full[:, a:e].cuda(), a).cpu())
            got.append(K.vocab_argmax(comm, wide[:, :e - a], a).cpu())  # a row stride wider than the shard
        K.check_device()
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        comm.close()
    torch.save(got, os.path.join(outdir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_argmax_world2_matches_torch_argmax():
    """``mg_vocab_argmax`` across two GPUs equals torch.argmax over the whole row on every rank: ties across
    shards go to the first index, -inf rows to 0, NaN counts as larger than every number."""
    import torch.multiprocessing as mp
    want = _argmax_rows_world(1001).argmax(1).to(torch.int32)
    assert want.tolist()[1:] == [0, 1000, 700, 17, 10, 0, 499]
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_vocab_argmax_worker, args=(2, _port(), d), nprocs=2, join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(2)]
    for got in outs:
        for g in got:
            assert torch.equal(g.to(torch.int32), want), (g, want)

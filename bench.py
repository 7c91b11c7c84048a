"""Decode-step benchmark: INT8 tensor-parallel linears + paged decode attention on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload llama3b|qwen05b|gpt2]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...   (N > 1, TP = N)
    python bench.py --impl reference ...   (the reference's CPU path, restated as the oracle port)
    python bench.py --sweep c4 [--steps R]  (isolated kernel sweep; torchrun for the sharded cases)

Workload (default): Llama-3.2-3B-shaped decoder (28 layers, hidden 3072, 24/8 heads of 128,
SwiGLU 8192, vocab 128256), random-init N(0, 0.02) weights quantized to INT8 per output
channel, batch 32, prompts of 2048 uniform random ids whose first 1024 are shared (prefilled
once, blocks shared by reference count), block tables from a seeded shuffled free list,
then greedy decode. A step is one decode step of the whole batch (all layers, lm_head,
argmax). ``value`` = batch / device time per step (tokens/s), timed with CUDA events over K
CUDA-graph replays whose mean context equals the decode phase's mean (2048 + 256); the
per-step working set (3.2 GB of weights + 4.8 GB of KV) is far larger than L2, so no flush
is needed. ``e2e`` is the same decode through the backend's public API (host token ids in,
greedy ids out) with the host<->device copies inside the timed region. At N > 1 the line also
carries ``nvlink`` (the step's row-parallel push + reduce launches on their own) and
``baseline_nccl``: the same step, weights, prompts and window with the row-parallel reduction as
an NCCL all_reduce, timed the same way in the same run. ``--kv int8`` stores the KV cache as
int8 codes with per-vector scales (the reference's ``quantize_kv``); the default is bf16.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "llama3b": dict(shape="LLAMA_3B", batch=32, prompt=2048, shared=1024, decode=512),
    "qwen05b": dict(shape="QWEN_05B", batch=16, prompt=1024, shared=0, decode=256),
    "gpt2": dict(shape="GPT2_SMALL", batch=8, prompt=512, shared=0, decode=256),
}
METRIC = "decode tokens/s at 1/2/4/8 B200; INT8 TP-linear HBM GB/s vs roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="llama3b", choices=sorted(WORKLOADS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-nccl", action="store_true", help="N > 1: skip the same-run NCCL-reduce baseline")
    ap.add_argument("--prompt", type=int, default=0, help="override the prompt length (debug)")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small ncu captures)")
    ap.add_argument("--sweep", default="", choices=["", "c4", "scheduler"],
                    help="c4: the isolated INT8-linear and paged-attention kernel sweep, one JSON line per case; "
                         "scheduler: continuous batching throughput, batched decode vs one decode per request")
    ap.add_argument("--kv", default="bf16", choices=["bf16", "int8"],
                    help="KV cache storage: bf16 (the workload's default) or int8 codes with per-vector scales "
                         "(the reference's quantize_kv option)")
    ap.add_argument("--profile", action="store_true",
                    help="ncu mode: KV filled with random values instead of a prefill, no window centering, "
                         "no probe / e2e / CPU legs")
    return ap.parse_args()


def kv_vec_bytes(eng) -> int:
    """Bytes of one K (or V) vector of one token and kv head in the pool: bf16, or int8 codes + an fp32 scale."""
    return eng.D + 4 if eng.pool.quantize else 2 * eng.D


def kernel_chains(eng, spec, b: int, n_shared_blocks: int, kv_tokens: int, reps: int = 10) -> dict:
    """Device time of each hot kernel family on its own: one CUDA graph holding every launch of that
    family in a decode step (the step's weights, pools, shapes and epilogues, back to back as in the
    step; residual adds go to a scratch buffer), replayed ``reps`` times between CUDA events on the
    launch stream. Per family: launches, microseconds per step and per launch, algorithmic bytes
    (INT8 codes + scales + activations in/out; K/V bytes read) and GB/s."""
    import torch
    from microgen_b200 import kernels as K
    w, H = eng.w, spec.hidden
    scratch = torch.zeros((b, H), dtype=torch.float32, device=eng.h.device)
    nqkv = (eng.hq + 2 * eng.hkv) * eng.D
    epi_mlp = K.EPI_GELU_BF16 if spec.family == "gpt2" else K.EPI_SWIGLU_BF16
    lin = []  # (x, q, s, bias, y, epilogue, bytes)
    for L in w.layers:
        lin.append((eng.x[:b], L.qkv_q, L.qkv_s, L.qkv_b, eng.qkv[:b], K.EPI_STORE_F32,
                    eng.linear_bytes(L.qkv_q, b, 4, nqkv)))
        lin.append((eng.attn[:b], L.o_q, L.o_s, None, scratch, K.EPI_ADD_F32, eng.linear_bytes(L.o_q, b, 8, H)))
        lin.append((eng.x[:b], L.gu_q, L.gu_s, L.gu_b, eng.act[:b], epi_mlp,
                    eng.linear_bytes(L.gu_q, b, 2, eng.act.shape[1])))
        lin.append((eng.act[:b], L.d_q, L.d_s, None, scratch, K.EPI_ADD_F32, eng.linear_bytes(L.d_q, b, 8, H)))
    lin.append((eng.x[:b], w.lm_q, w.lm_s, None, eng.logits[:b, :eng.vocab_local], K.EPI_STORE_F32,
                eng.linear_bytes(w.lm_q, b, 4, eng.vocab_local)))
    tab, ctx = eng.tables[:b], eng.ctx[:b]
    attn_bytes = kv_tokens * eng.hkv * kv_vec_bytes(eng) * 2 + b * eng.hq * eng.D * (4 + 2)

    def run_lin():
        for x, q, sc, bias, y, e, _ in lin:
            K.i8_linear(x, q, sc, bias, y=y, epilogue=e, workspace=eng.lin_ws)

    families = [("i8_linear", run_lin, len(lin), sum(t[-1] for t in lin))]
    if eng.block_args is not None:
        # the step's persistent layer launches (every linear, norm and RoPE/KV append of the layers), and
        # the lm_head linear on its own
        def run_block():
            for a in eng.block_args:
                a.m = b
                K.decode_block(a, eng.block_ws, eng.comm)

        head = lin[-1]

        def run_head():
            x, q, sc, bias, y, e, _ = head
            K.i8_linear(x, q, sc, bias, y=y, epilogue=e)

        nb = len(eng.block_args)
        families = [("decode_block", run_block, nb, sum(eng.block_bytes(i, b) for i in range(nb))),
                    ("lm_head", run_head, 1, head[-1])]

    def run_attn():
        for l in range(len(w.layers)):
            K.paged_decode_attn(eng.q[:b], eng.pool.k[l], eng.pool.v[l], tab, ctx, eng.scale,
                                n_shared_blocks=n_shared_blocks, out=eng.attn[:b], workspace=eng.workspace,
                                **eng.pool.scales(l))

    out = {}
    families.append(("paged_attn", run_attn, len(w.layers), attn_bytes * len(w.layers)))
    for name, fn, n, nbytes in families:
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        us = e0.elapsed_time(e1) * 1e3 / reps
        out[name] = {"launches_per_step": n, "us_per_step": round(us, 2), "us_per_launch": round(us / n, 3),
                     "bytes_per_launch": int(nbytes // n), "gbs": round(nbytes / us / 1e3, 1),
                     "timing": f"CUDA graph of the step's {n} {name} launches, {reps} replays, CUDA events"}
    K.check_device()
    return out


def push_chain(eng, spec, b: int, reps: int = 10) -> dict:
    """NVLink traffic of the fused row-parallel all-reduce: one CUDA graph holding a step's row-parallel
    pushes and reduces (o and down projections of every layer, no norm), replayed ``reps`` times after a
    barrier on every rank. Each rank sends every output element of its partial to each peer, two bf16
    values per 8-byte tagged word: egress per GPU per step = layers x 2 x (world - 1) x b x hidden x 4 B."""
    import torch
    import torch.distributed as dist
    from microgen_b200 import kernels as K
    scratch = torch.zeros((b, spec.hidden), dtype=torch.float32, device=eng.h.device)

    def run():
        for L in eng.w.layers:
            K.i8_linear_rowpar(eng.attn[:b], L.o_q, L.o_s, eng.comm, workspace=eng.lin_ws)
            K.rowpar_reduce_norm(eng.comm, scratch, None, K.NORM_NONE)
            K.i8_linear_rowpar(eng.act[:b], L.d_q, L.d_s, eng.comm, workspace=eng.lin_ws)
            K.rowpar_reduce_norm(eng.comm, scratch, None, K.NORM_NONE)

    dist.barrier()
    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    dist.barrier()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    K.check_device()
    us = e0.elapsed_time(e1) * 1e3 / reps
    t = torch.tensor([us], device=eng.h.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())
    n_ar = 2 * len(eng.w.layers)
    egress = n_ar * (eng.world - 1) * b * spec.hidden * 4
    return {"all_reduces_per_step": n_ar, "us_per_step": round(us, 2), "egress_bytes_per_step": egress,
            "achieved_gbs": round(egress / us / 1e3, 1), "peak_gbs": 770.0, "peak_source": "measured peer copy",
            "nominal_gbs": 900.0, "frac": round(egress / us / 1e3 / 770.0, 4),
            "timing": f"CUDA graph of the step's {n_ar} row-parallel push linears + reduce kernels, {reps} "
                      "replays, CUDA events, max over ranks (linear compute included)"}


C4_LINEAR = [(3072, 9216), (3072, 8192), (8192, 3072), (4096, 14336)]  # (K, N)
C4_M = [1, 8, 32, 128, 256]
C4_ATTN = dict(hq=32, hkv=8, d=128, ctx=[512, 2048, 8192, 32768], batch=[1, 16, 64])


def _timed(fn, reps: int, flush) -> float:
    """Mean device microseconds of ``fn()``: each launch follows an L2 flush (a read of a buffer larger
    than L2) and sits between two CUDA events on the launch stream; ``fn`` must do no host synchronisation."""
    import torch
    st = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    fn()
    torch.cuda.synchronize()
    for a, b in evs:
        flush.sum()  # read (not write) the buffer: L2 is left holding clean lines of it
        a.record(st)
        fn()
        b.record(st)
    torch.cuda.synchronize()
    return 1e3 * sum(a.elapsed_time(b) for a, b in evs) / reps


def sweep_scheduler(args) -> None:
    """Continuous batching on one GPU, the workload's model shape: 48 requests with prompts of 192-320 ids
    (a 128-id prefix shared by half of them), 48 new tokens each, greedy, at most 32 running. Two runs over
    the same requests and backend: ``BatchedScheduler`` (one decode step for all running requests) and the
    reference scheduler's decode loop (``scheduler.py:199-226``: one ``decode`` + ``sample`` per running
    request and step, batch 1), both with the same admission and prefill. Wall-clock tokens/s of generated
    tokens, prefill included; one JSON line per run."""
    import torch
    from microgen_b200 import model_spec as MS
    from microgen_b200.backends import B200QuantizedBackend
    from microgen_b200.scheduler import BatchedScheduler, Request, RequestStatus
    from microgen_b200.synthetic import SyntheticState
    torch.cuda.set_device(0)
    wl = dict(WORKLOADS[args.workload])
    shape = dict(getattr(MS, wl["shape"]))
    if args.layers:
        shape["layers"] = args.layers
    spec = MS.ModelSpec(**shape)
    n_req, new, max_run = 48, 48, 32
    be = B200QuantizedBackend(max_batch=max_run, max_seq_len=512, num_blocks=max_run * 24 + 64, free_list_seed=0,
                              prefix_cache_capacity=8)
    be.load_state(spec, SyntheticState(spec, seed=0, device=torch.device("cuda", 0)))
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, spec.vocab, (128,), generator=g).tolist()

    def requests():
        out = []
        for i in range(n_req):
            n = 192 + (i * 37) % 129
            ids = torch.randint(0, spec.vocab, (n,), generator=g).tolist()
            if i % 2 == 0:
                ids[:128] = shared
            out.append(Request(request_id=f"r{i}", prompt="", prompt_ids=ids, max_new_tokens=new, temperature=0.0))
        return out

    class Batched(BatchedScheduler):
        decode_s = 0.0

        def _decode(self, reqs):
            t0 = time.perf_counter()
            done = super()._decode(reqs)
            self.decode_s += time.perf_counter() - t0  # the sampled ids reached the host inside
            return done

    class PerRequest(Batched):
        """The reference scheduler's decode loop: every running request decoded on its own (batch 1)."""

        def _decode(self, reqs):
            t0 = time.perf_counter()
            done = []
            for r in list(reqs):
                self._batch.tables = [self._tables[r.request_id]]
                self._batch.n_shared_blocks = 0
                self._batch.mirror = None
                lg, _ = self.backend.decode(torch.tensor([[r.generated_token_ids[-1]]]), cache=self._batch)
                done += self._finish([r], self._sample_rows([r], lg))
            self.decode_batch_sizes.append(1)
            self.decode_s += time.perf_counter() - t0
            return done

    for name, cls in (("batched", Batched), ("per_request", PerRequest), ("batched", Batched)):
        reqs = requests()
        sch = cls(be, max_batch_size=max_run)
        for r in reqs:
            sch.add_request(r)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        sch.run_until_complete()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert all(r.status == RequestStatus.COMPLETED for r in reqs)
        toks = sum(len(r.generated_token_ids) for r in reqs)
        print(json.dumps({"sweep": "scheduler", "scheduler": name, "workload": f"{args.workload} shape "
                          f"({spec.layers} layers), {n_req} requests, prompts 192-320 (128 shared by half), "
                          f"{new} new tokens each, <= {max_run} running", "generated_tokens": toks,
                          "seconds": round(dt, 3), "tokens_per_s": round(toks / dt, 1),
                          "decode_seconds": round(sch.decode_s, 3),
                          "decode_tokens_per_s": round((toks - n_req) / sch.decode_s, 1),
                          "decode_steps": len(sch.decode_batch_sizes),
                          "mean_decode_batch": round(sum(sch.decode_batch_sizes) / max(1, len(sch.decode_batch_sizes)), 2),
                          "profile_ms": {k: round(v, 1) for k, v in sch.get_profile_breakdown().items()}}), flush=True)


def sweep_c4(args) -> None:
    """Isolated kernel sweep (one JSON line per configuration):

    * INT8 linear, (K, N) x M: W N(0, 0.02) quantized per output channel on the device, x bf16 N(0, 1).
      At N GPUs (torchrun) each rank runs its column-parallel shard (N/world output rows) and its
      row-parallel shard (K/world input columns) with the fused peer-memory all-reduce (push + reduce),
      and the same row-parallel partial followed by an NCCL all_reduce (the baseline), max over ranks.
      At one GPU the column and row shards are the whole matrix; the tensor-core kernel (tile-packed codes)
      and the CUDA-core GEMV (row-major codes) are both timed.
    * Paged decode attention: 32 query / 8 KV heads, head_dim 128, bf16 K/V N(0, 1), shuffled block tables,
      the first half of each sequence's blocks shared by the batch (read once per batch).
    Algorithmic bytes: linear K*N codes + 4N scales + 2MK x + 2MN y; attention the unique K/V bytes + q + out."""
    import torch
    import torch.distributed as dist
    from microgen_b200 import kernels as K
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    hbm, hbm_kind = peaks()
    flush = torch.ones(80 << 20, dtype=torch.float32, device=dev)  # 320 MB
    reps = max(3, args.steps)
    g = torch.Generator(device=dev).manual_seed(0)

    def emit(d):
        if rank == 0:
            print(json.dumps(d), flush=True)

    def maxrank(us):
        if world == 1:
            return us
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    comm = None
    if world > 1:
        comm = K.Comm(rank, world, max(C4_M) * max(n for _, n in C4_LINEAR))
    skws = K.sk_workspace(128, dev)  # stream-K form for M <= 128 (larger M runs the cluster kernel)
    for k, n in C4_LINEAR:
        w = torch.randn((n, k), generator=g, device=dev).mul_(0.02)
        q, s = K.quantize_rows_i8(w)
        del w
        qp = K.pack_weights(q)
        ncol, krow = n // world, k // world
        qc = K.pack_weights(q[rank * ncol:(rank + 1) * ncol].contiguous()) if world > 1 else qp
        sc = s[rank * ncol:(rank + 1) * ncol].contiguous() if world > 1 else s
        qr_rm = q[:, rank * krow:(rank + 1) * krow].contiguous() if world > 1 else q
        qr = K.pack_weights(qr_rm) if world > 1 else qp
        for m in C4_M:
            x = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            line = {"sweep": "c4_linear", "K": k, "N": n, "M": m, "world": world,
                    "bytes": k * n + 4 * n + 2 * m * k + 2 * m * n, "peak_gbs": hbm, "peak_source": hbm_kind,
                    "l2": "flushed before every launch"}
            if world == 1:
                us_sk = _timed(lambda: K.i8_linear(x, qp, s, y=y, epilogue=K.EPI_STORE_BF16, workspace=skws), reps,
                               flush) if skws is not None else None
                us_tc = _timed(lambda: K.i8_linear(x, qp, s, y=y, epilogue=K.EPI_STORE_BF16), reps, flush)
                us_simt = _timed(lambda: K.i8_linear(x, q, s, y=y, epilogue=K.EPI_STORE_BF16, algo="simt"), reps,
                                 flush)
                for name, us in (("tc_streamk", us_sk), ("tc", us_tc), ("simt", us_simt)):
                    if us is None:
                        continue
                    gbs = line["bytes"] / us / 1e3
                    line[name] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4)}
            else:
                xc = x
                yc = torch.empty((m, ncol), dtype=torch.bfloat16, device=dev)
                us_col = maxrank(_timed(lambda: K.i8_linear(xc, qc, sc, y=yc, epilogue=K.EPI_STORE_BF16), reps,
                                        flush))
                xr = x[:, rank * krow:(rank + 1) * krow]
                h = torch.zeros((m, n), dtype=torch.float32, device=dev)

                def fused():
                    K.i8_linear_rowpar(xr, qr, s, comm)
                    K.rowpar_reduce_norm(comm, h, None, K.NORM_NONE)

                def nccl():
                    K.i8_linear(xr, qr, s, y=h, epilogue=K.EPI_STORE_F32)
                    dist.all_reduce(h)

                dist.barrier()
                us_fused = maxrank(_timed(fused, reps, flush)) if n % 128 == 0 and n <= 8192 else None
                dist.barrier()
                us_nccl = maxrank(_timed(nccl, reps, flush))
                col_bytes = k * ncol + 4 * ncol + 2 * m * k + 2 * m * ncol
                row_bytes = krow * n + 4 * n + 2 * m * krow + 4 * m * n
                line.update({"column": {"us": round(us_col, 2), "gbs_per_rank": round(col_bytes / us_col / 1e3, 1)},
                             "row_fused": None if us_fused is None else
                             {"us": round(us_fused, 2), "gbs_per_rank": round(row_bytes / us_fused / 1e3, 1),
                              "nvlink_egress_bytes": (world - 1) * m * n * 4},
                             "row_nccl": {"us": round(us_nccl, 2), "gbs_per_rank": round(row_bytes / us_nccl / 1e3, 1)},
                             "timing": "max over ranks of per-rank CUDA-event means"})
            emit(line)
        del q, qp, qc, qr, qr_rm
    if comm is not None:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
    # ---- attention (every rank runs the same single-GPU cases; rank 0 reports)
    import random
    hq, hkv, d = C4_ATTN["hq"], C4_ATTN["hkv"], C4_ATTN["d"]
    for ctx in C4_ATTN["ctx"]:
        for b in C4_ATTN["batch"]:
            nb = (ctx + 15) // 16
            ns = nb // 2
            nblocks = ns + b * (nb - ns)
            order = list(range(nblocks))
            random.Random(ctx * 131 + b).shuffle(order)
            tables = torch.empty((b, nb), dtype=torch.int32)
            tables[:, :ns] = torch.tensor(order[:ns], dtype=torch.int32)
            for i in range(b):
                tables[i, ns:] = torch.tensor(order[ns + i * (nb - ns):ns + (i + 1) * (nb - ns)], dtype=torch.int32)
            kp = torch.randn((nblocks, hkv, 16, d), generator=g, device=dev).to(torch.bfloat16)
            vp = torch.randn((nblocks, hkv, 16, d), generator=g, device=dev).to(torch.bfloat16)
            qq = torch.randn((b, hq, d), generator=g, device=dev)
            tab = tables.to(dev)
            ctxs = torch.full((b,), ctx, dtype=torch.int32, device=dev)
            out = torch.empty((b, hq * d), dtype=torch.bfloat16, device=dev)
            ws = torch.zeros(max(16, K.attn_workspace_bytes(b, hq, hkv, d, nb, ns)), dtype=torch.uint8, device=dev)
            us = _timed(lambda: K.paged_decode_attn(qq, kp, vp, tab, ctxs, d ** -0.5, n_shared_blocks=ns, out=out,
                                                    workspace=ws, validate=False), reps, flush)
            nbytes = (ns * 16 + b * (ctx - ns * 16)) * hkv * d * 2 * 2 + b * hq * d * (4 + 2)
            gbs = nbytes / us / 1e3
            emit({"sweep": "c4_attention", "ctx": ctx, "batch": b, "hq": hq, "hkv": hkv, "d": d,
                  "shared_blocks": ns, "bytes": nbytes, "us": round(us, 2), "gbs": round(gbs, 1),
                  "frac": round(gbs / hbm, 4), "peak_gbs": hbm, "peak_source": hbm_kind,
                  "l2": "flushed before every launch"})
            del kp, vp
    K.check_device()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid, self.proc, self.path = uuid, None, None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def host_threads() -> int:
    """Give torch's CPU ops every host CPU this process may run on (torchrun sets OMP_NUM_THREADS=1 in its
    workers, which would time the CPU legs on one thread) and return that count."""
    import torch
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def cpu_baseline(spec, wl, ctx, budget_s=20.0) -> dict:
    from oracle.cpu_baseline import measure
    host_threads()
    r = measure(spec.hidden, spec.heads, spec.kv_heads, spec.head_dim, spec.inter, spec.vocab, spec.layers,
                wl["batch"], ctx, budget_s=budget_s, eps=spec.eps, theta=spec.rope_theta)
    return {"value": round(r["tokens_per_s"], 4), "unit": "tokens/s", "cores": r["threads"], "kind": "port",
            "sample": (f"torch CPU fp32 restatement of the reference CPU decode step (its ops: dequantize-per-call "
                       f"linears, cat-grown cache, SDPA; within 0.8-1.15x of the reference's own decode step time on "
                       f"the same cores) at the full {wl['shape']} shape, batch {wl['batch']}, ctx {ctx}: "
                       f"{r['layers_timed']} single-layer steps timed ({r['layer_s']:.3f} s each) + lm_head "
                       f"({r['head_s']:.3f} s); step = {spec.layers} x layer + head = {r['step_s']:.2f} s")}


def workload_config(name: str, wl: dict, world: int) -> dict:
    """The workload both arms report (identical keys and values): model shape, batch, prompt, shared
    prefix, decode length and the mean context of the timed window."""
    mean_ctx = wl["prompt"] + wl["decode"] // 2
    return {"workload": f"{name}: {wl['shape']} INT8, batch {wl['batch']}, prompt {wl['prompt']} "
                        f"({wl['shared']} shared), decode {wl['decode']}; timed at mean ctx {mean_ctx}",
            "batch": wl["batch"], "prompt": wl["prompt"], "shared_prefix": wl["shared"], "decode": wl["decode"],
            "mean_ctx": mean_ctx, "tp": world, "parallelism": f"tp{world}"}


def run_reference(args) -> None:
    """The reference arm: the reference's decode path is Python on the host CPU (fp32, dequantize-per-call
    linears, cat-grown cache); its torch CPU restatement (the oracle port) runs WHOLE decode steps of the
    workload on the host cores, warm-up then as many timed steps as fit in the time budget, and the line
    reports the steps it actually timed. Under torchrun only rank 0 runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from microgen_b200 import model_spec as MS
    from oracle.cpu_baseline import measure_steps
    host_threads()
    wl = WORKLOADS[args.workload]
    spec = MS.ModelSpec(**getattr(MS, wl["shape"]))
    ctx = wl["prompt"] + wl["decode"] // 2
    budget = float(os.environ.get("MG_REFERENCE_BUDGET_S", "60"))
    r = measure_steps(spec.hidden, spec.heads, spec.kv_heads, spec.head_dim, spec.inter, spec.vocab, spec.layers,
                      wl["batch"], ctx, budget_s=budget, max_steps=max(1, args.steps), warmup=1, eps=spec.eps,
                      theta=spec.rope_theta)
    v = round(r["tokens_per_s"], 4)
    sample = (f"torch CPU fp32 restatement of the reference CPU decode step (its ops: dequantize-per-call linears, "
              f"cat-grown cache, SDPA; within 0.8-1.15x of the reference's own decode step time on the same cores) "
              f"at the full {wl['shape']} shape, batch {wl['batch']}, ctx {ctx}: {r['steps']} whole "
              f"steps ({spec.layers} layers + lm_head) timed after {r['warmup']} warm-up step, "
              f"{r['timed_s']:.1f} s; {args.steps} requested, bounded by a {budget:.0f} s budget")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": r["steps"], "warmup": r["warmup"], "ms_per_step": round(1000.0 * r["step_s"], 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.workload, wl, args.gpus),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": r["threads"], "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


T0 = time.time()


def log(msg: str) -> None:
    """Progress line on stderr (rank-tagged), so a stalled run shows its phase."""
    print(f"[bench r{os.environ.get('RANK', '0')} +{time.time() - T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def random_fill(be, prompts, n_shared):
    """Profile mode: block tables as a prefill would leave them (shared prefix by reference
    count), the KV pool filled with seeded random bf16 values instead of computed K/V."""
    import torch
    from microgen_b200.backends.b200 import PagedKVCache
    b, p = prompts.shape
    cache = PagedKVCache(be.allocator)
    if n_shared:
        cache.prefix = be.allocator.allocate_sequence("prefix", n_shared * 16)
        cache.tables = [be.allocator.share_prefix(cache.prefix, n_shared, f"seq{i}", p) for i in range(b)]
    else:
        cache.tables = [be.allocator.allocate_sequence(f"seq{i}", p) for i in range(b)]
    cache.n_shared_blocks = n_shared
    pool = be.engine.pool
    g = torch.Generator(device=pool.k.device).manual_seed(2)
    for t in (pool.k, pool.v):
        for l in range(t.shape[0]):
            if pool.quantize:  # int8 codes; scales as a unit-normal vector would get
                t[l].copy_(torch.randint(-127, 128, t[l].shape, generator=g, device=t.device, dtype=torch.int8))
            else:
                t[l].normal_(generator=g)
    if pool.quantize:
        pool.k_scale.fill_(3.0 / 127)
        pool.v_scale.fill_(3.0 / 127)
    return cache


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.sweep == "c4":
        sweep_c4(args)
        return
    if args.sweep == "scheduler":
        sweep_scheduler(args)
        return
    import torch
    import torch.distributed as dist

    from microgen_b200 import _lib
    from microgen_b200 import kernels as K
    from microgen_b200 import model_spec as MS
    from microgen_b200.backends import B200QuantizedBackend, B200TensorParallelBackend
    from microgen_b200.synthetic import SyntheticState

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        group = dist.group.WORLD

    wl = dict(WORKLOADS[args.workload])
    if args.prompt:
        wl["prompt"], wl["shared"] = args.prompt, min(wl["shared"], args.prompt // 2)
    shape = dict(getattr(MS, wl["shape"]))
    if args.layers:
        shape["layers"] = args.layers
    spec = MS.ModelSpec(**shape)
    B, P, S, Dec = wl["batch"], wl["prompt"], wl["shared"], wl["decode"]
    W, Kst = args.warmup, args.steps
    skip = 0 if args.profile else max(0, Dec // 2 - W - Kst // 2)
    run = skip + W + Kst
    max_seq = P + max(Dec, run) + 16
    max_blocks = (max_seq + 15) // 16
    n_shared = S // 16
    num_blocks = n_shared + B * (max_blocks - n_shared) + 16

    kw = dict(max_batch=B, max_seq_len=max_seq, num_blocks=num_blocks, free_list_seed=0,
              quantize_kv=args.kv == "int8")
    be = (B200TensorParallelBackend(world_size=world, group=group, **kw) if world > 1
          else B200QuantizedBackend(**kw))
    t0 = time.time()
    log(f"loading {wl['shape']} tp={world}")
    be.load_state(spec, SyntheticState(spec, seed=0, device=torch.device("cuda", local)))
    torch.cuda.synchronize()
    t_load = time.time() - t0
    eng = be.engine
    reduce_kind = ("fused peer-memory push" if eng.comm is not None else
                   ("nccl all_reduce" if world > 1 else "none (tp1)"))

    g = torch.Generator().manual_seed(1)
    shared = torch.randint(0, spec.vocab, (S,), generator=g)
    prompts = torch.stack([torch.cat([shared, torch.randint(0, spec.vocab, (P - S,), generator=g)])
                           for _ in range(B)])
    t0 = time.time()
    log("prefill")
    if args.profile:
        cache = random_fill(be, prompts, n_shared)
        first = prompts[:, -1].to(torch.int32)
    else:
        logits, cache = be.prefill(prompts)
        first = be.sample(logits)[:, 0].to(torch.int32).cpu()
    torch.cuda.synchronize()
    t_prefill = time.time() - t0

    log("decode: capture + timed replays")
    # ---- device-timed decode: graph replays, inputs resident, device-side advance --------------
    alloc = be.allocator
    for t in cache.tables:
        for _ in range(run + 1):
            alloc.append_token(t)
    from microgen_b200.runtime.paged_kv import block_table_tensor
    tab = block_table_tensor(cache.tables, eng.max_blocks)
    slots = [t.slot(P) for t in cache.tables]
    eng.set_inputs(first.tolist(), [P] * B, slots, [P + 1] * B, tab)
    before = _lib.LAUNCHES[0]
    graph = eng.capture(B, cache.n_shared_blocks, advance=True)
    per_step_launches = _lib.LAUNCHES[0] - before
    # capture() ran one warm-up step (not advanced); the launch count of capture = warm-up + graph
    per_step_launches //= 2
    for _ in range(skip + W):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    except Exception:
        pass
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuid) as clk:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(Kst):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / Kst
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = B / (ms / 1e3)
    mean_pos = P + skip + W + (Kst - 1) / 2.0
    kv_tokens = n_shared * 16 + B * (int(mean_pos) + 1 - n_shared * 16)

    if args.profile:
        del graph  # a graph holding NCCL calls must be gone before the process group is destroyed
        eng.release_graphs()
        if rank == 0:
            print(json.dumps({"profile": args.workload, "ms_per_step": round(ms, 4), "value": round(value, 1)}))
        if world > 1:
            torch.cuda.synchronize()
            dist.barrier()
            eng.close()
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---- per-kernel device time (probe pass: CUDA events on the launch stream around each launch;
    # a short spin kernel ahead of each launch keeps the host's launch latency out of the interval)
    stats: dict = {}

    class Probe:
        def __init__(self, kind, nbytes):
            self.kind, self.nbytes = kind, nbytes

        def __enter__(self):
            torch.cuda._sleep(40000)
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            self.a.record(torch.cuda.current_stream())

        def __exit__(self, *e):
            self.b.record(torch.cuda.current_stream())
            stats.setdefault(self.kind, []).append((self.a, self.b, self.nbytes))

    log("per-kernel probe")
    pos = int(mean_pos)
    eng.set_inputs(first.tolist(), [pos] * B, [t.slot(pos) for t in cache.tables], [pos + 1] * B, tab)
    for rep in range(4):
        if rep == 1:
            stats.clear()
        eng.forward(B, cache.n_shared_blocks, probe=Probe, kv_tokens=kv_tokens)
    torch.cuda.synchronize()
    kernels = {}
    for kind, recs in stats.items():
        tsum = sum(a.elapsed_time(b) for a, b, _ in recs) / 1e3
        bsum = sum(n for _, _, n in recs)
        kernels[kind] = {"launches_per_step": len(recs) // 3, "us_per_step": round(tsum / 3 * 1e6, 2),
                         "gbs": round(bsum / tsum / 1e9, 1)}
    hbm, hbm_kind = peaks()
    log("kernel chains")
    chains = kernel_chains(eng, spec, B, cache.n_shared_blocks, kv_tokens)
    nvlink = None
    if eng.comm is not None:
        log("nvlink push chain")
        nvlink = push_chain(eng, spec, B)
    dom = max(chains, key=lambda k: chains[k]["us_per_step"])
    achieved = chains[dom]["gbs"]
    # DRAM bytes per launch: the committed capture's DRAM / algorithmic ratio for this kernel family times this
    # run's algorithmic bytes per launch (the capture ran at TP=1 on a 2-layer cut of the same shapes)
    traffic = None
    tr_path = os.path.join(ROOT, "profiles", "traffic_per_launch.txt")
    if os.path.exists(tr_path):
        try:
            tr = json.load(open(tr_path)).get(f"{args.workload}:{dom}")
            if tr:
                traffic = int(round(tr["dram_bytes"] / tr["algorithmic_bytes"] * chains[dom]["bytes_per_launch"]))
        except Exception:
            traffic = None
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": hbm_kind,
                "algorithmic_bytes_per_launch": chains[dom]["bytes_per_launch"],
                "us_per_launch": chains[dom]["us_per_launch"], "timing": chains[dom]["timing"]}
    step_bytes = eng.w.int8_bytes() + kv_tokens * eng.hkv * kv_vec_bytes(eng) * 2 * spec.layers
    step_roofline = {"bytes_per_step": step_bytes, "achieved_gbs": round(step_bytes / (ms / 1e3) / 1e9, 1),
                     "frac": round(step_bytes / (ms / 1e3) / 1e9 / hbm, 4)}

    # ---- end to end through the public API (host ids in, host ids out) -------------------------
    e2e = None
    log("e2e")
    if not args.no_e2e:
        for t in cache.tables:
            alloc.rollback(t, t.num_tokens - (P + skip))
        tok = first[:, None].to(torch.int64)
        for _ in range(W):
            lg, cache = be.decode(tok, cache=cache)
            tok = be.sample(lg).cpu()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for _ in range(Kst):
            lg, cache = be.decode(tok, cache=cache)
            tok = be.sample(lg).cpu()
        f1.record()
        torch.cuda.synchronize()
        ems = f0.elapsed_time(f1) / Kst
        if world > 1:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(B / (ems / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": eng.h2d_bytes,
               "d2h_bytes_per_step": B * 8, "ms_per_step": round(ems, 4)}
    K.check_device()

    # ---- same-run NCCL baseline (N > 1): the same step with the row-parallel reduction as an NCCL
    # all_reduce (store-or-add) instead of the fused peer push, device-timed the same way
    nccl = None
    if world > 1 and eng.comm is not None and not args.no_nccl:
        log("nccl baseline")
        os.environ["MG_FUSED_AR"] = "0"
        be2 = B200TensorParallelBackend(world_size=world, group=group, **kw)
        be2.load_state(spec, SyntheticState(spec, seed=0, device=torch.device("cuda", local)))
        eng2 = be2.engine
        lg2, cache2 = be2.prefill(prompts)
        first2 = be2.sample(lg2)[:, 0].to(torch.int32).cpu()
        for t in cache2.tables:
            for _ in range(run + 1):
                be2.allocator.append_token(t)
        tab2 = block_table_tensor(cache2.tables, eng2.max_blocks)
        eng2.set_inputs(first2.tolist(), [P] * B, [t.slot(P) for t in cache2.tables], [P + 1] * B, tab2)
        g2 = eng2.capture(B, cache2.n_shared_blocks, advance=True)
        for _ in range(skip + W):
            g2.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0.record(stream)
        for _ in range(Kst):
            g2.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / Kst], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms2 = float(t.item())
        nccl = {"value": round(B / (ms2 / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms2, 4),
                "row_parallel_reduce": "nccl all_reduce (store-or-add), same weights / prompts / window",
                "fused_over_nccl": round(ms2 / ms, 3),
                "timing": f"CUDA graph of one step, {Kst} replays, CUDA events, max over ranks"}
        del g2
        eng2.release_graphs()
        del be2, eng2, cache2, lg2
        os.environ["MG_FUSED_AR"] = "1"

    cpu = None
    log("cpu baseline / report")
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(spec, wl, P + Dec // 2, budget_s=20.0)

    del graph  # a graph holding NCCL calls must be gone before the process group is destroyed
    eng.release_graphs()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        eng.close()  # peers are done writing into this rank's receive area
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": Kst,
        "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 weights x bf16 activations, fp32 accumulate", "data": "synthetic",
        "config": dict(workload_config(args.workload, wl, world), **({"kv": "int8"} if args.kv == "int8" else {})),
        "setup": {"l2": "working set per step >> L2 (no flush needed)", "cuda_graph": True,
                  "row_parallel_reduce": reduce_kind,
                  "linear_kernel": ("persistent layer kernel (decode_block) + cluster split-K lm_head"
                                    if eng.block_args is not None else
                                    "stream-K" if eng.lin_ws is not None else "cluster split-K"),
                  "timed_window_mean_ctx": round(mean_pos + 1)},
        "roofline": roofline, "step_roofline": step_roofline, "kernel_chains": chains, "nvlink": nvlink,
        "kernels": kernels,
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": per_step_launches * Kst, "baseline_nccl": nccl,
        "clocks": clk.summary(), "setup_s": {"load": round(t_load, 1), "prefill": round(t_prefill, 1)},
    }
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

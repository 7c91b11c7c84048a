"""Decode engine: one decode step of a Llama / Qwen2 / GPT-2 model as a sequence of
libmicrogen_b200 kernel launches over device-resident INT8 weights and a paged KV pool.

This is what runs inside ``backend.decode`` (``microgen/backends/pytorch.py:118-142``)
once the backend has swapped in the INT8 tensor-parallel linears:

    embed → per layer: norm → QKV (column-parallel INT8 linear) → RoPE + paged KV
    append → paged decode attention → o_proj (row-parallel INT8 linear, residual
    add, all-reduce) → norm → gate/up with fused SwiGLU (or c_fc with GELU) →
    down (row-parallel, residual add, all-reduce) → final norm → lm_head → argmax

Weights are quantized on the device with the bit-exact per-channel kernel from the
FULL fp32 matrices, then sharded (column: rows and scales split per head group;
row: input columns split, scales replicated), so codes at TP=N equal codes at TP=1.
The residual stream stays fp32; activations entering a linear are bf16; K/V are bf16.

Row-parallel linears reduce with the "store-or-add" trick: rank 0 adds its partial
(and the bias) into the residual in place, the other ranks overwrite their copy
with their partial, and one in-place sum all-reduce of the residual completes
``h + Σ partials`` — no extra kernel on the path.
"""

from __future__ import annotations

import contextlib
import math
import os
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import kernels as K
from .model_spec import ModelSpec
from .runtime.paged_kv import PagedKVPool


@dataclass
class LayerWeights:
    ln1_w: torch.Tensor
    ln1_b: Optional[torch.Tensor]
    qkv_q: torch.Tensor
    qkv_s: torch.Tensor
    qkv_b: Optional[torch.Tensor]
    o_q: torch.Tensor
    o_s: torch.Tensor
    o_b: Optional[torch.Tensor]
    ln2_w: torch.Tensor
    ln2_b: Optional[torch.Tensor]
    gu_q: torch.Tensor
    gu_s: torch.Tensor
    gu_b: Optional[torch.Tensor]
    d_q: torch.Tensor
    d_s: torch.Tensor
    d_b: Optional[torch.Tensor]


@dataclass
class ModelWeights:
    embed: torch.Tensor
    wpe: Optional[torch.Tensor]
    norm_w: torch.Tensor
    norm_b: Optional[torch.Tensor]
    lm_q: torch.Tensor
    lm_s: torch.Tensor
    layers: list = field(default_factory=list)
    # vocab-parallel lm_head: this rank holds rows [lm_offset, lm_offset + lm_s.numel()) of the full head
    vocab_parallel: bool = False
    lm_offset: int = 0

    def nbytes(self) -> int:
        n = 0
        for t in [self.embed, self.wpe, self.norm_w, self.norm_b, self.lm_q, self.lm_s]:
            n += 0 if t is None else t.numel() * t.element_size()
        for L in self.layers:
            for t in vars(L).values():
                n += 0 if t is None else t.numel() * t.element_size()
        return n

    def int8_bytes(self) -> int:
        """Weight bytes a decode step streams: int8 codes + fp32 scales of every linear."""
        n = self.lm_q.shape[0] * self.lm_q.shape[1] + 4 * self.lm_s.numel()
        for L in self.layers:
            for q, s in ((L.qkv_q, L.qkv_s), (L.o_q, L.o_s), (L.gu_q, L.gu_s), (L.d_q, L.d_s)):
                n += q.shape[0] * q.shape[1] + 4 * s.numel()
        return n


def _interleave_gate_up(gq, gs, uq, us, gb=None, ub=None):
    """Rows grouped as [64 gate rows, the 64 matching up rows] per 128 (the SwiGLU epilogue layout)."""
    i, k = gq.shape
    if i % 64:
        raise ValueError(f"intermediate size per rank ({i}) must be a multiple of 64")
    q = torch.stack([gq.view(i // 64, 64, k), uq.view(i // 64, 64, k)], dim=1).reshape(2 * i, k).contiguous()
    s = torch.stack([gs.view(i // 64, 64), us.view(i // 64, 64)], dim=1).reshape(2 * i).contiguous()
    b = None
    if gb is not None or ub is not None:
        gb = gb if gb is not None else torch.zeros_like(gs)
        ub = ub if ub is not None else torch.zeros_like(us)
        b = torch.stack([gb.view(i // 64, 64), ub.view(i // 64, 64)], dim=1).reshape(2 * i).contiguous()
    return q, s, b


def row_parallel_residual(h: torch.Tensor, launch, rank: int, world: int, group=None) -> None:
    """Row-parallel linear folded into the fp32 residual ``h`` (replicated on every rank).

    ``launch(y, epilogue)`` runs this rank's partial linear into ``y`` with the given epilogue.
    Rank 0 adds its partial (and the bias) into ``h`` in place; every other rank overwrites its copy of
    ``h`` with its partial; one in-place sum all-reduce then leaves ``h + Σ partials`` on every rank —
    the reference's ``sum(partial_outputs) + bias`` (``parallel.py:65-81``) added to the residual."""
    launch(h, K.EPI_ADD_F32 if rank == 0 else K.EPI_STORE_F32)
    if world > 1:
        torch.distributed.all_reduce(h, group=group)


def vocab_bounds(vocab: int, world: int) -> list[tuple[int, int]]:
    """[start, end) of each rank's lm_head rows: the reference's split rule for sharded linears
    (``N // world`` rows per rank, the last rank taking the remainder; ``parallel.py:19-24``)."""
    per = vocab // world
    return [(r * per, (r + 1) * per if r < world - 1 else vocab) for r in range(world)]


def merge_vocab_argmax(val: torch.Tensor, gidx: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Global greedy token of a vocab-parallel lm_head over a process group (the NCCL form of
    ``mg_vocab_argmax``): ``val`` fp32 [b] and ``gidx`` int32 [b] are this rank's maximal logit and its global
    column. All ranks' pairs are gathered; each row takes the largest value (NaN above every number) and, on
    ties, the lowest rank, whose columns come first — torch.argmax's first maximal index over the whole row
    (``pytorch.py:153-155``), as the local argmax kernel keeps it within a shard."""
    import torch.distributed as dist
    rec = torch.stack([val.contiguous().view(torch.int32), gidx.to(torch.int32)], 1)
    parts = [torch.empty_like(rec) for _ in range(world)]
    dist.all_gather(parts, rec, group=group)
    allr = torch.stack(parts)                                   # [world, b, 2]
    vals = allr[..., 0].contiguous().view(torch.float32)
    r = vals.argmax(0)                                          # first maximal rank (NaN first, as torch)
    return allr[r, torch.arange(allr.shape[1], device=allr.device), 1]


class WeightLoader:
    """Quantize full fp32 matrices on the device and keep this rank's shard.

    ``quantize`` maps an fp32 [N, K] weight to (int8 codes, fp32 scales) — the bit-exact device kernel
    by default; ``pack`` repacks the kept codes into the tile-packed layout. ``vocab_parallel`` keeps only
    this rank's rows of lm_head (``vocab_bounds``); otherwise lm_head is replicated, as in the reference."""

    def __init__(self, spec: ModelSpec, device, rank: int = 0, world: int = 1, pack: bool = True, quantize=None,
                 vocab_parallel: bool = False):
        self.spec, self.device, self.rank, self.world, self.pack = spec, torch.device(device), rank, world, pack
        self.vocab_parallel = bool(vocab_parallel) and world > 1
        self.quantize = quantize or K.quantize_rows_i8
        if spec.heads % world or spec.kv_heads % world:
            raise ValueError(f"{spec.heads} query / {spec.kv_heads} kv heads do not split over {world} ranks")

    def f32(self, t) -> torch.Tensor:
        return t.detach().to(device=self.device, dtype=torch.float32).contiguous()

    def quant(self, w_out_in) -> tuple[torch.Tensor, torch.Tensor]:
        return self.quantize(self.f32(w_out_in))

    def rows(self, t, n_total):
        per = n_total // self.world
        return t[self.rank * per:(self.rank + 1) * per].contiguous()

    def cols(self, q, k_total):
        per = k_total // self.world
        return q[:, self.rank * per:(self.rank + 1) * per].contiguous()

    def bias(self, b):
        return None if b is None else self.f32(b)

    def load(self, state: dict) -> ModelWeights:
        s = self.spec
        D = s.head_dim
        qn, kn = s.heads * D, s.kv_heads * D
        g = lambda k: state[k] if k in state else None
        layers = []
        gpt2 = s.family == "gpt2"
        for i in range(s.layers):
            if gpt2:
                p = f"transformer.h.{i}."
                wqkv = g(p + "attn.c_attn.weight").t()
                bqkv = g(p + "attn.c_attn.bias")
                wq, wk, wv = wqkv[:qn], wqkv[qn:qn + kn], wqkv[qn + kn:]
                bq, bk, bv = (None, None, None) if bqkv is None else (bqkv[:qn], bqkv[qn:qn + kn], bqkv[qn + kn:])
                wo, bo = g(p + "attn.c_proj.weight").t(), g(p + "attn.c_proj.bias")
                wfc, bfc = g(p + "mlp.c_fc.weight").t(), g(p + "mlp.c_fc.bias")
                wd, bd = g(p + "mlp.c_proj.weight").t(), g(p + "mlp.c_proj.bias")
                ln1 = (g(p + "ln_1.weight"), g(p + "ln_1.bias"))
                ln2 = (g(p + "ln_2.weight"), g(p + "ln_2.bias"))
            else:
                p = f"model.layers.{i}."
                wq, wk, wv = (g(p + f"self_attn.{n}_proj.weight") for n in "qkv")
                bq, bk, bv = (g(p + f"self_attn.{n}_proj.bias") for n in "qkv")
                wo, bo = g(p + "self_attn.o_proj.weight"), g(p + "self_attn.o_proj.bias")
                wg, wu = g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")
                bg, bu = g(p + "mlp.gate_proj.bias"), g(p + "mlp.up_proj.bias")
                wd, bd = g(p + "mlp.down_proj.weight"), g(p + "mlp.down_proj.bias")
                ln1 = (g(p + "input_layernorm.weight"), None)
                ln2 = (g(p + "post_attention_layernorm.weight"), None)
            # column-parallel QKV: each projection quantized whole, then this rank's head rows
            parts_q, parts_s, parts_b = [], [], []
            for w_, b_, n_ in ((wq, bq, qn), (wk, bk, kn), (wv, bv, kn)):
                q_, s_ = self.quant(w_)
                parts_q.append(self.rows(q_, n_))
                parts_s.append(self.rows(s_, n_))
                parts_b.append(self.rows(self.f32(b_), n_) if b_ is not None else None)
            qkv_b = None
            if any(b is not None for b in parts_b):
                qkv_b = torch.cat([b if b is not None else torch.zeros_like(sq) for b, sq in zip(parts_b, parts_s)])
            # row-parallel o / down: full-matrix scales replicated, input columns split
            o_q, o_s = self.quant(wo)
            d_q, d_s = self.quant(wd)
            if gpt2:
                fq, fs = self.quant(wfc)
                gu_q, gu_s = self.rows(fq, s.inter), self.rows(fs, s.inter)
                gu_b = self.rows(self.f32(bfc), s.inter) if bfc is not None else None
            else:
                gq, gs = self.quant(wg)
                uq, us = self.quant(wu)
                gu_q, gu_s, gu_b = _interleave_gate_up(
                    self.rows(gq, s.inter), self.rows(gs, s.inter), self.rows(uq, s.inter), self.rows(us, s.inter),
                    self.rows(self.f32(bg), s.inter) if bg is not None else None,
                    self.rows(self.f32(bu), s.inter) if bu is not None else None)
            layers.append(LayerWeights(
                ln1_w=self.f32(ln1[0]), ln1_b=self.bias(ln1[1]),
                qkv_q=torch.cat(parts_q).contiguous(), qkv_s=torch.cat(parts_s).contiguous(), qkv_b=qkv_b,
                o_q=self.cols(o_q, qn), o_s=o_s, o_b=self.bias(bo),
                ln2_w=self.f32(ln2[0]), ln2_b=self.bias(ln2[1]),
                gu_q=gu_q, gu_s=gu_s, gu_b=gu_b,
                d_q=self.cols(d_q, s.inter), d_s=d_s, d_b=self.bias(bd)))
        if gpt2:
            embed, wpe = self.f32(state["transformer.wte.weight"]), self.f32(state["transformer.wpe.weight"])
            norm_w, norm_b = self.f32(state["transformer.ln_f.weight"]), self.f32(state["transformer.ln_f.bias"])
            head = state.get("lm_head.weight", state["transformer.wte.weight"])
        else:
            embed, wpe = self.f32(state["model.embed_tokens.weight"]), None
            norm_w, norm_b = self.f32(state["model.norm.weight"]), None
            head = state.get("lm_head.weight", state["model.embed_tokens.weight"])
        lm_q, lm_s = self.quant(head)
        lm_off = 0
        if self.vocab_parallel:
            lm_off, end = vocab_bounds(lm_q.shape[0], self.world)[self.rank]
            lm_q, lm_s = lm_q[lm_off:end].contiguous(), lm_s[lm_off:end].contiguous()
        w = ModelWeights(embed=embed, wpe=wpe, norm_w=norm_w, norm_b=norm_b, lm_q=lm_q, lm_s=lm_s, layers=layers,
                         vocab_parallel=self.vocab_parallel, lm_offset=lm_off)
        if self.pack:
            w.lm_q = K.pack_weights(w.lm_q)
            for L in layers:
                for name in ("qkv_q", "o_q", "gu_q", "d_q"):
                    setattr(L, name, K.pack_weights(getattr(L, name)))
        return w


def rope_table(head_dim: int, theta: float, max_pos: int) -> torch.Tensor:
    """fp32 [max_pos, head_dim]: cos of the head_dim/2 frequencies, then sin — computed as HF's
    default rotary embedding does (fp32 inv_freq, fp32 angle, fp32 cos/sin)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float32)
    ang = pos[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).contiguous()


class DecodeEngine:
    """Device state of one rank: weights, paged KV pool, step buffers, captured graphs."""

    def __init__(self, spec: ModelSpec, weights: ModelWeights, device, max_batch: int, num_blocks: int,
                 max_blocks_per_seq: int, rank: int = 0, world: int = 1, group=None, max_pos: int = 0,
                 quantize_kv: bool = False):
        self.spec, self.w, self.device = spec, weights, torch.device(device)
        self.rank, self.world, self.group = rank, world, group
        self.hq, self.hkv, self.D = spec.heads // world, spec.kv_heads // world, spec.head_dim
        self.inter = spec.inter // world
        self.max_batch, self.max_blocks = max_batch, max_blocks_per_seq
        self.max_ctx = max_blocks_per_seq * 16
        # quantize_kv: int8 K/V codes with a per-vector scale (the reference's KVCacheState(quantize_kv=True))
        self.pool = PagedKVPool(spec.layers, num_blocks, self.hkv, self.D, self.device, quantize=quantize_kv)
        self.scale = 1.0 / math.sqrt(self.D)
        dev = self.device
        if spec.family == "gpt2":
            self.cos_sin = None
        else:
            self.cos_sin = rope_table(self.D, spec.rope_theta, max(max_pos, self.max_ctx)).to(dev)
        B, H = max_batch, spec.hidden
        i32 = dict(dtype=torch.int32, device=dev)
        # step inputs in one device buffer (one host-to-device copy per step):
        # tokens | positions | slots | ctx | tables [B, max_blocks]
        self.inputs = torch.zeros(4 * B + B * max_blocks_per_seq, **i32)
        self.tokens, self.positions, self.slots, self.ctx = (self.inputs[i * B:(i + 1) * B] for i in range(4))
        self.ctx.fill_(1)
        self.tables = self.inputs[4 * B:].view(B, max_blocks_per_seq)
        self.next_tokens = torch.zeros(B, **i32)
        self.h = torch.zeros((B, H), dtype=torch.float32, device=dev)
        self.x = torch.zeros((B, H), dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros((B, (self.hq + 2 * self.hkv) * self.D), dtype=torch.float32, device=dev)
        self.q = torch.zeros((B, self.hq, self.D), dtype=torch.float32, device=dev)
        self.attn = torch.zeros((B, self.hq * self.D), dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros((B, self.inter), dtype=torch.bfloat16, device=dev)
        # logits: the full vocab, or with a vocab-parallel lm_head this rank's columns in a buffer as wide as
        # the widest shard (so the shards of all ranks gather into one [world, B, width] tensor)
        self.vocab_parallel = weights.vocab_parallel
        self.vocab_local = weights.lm_s.numel()
        width = max(e - s_ for s_, e in vocab_bounds(spec.vocab, world)) if self.vocab_parallel else spec.vocab
        self.logits = torch.zeros((B, width), dtype=torch.float32, device=dev)
        ws = max(K.attn_workspace_bytes(b, self.hq, self.hkv, self.D, max_blocks_per_seq, ns)
                 for b in {1, max_batch} for ns in {0, max_blocks_per_seq})
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)  # tickets start at zero
        # pinned host staging for step inputs: tokens, positions, slots, ctx, then the table
        self.stage = torch.zeros(4 * B + B * max_blocks_per_seq, dtype=torch.int32, pin_memory=True)
        self.stage_np = self.stage.numpy()
        self.graphs: dict = {}
        self._pf: Optional[dict] = None  # prefill buffers, sized on first use
        # MG_STREAMK=1 runs the linears on the stream-K kernel (one wave of CTAs, equal weight bytes each;
        # it needs a zero-filled workspace for partial tiles); the default is the cluster split-K kernel,
        # which measured faster in the decode step (A/B in the same run)
        self.lin_ws = None
        if isinstance(weights.lm_q, K.PackedWeight) and os.environ.get("MG_STREAMK", "0") == "1":
            self.lin_ws = K.sk_workspace(max_batch, dev)
        # TP > 1: row-parallel linears push their partials straight into every rank's memory and a
        # fused reduce(+norm) kernel finishes the all-reduce (MG_FUSED_AR=0 falls back to NCCL).
        self.comm = None
        # (the push epilogue works on whole 128-row output tiles: hidden % 128 == 0, else NCCL)
        if world > 1 and self.fused_allreduce_choice(group) and isinstance(weights.lm_q, K.PackedWeight) \
                and spec.hidden % 128 == 0 and spec.hidden <= 8192:
            self.comm = K.Comm(rank, world, max_batch * spec.hidden, group=group)
        # MG_BLOCK=1: the persistent layer kernel (one launch per layer boundary: o_proj, norm, MLP, norm,
        # QKV + RoPE + KV append) where its shapes allow. Off by default: on the Llama-3.2-3B workload it
        # measured slower than the kernel-per-op step (bound by its tensor-core issue rate at 32 tokens and by
        # the activation reads at each phase start).
        self.block_args = None
        if self.block_supported(world):
            self._init_block()

    def block_supported(self, world: int) -> bool:
        s, w = self.spec, self.w
        if os.environ.get("MG_BLOCK", "0") != "1" or not isinstance(w.lm_q, K.PackedWeight) or self.pool.quantize:
            return False
        if self.max_batch > K.BLOCK_MAX_TOKENS or s.hidden % 128 or self.D not in (32, 64, 128):
            return False
        if world > 1 and self.comm is None:
            return False
        L = w.layers[0]
        return L.gu_q.shape[0] % 128 == 0 and L.o_q.shape[1] % 16 == 0 and L.d_q.shape[1] % 16 == 0

    def _init_block(self) -> None:
        """One mg_block_args per layer boundary: [0] = input norm + QKV of layer 0; [l+1] = o_proj, MLP and
        the next input norm (the final norm after the last layer) + the next layer's QKV."""
        s, w, dev = self.spec, self.w, self.device
        B, H = self.max_batch, s.hidden
        self.x2 = torch.zeros((B, H), dtype=torch.bfloat16, device=dev)
        norm = K.NORM_LAYER if s.family == "gpt2" else K.NORM_RMS
        mlp = K.EPI_GELU_BF16 if s.family == "gpt2" else K.EPI_SWIGLU_BF16
        ptr = lambda t: 0 if t is None else t.data_ptr()
        nL = len(w.layers)
        args = []
        for i in range(nL + 1):
            a = K.BlockArgs()
            a.m, a.hidden, a.hq, a.hkv, a.head_dim = B, H, self.hq, self.hkv, self.D
            a.norm, a.mlp, a.eps = norm, mlp, float(s.eps)
            a.h, a.attn, a.x2, a.act, a.x1 = ptr(self.h), ptr(self.attn), ptr(self.x2), ptr(self.act), ptr(self.x)
            a.positions, a.slots, a.q_out = ptr(self.positions), ptr(self.slots), ptr(self.q)
            if self.cos_sin is not None:
                a.cos_sin, a.max_pos = ptr(self.cos_sin), self.cos_sin.shape[0]
            flags = 0
            if i > 0:  # o_proj + MLP of layer i-1
                P = w.layers[i - 1]
                flags |= K.BLK_O | K.BLK_MLP
                a.o = K.block_linear(P.o_q, P.o_s, P.o_b)
                a.gate_up = K.block_linear(P.gu_q, P.gu_s, P.gu_b)
                a.down = K.block_linear(P.d_q, P.d_s, P.d_b)
                a.n2_w, a.n2_b = ptr(P.ln2_w), ptr(P.ln2_b)
            flags |= K.BLK_N1
            if i < nL:  # input norm + QKV of layer i
                N = w.layers[i]
                flags |= K.BLK_QKV
                a.n1_w, a.n1_b = ptr(N.ln1_w), ptr(N.ln1_b)
                a.qkv = K.block_linear(N.qkv_q, N.qkv_s, N.qkv_b)
                a.k_pool, a.v_pool = ptr(self.pool.k[i]), ptr(self.pool.v[i])
                a.num_blocks = self.pool.k[i].shape[0]
            else:      # final norm (lm_head input)
                a.n1_w, a.n1_b = ptr(w.norm_w), ptr(w.norm_b)
            a.flags = flags
            args.append(a)
        need = max(K.block_workspace_bytes(a) for a in args)
        self.block_ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        self.block_args = args

    def block_bytes(self, i: int, b: int) -> int:
        """Algorithmic bytes of block launch ``i`` at batch ``b``: INT8 codes + scales of its linears, the
        activations each linear reads (bf16) and writes, the residual read and written per norm."""
        w, H = self.w, self.spec.hidden
        n = 0
        if i > 0:
            P = w.layers[i - 1]
            n += self.linear_bytes(P.o_q, b, 8, H) + self.linear_bytes(P.gu_q, b, 2, self.act.shape[1])
            n += self.linear_bytes(P.d_q, b, 8, H) + b * H * 6
        n += b * H * 6
        if i < len(w.layers):
            N = w.layers[i]
            nq = (self.hq + 2 * self.hkv) * self.D
            n += self.linear_bytes(N.qkv_q, b, 0, nq) + b * self.hq * self.D * 4 + b * 2 * self.hkv * self.D * 2
        return n

    @staticmethod
    def rank0_flag(name: str, group=None) -> bool:
        """Environment switch ``name`` (on unless set to "0") as the group's first rank sees it, broadcast so
        every rank takes the same path even when their environments differ (a mix of paths would wait on
        pushes that never come)."""
        want = [os.environ.get(name, "1") != "0"]
        import torch.distributed as dist
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(want, src=src, group=group)
        return bool(want[0])

    @classmethod
    def fused_allreduce_choice(cls, group=None) -> bool:
        """Whether the row-parallel linears reduce through the fused peer-memory push (MG_FUSED_AR unset or
        not "0") or NCCL."""
        return cls.rank0_flag("MG_FUSED_AR", group)

    # ---- the step -----------------------------------------------------------------------------
    def _norm(self, h, w, b, x):
        if self.spec.family == "gpt2":
            K.layernorm(h, w, b, self.spec.eps, x=x)
        else:
            K.rmsnorm(h, w, self.spec.eps, x=x)

    @staticmethod
    def linear_bytes(q: torch.Tensor, m: int, out_bytes: int, n_out: int) -> int:
        """Algorithmic bytes of one INT8 linear launch: codes + scales + x (bf16) + y."""
        n, k = q.shape
        return n * k + 4 * n + 2 * m * k + out_bytes * m * n_out

    def forward(self, b: int, n_shared_blocks: int = 0, compute_logits: bool = True, probe=None,
                kv_tokens: int = 0) -> None:
        """One decode step for the first ``b`` rows of the input buffers (tokens, positions,
        slots, ctx, tables). Writes logits[:b] and next_tokens[:b] when compute_logits.

        ``probe(kind, algorithmic_bytes)`` — optional context-manager factory wrapped around
        each launch (per-kernel timing); ``kv_tokens`` is the unique KV token count the
        attention launches read (for the probe's byte count)."""
        s, w = self.spec, self.w
        h, x = self.h[:b], self.x[:b]
        tab, ctx = self.tables[:b], self.ctx[:b]
        P = probe if probe is not None else (lambda kind, nbytes: contextlib.nullcontext())
        H, D = s.hidden, self.D
        nqkv = (self.hq + 2 * self.hkv) * D
        kv_vec = D + 4 if self.pool.quantize else 2 * D  # one K or V vector: bf16, or int8 codes + a scale
        attn_bytes = kv_tokens * self.hkv * kv_vec * 2 + b * self.hq * D * (4 + 2)
        with P("embed", b * H * 8):
            K.embed(self.tokens[:b], self.positions[:b], w.embed, w.wpe, h)
        if self.block_args is not None:
            comm = self.comm
            for i, a in enumerate(self.block_args):
                if i > 0:
                    l = i - 1
                    with P("paged_attn", attn_bytes):
                        K.paged_decode_attn(self.q[:b], self.pool.k[l], self.pool.v[l], tab, ctx, self.scale,
                                            n_shared_blocks=n_shared_blocks, out=self.attn[:b],
                                            workspace=self.workspace, validate=False, **self.pool.scales(l))
                a.m = b
                with P("decode_block", self.block_bytes(i, b)):
                    K.decode_block(a, self.block_ws, comm)
            if compute_logits:
                self._head(b, P)
            return
        fused = self.comm is not None
        norm_kind = K.NORM_LAYER if s.family == "gpt2" else K.NORM_RMS
        push_bytes = b * H * 4 * self.world
        if fused:  # later norms come out of the fused reduce of the preceding row-parallel linear
            with P("norm", b * H * 6):
                self._norm(h, w.layers[0].ln1_w, w.layers[0].ln1_b, x)
        for l, L in enumerate(w.layers):
            if not fused:
                with P("norm", b * H * 6):
                    self._norm(h, L.ln1_w, L.ln1_b, x)
            with P("i8_linear", self.linear_bytes(L.qkv_q, b, 4, nqkv)):
                K.i8_linear(x, L.qkv_q, L.qkv_s, L.qkv_b, y=self.qkv[:b], epilogue=K.EPI_STORE_F32,
                            workspace=self.lin_ws)
            with P("rope_kv_append", b * nqkv * 4 + b * self.hq * D * 4 + b * 2 * self.hkv * D * 2):
                K.rope_kv_append(self.qkv[:b], self.positions[:b], self.cos_sin, self.slots[:b], self.hq,
                                 self.hkv, self.D, self.pool.k[l], self.pool.v[l], q_out=self.q[:b],
                                 **self.pool.scales(l))
            with P("paged_attn", attn_bytes):
                K.paged_decode_attn(self.q[:b], self.pool.k[l], self.pool.v[l], tab, ctx, self.scale,
                                    n_shared_blocks=n_shared_blocks, out=self.attn[:b], workspace=self.workspace,
                                    validate=False, **self.pool.scales(l))
            if fused:
                with P("i8_linear", self.linear_bytes(L.o_q, b, 0, H) + push_bytes):
                    K.i8_linear_rowpar(self.attn[:b], L.o_q, L.o_s, self.comm, workspace=self.lin_ws)
                with P("rowpar_reduce", push_bytes + b * H * 10):
                    K.rowpar_reduce_norm(self.comm, h, L.o_b, norm_kind, L.ln2_w, L.ln2_b, s.eps, x)
            else:
                bias_o = L.o_b if self.rank == 0 else None
                with P("i8_linear", self.linear_bytes(L.o_q, b, 8, H)):
                    row_parallel_residual(h, lambda y, e: K.i8_linear(self.attn[:b], L.o_q, L.o_s, bias_o, y=y,
                                                                      epilogue=e, workspace=self.lin_ws),
                                          self.rank, self.world, self.group)
                with P("norm", b * H * 6):
                    self._norm(h, L.ln2_w, L.ln2_b, x)
            epi_mlp = K.EPI_GELU_BF16 if s.family == "gpt2" else K.EPI_SWIGLU_BF16
            with P("i8_linear", self.linear_bytes(L.gu_q, b, 2, self.act.shape[1])):
                K.i8_linear(x, L.gu_q, L.gu_s, L.gu_b, y=self.act[:b], epilogue=epi_mlp, workspace=self.lin_ws)
            if fused:
                nxt_w, nxt_b = ((w.layers[l + 1].ln1_w, w.layers[l + 1].ln1_b) if l + 1 < len(w.layers)
                                else (w.norm_w, w.norm_b))
                with P("i8_linear", self.linear_bytes(L.d_q, b, 0, H) + push_bytes):
                    K.i8_linear_rowpar(self.act[:b], L.d_q, L.d_s, self.comm, workspace=self.lin_ws)
                with P("rowpar_reduce", push_bytes + b * H * 10):
                    K.rowpar_reduce_norm(self.comm, h, L.d_b, norm_kind, nxt_w, nxt_b, s.eps, x)
            else:
                bias_d = L.d_b if self.rank == 0 else None
                with P("i8_linear", self.linear_bytes(L.d_q, b, 8, H)):
                    row_parallel_residual(h, lambda y, e: K.i8_linear(self.act[:b], L.d_q, L.d_s, bias_d, y=y,
                                                                      epilogue=e, workspace=self.lin_ws),
                                          self.rank, self.world, self.group)
        if compute_logits:
            if not fused:
                with P("norm", b * H * 6):
                    self._norm(h, w.norm_w, w.norm_b, x)
            self._head(b, P)

    def _head(self, b: int, P) -> None:
        """lm_head on x (this rank's rows of it when vocab-parallel) and the greedy token of every row."""
        w, nl = self.w, self.vocab_local
        lg = self.logits[:b, :nl]
        with P("i8_linear", self.linear_bytes(w.lm_q, b, 4, nl)):
            K.i8_linear(self.x[:b], w.lm_q, w.lm_s, None, y=lg, epilogue=K.EPI_STORE_F32, workspace=self.lin_ws)
        with P("argmax", b * nl * 4):
            if not self.vocab_parallel:
                K.argmax_rows(lg, out=self.next_tokens[:b])
            elif self.comm is not None:
                K.vocab_argmax(self.comm, lg, w.lm_offset, out=self.next_tokens[:b])
            else:
                idx = K.argmax_rows(lg, out=self.next_tokens[:b])
                val = lg.gather(1, idx.long()[:, None])[:, 0]
                self.next_tokens[:b] = merge_vocab_argmax(val, idx + w.lm_offset, self.world, self.group)

    def full_logits(self, b: int) -> torch.Tensor:
        """fp32 [b, vocab] logits of the last step with logits, as a new tensor (every rank gets the whole
        vocab: with a vocab-parallel lm_head the shards are gathered over the process group)."""
        if not self.vocab_parallel:
            return self.logits[:b].clone()
        import torch.distributed as dist
        mine = self.logits[:b]
        width = mine.shape[1]
        allv = torch.empty((self.world, b, width), dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(allv, mine, group=self.group)
        bounds = vocab_bounds(self.spec.vocab, self.world)
        if all(e - s_ == width for s_, e in bounds):  # equal shards: one transposing copy
            return allv.transpose(0, 1).reshape(b, self.spec.vocab)
        return torch.cat([allv[r, :, :e - s_] for r, (s_, e) in enumerate(bounds)], 1)

    # ---- prefill: many positions per launch ------------------------------------------------------
    PREFILL_CHUNK = 64

    def _prefill_buffers(self, rows: int, width: int) -> dict:
        pf = self._pf
        if pf is not None and pf["rows"] >= rows and pf["width"] >= width:
            return pf
        rows = max(rows, pf["rows"] if pf else 0)
        width = max(width, pf["width"] if pf else 0)
        self._pf = None
        s, dev, H = self.spec, self.device, self.spec.hidden
        n_in = 4 * rows + rows * width
        pf = dict(rows=rows, width=width,
                  h=torch.empty((rows, H), dtype=torch.float32, device=dev),
                  x=torch.empty((rows, H), dtype=torch.bfloat16, device=dev),
                  qkv=torch.empty((rows, (self.hq + 2 * self.hkv) * self.D), dtype=torch.float32, device=dev),
                  q=torch.empty((rows, self.hq, self.D), dtype=torch.float32, device=dev),
                  attn=torch.empty((rows, self.hq * self.D), dtype=torch.bfloat16, device=dev),
                  act=torch.empty((rows, self.inter), dtype=torch.bfloat16, device=dev),
                  inputs=torch.empty(n_in, dtype=torch.int32, device=dev),
                  stage=torch.empty(n_in, dtype=torch.int32, pin_memory=True),
                  ws=torch.zeros(16, dtype=torch.uint8, device=dev))
        pf["stage_np"] = pf["stage"].numpy()
        self._pf = pf
        return pf

    def prefill(self, ids, tables, start: int, end: int, compute_logits: bool = True,
                chunk: Optional[int] = None) -> None:
        """Positions [start, end) of ``b = len(ids)`` prompts, ``chunk`` positions of every prompt per pass
        (the prefill form of ``PyTorchBackend.prefill``, ``pytorch.py:90-116``, which runs the whole prompt
        in one forward): each linear runs once per pass on all b × chunk tokens (the tcgen05 kernel with
        up to 256 tokens per tile), RoPE + K/V append writes every token's slot, and causal attention runs
        per prompt on the decode kernel — the pass's queries share every block before the pass (read once
        for all of them), and each query reads its own tail up to its position. ``ids[s][p]`` is token p of
        prompt s; ``tables`` int32 [b, >= ceil(end/16)] already hold blocks for those positions. With
        ``compute_logits``, writes logits[:b] and next_tokens[:b] of position end - 1."""
        s, w = self.spec, self.w
        b = len(ids)
        C = int(chunk or self.PREFILL_CHUNK)
        tab = np.asarray(tables, dtype=np.int32)
        if tab.ndim != 2 or tab.shape[0] != b or tab.shape[1] * 16 < end or C < 1:
            raise ValueError("prefill needs one table per prompt covering every position")
        ids = np.asarray([list(r[start:end]) for r in ids], dtype=np.int32).reshape(b, end - start)
        epi_mlp = K.EPI_GELU_BF16 if s.family == "gpt2" else K.EPI_SWIGLU_BF16
        D = self.D
        for c0 in range(start, end, C):
            c1 = min(c0 + C, end)
            L = c1 - c0
            M, wc = b * L, (c1 + 15) // 16
            pf = self._prefill_buffers(M, wc)
            torch.cuda.current_stream(self.device).synchronize()  # the staging buffer may still be in flight
            st = pf["stage_np"]
            pos = np.arange(c0, c1, dtype=np.int32)
            st[:M] = ids[:, c0 - start:c1 - start].ravel()
            st[M:2 * M] = np.tile(pos, b)
            st[2 * M:3 * M] = (tab[:, pos // 16] * 16 + pos % 16).ravel()
            st[3 * M:4 * M] = np.tile(pos + 1, b)
            st[4 * M:4 * M + M * wc] = np.repeat(tab[:, :wc], L, axis=0).ravel()
            n = 4 * M + M * wc
            inp = pf["inputs"]
            inp[:n].copy_(pf["stage"][:n], non_blocking=True)
            tok, posd, slots, ctx = (inp[i * M:(i + 1) * M] for i in range(4))
            tabd = inp[4 * M:n].view(M, wc)
            n_sh = c0 // 16 if L > 1 else 0
            ws_need = K.attn_workspace_bytes(L, self.hq, self.hkv, D, wc, n_sh)
            if ws_need > pf["ws"].numel():
                pf["ws"] = torch.zeros(ws_need, dtype=torch.uint8, device=self.device)
            h, x, qkv, q, attn, act = (pf[k][:M] for k in ("h", "x", "qkv", "q", "attn", "act"))
            K.embed(tok, posd, w.embed, w.wpe, h)
            for l, Lw in enumerate(w.layers):
                self._norm(h, Lw.ln1_w, Lw.ln1_b, x)
                K.i8_linear(x, Lw.qkv_q, Lw.qkv_s, Lw.qkv_b, y=qkv, epilogue=K.EPI_STORE_F32)
                K.rope_kv_append(qkv, posd, self.cos_sin, slots, self.hq, self.hkv, D, self.pool.k[l],
                                 self.pool.v[l], q_out=q, **self.pool.scales(l))
                for si in range(b):
                    r = slice(si * L, (si + 1) * L)
                    K.paged_decode_attn(q[r], self.pool.k[l], self.pool.v[l], tabd[r], ctx[r], self.scale,
                                        n_shared_blocks=n_sh, out=attn[r], workspace=pf["ws"], validate=False,
                                        **self.pool.scales(l))
                bias_o = Lw.o_b if self.rank == 0 else None
                row_parallel_residual(h, lambda y, e: K.i8_linear(attn, Lw.o_q, Lw.o_s, bias_o, y=y, epilogue=e),
                                      self.rank, self.world, self.group)
                self._norm(h, Lw.ln2_w, Lw.ln2_b, x)
                K.i8_linear(x, Lw.gu_q, Lw.gu_s, Lw.gu_b, y=act, epilogue=epi_mlp)
                bias_d = Lw.d_b if self.rank == 0 else None
                row_parallel_residual(h, lambda y, e: K.i8_linear(act, Lw.d_q, Lw.d_s, bias_d, y=y, epilogue=e),
                                      self.rank, self.world, self.group)
            if compute_logits and c1 == end:
                self.h[:b].copy_(h[L - 1::L])
                self._norm(self.h[:b], w.norm_w, w.norm_b, self.x[:b])
                self._head(b, lambda kind, nbytes: contextlib.nullcontext())

    def set_inputs(self, tokens, positions, slots, ctx, tables) -> int:
        """Stage one step's inputs in pinned host memory and copy them to the device input buffer in
        one asynchronous copy on the current stream. Returns the batch size; also records the
        host-to-device bytes of the step in ``self.h2d_bytes``."""
        b = len(tokens)
        if b > self.max_batch:
            raise ValueError(f"batch {b} > max_batch {self.max_batch}")
        t = np.asarray(tables, dtype=np.int32)
        if t.ndim != 2 or t.shape[0] != b:
            raise ValueError("tables must be [batch, blocks]")
        w = t.shape[1]
        if w > self.max_blocks:
            raise ValueError(f"block table of {w} blocks > {self.max_blocks}")
        torch.cuda.current_stream(self.device).synchronize()  # the staging buffer may still be in flight
        st = self.stage_np
        B, MB = self.max_batch, self.max_blocks
        for i, v in enumerate((tokens, positions, slots, ctx)):
            st[i * B:i * B + b] = v
        tab = st[4 * B:4 * B + b * MB].reshape(b, MB)
        tab[:, :w] = t
        tab[:, w:] = 0
        n = 4 * B + b * MB
        self.inputs[:n].copy_(self.stage[:n], non_blocking=True)
        self.h2d_bytes = 4 * n
        return b

    # ---- CUDA graphs -------------------------------------------------------------------------------
    def capture(self, b: int, n_shared_blocks: int = 0, advance: bool = False,
                compute_logits: bool = True) -> torch.cuda.CUDAGraph:
        """Capture one decode step for batch ``b`` (plus, with ``advance``, the device-side
        move to the next position: tokens = argmax, positions/ctx += 1, new slots)."""
        key = (b, n_shared_blocks, advance, compute_logits)
        if key in self.graphs:
            return self.graphs[key]
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.forward(b, n_shared_blocks, compute_logits)  # warm-up: loads kernels, sets attributes
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward(b, n_shared_blocks, compute_logits)
            if advance:
                K.decode_advance(self.tokens[:b], self.next_tokens[:b], self.positions[:b], self.ctx[:b],
                                 self.slots[:b], self.tables[:b])
        self.graphs[key] = g
        return g

    def release_graphs(self) -> None:
        self.graphs.clear()

    def close(self) -> None:
        """Drop the captured graphs and the peer-memory communicator. With TP > 1, call it on every rank
        after a barrier: peers write into this rank's receive area until their last step is done."""
        self.graphs.clear()
        if self.comm is not None:
            torch.cuda.synchronize(self.device)
            self.comm.close()
            self.comm = None

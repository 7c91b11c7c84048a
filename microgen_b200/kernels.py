"""Torch-tensor wrappers over the C ABI (device memory and streams come from torch).

Each wrapper checks dtypes, devices and layout, then launches the kernel on the
current CUDA stream. Tensors must live on a CUDA device; there is no CPU path.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import (EPI_ADD_F32, EPI_GELU_BF16, EPI_STORE_BF16, EPI_STORE_F32,  # noqa: F401
                   EPI_SWIGLU_BF16)

BLOCK_SIZE = 16


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(0 if t is None else t.data_ptr())


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, contiguous: bool = True) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the decode path has no CPU fallback)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def quantize_rows_i8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(codes int8 [N,K], scales fp32 [N]) of an fp32 weight, bit-exact with the reference."""
    _need(w, torch.float32, "w")
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    s = torch.empty((n,), dtype=torch.float32, device=w.device)
    _lib.call("mg_quantize_rows_i8", _ptr(w), n, k, _ptr(q), _ptr(s), _stream())
    return q, s


class PackedWeight:
    """INT8 codes in the tile-packed layout (contiguous 16 KB block per 128x128 tile) with the
    logical [n, k] shape of the row-major codes they were packed from."""
    __slots__ = ("data", "n", "k")

    def __init__(self, data: torch.Tensor, n: int, k: int) -> None:
        self.data, self.n, self.k = data, n, k

    @property
    def shape(self):
        return (self.n, self.k)

    @property
    def device(self):
        return self.data.device

    def numel(self) -> int:
        return self.data.numel()

    def element_size(self) -> int:
        return 1


def packed_bytes(n: int, k: int) -> int:
    return int(_lib.load().mg_i8_packed_bytes(n, k))


def pack_weights(q: torch.Tensor) -> PackedWeight:
    """Row-major int8 codes [n, k] -> tile-packed layout (see include/microgen_b200.h)."""
    _need(q, torch.int8, "q")
    n, k = q.shape
    data = torch.empty(packed_bytes(n, k), dtype=torch.int8, device=q.device)
    _lib.call("mg_i8_pack_weights", _ptr(q), n, k, _ptr(data), _stream())
    return PackedWeight(data, n, k)


def _linear_args(x, q, scales, bias, y, epilogue):
    _need(q.data if isinstance(q, PackedWeight) else q, torch.int8, "q")
    _need(scales, torch.float32, "scales")
    if bias is not None:
        _need(bias, torch.float32, "bias")
    _need(x, torch.bfloat16, "x", contiguous=False)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with unit inner stride")
    n, k = q.shape
    if x.shape[1] != k:
        raise ValueError(f"x has {x.shape[1]} features, weight expects {k}")
    m = x.shape[0]
    if y is None:
        nout = n // 2 if epilogue == EPI_SWIGLU_BF16 else n
        dt = torch.float32 if epilogue in (EPI_STORE_F32, EPI_ADD_F32) else torch.bfloat16
        y = torch.empty((m, nout), dtype=dt, device=x.device)
    want = torch.float32 if epilogue in (EPI_STORE_F32, EPI_ADD_F32) else torch.bfloat16
    _need(y, want, "y", contiguous=False)
    if y.dim() != 2 or y.stride(1) != 1 or y.shape[0] != m:
        raise ValueError("y must be [m, n] with unit inner stride")
    return m, k, n, y


def sk_workspace_bytes(m: int) -> int:
    """Workspace bytes of the stream-K linear for m tokens (0 when m > 128: that path is not used)."""
    return int(_lib.load().mg_i8_linear_sk_workspace_bytes(int(m)))


def sk_workspace(max_m: int, device) -> torch.Tensor | None:
    """A zero-filled workspace that serves every stream-K linear call with m <= max_m on ``device``."""
    need = max([sk_workspace_bytes(m) for m in (1, 17, 33, 65) if m <= max_m] or [0])
    return torch.zeros(need, dtype=torch.uint8, device=device) if need else None


def i8_linear(x, q, scales, bias=None, y=None, epilogue=EPI_STORE_BF16, algo: str = "auto", split_k: int = 0,
              workspace=None):
    """y = epilogue(x · (q·s)ᵀ + bias); returns y. algo: "auto" | "tc" | "simt" (row-major q);
    a PackedWeight q runs the tensor-core kernel on tile-packed codes: the stream-K form when a zero-filled
    ``workspace`` (``sk_workspace``) is given, else the cluster split-K form (``split_k``)."""
    m, k, n, y = _linear_args(x, q, scales, bias, y, epilogue)
    if isinstance(q, PackedWeight):
        if workspace is not None:
            _lib.call("mg_i8_linear_packed_sk", _ptr(x), m, k, x.stride(0), _ptr(q.data), _ptr(scales), _ptr(bias),
                      n, _ptr(y), y.stride(0), int(epilogue), _ptr(workspace),
                      workspace.numel() * workspace.element_size(), _stream())
            return y
        _lib.call("mg_i8_linear_packed", _ptr(x), m, k, x.stride(0), _ptr(q.data), _ptr(scales), _ptr(bias), n,
                  _ptr(y), y.stride(0), int(epilogue), int(split_k), _stream())
        return y
    args = (_ptr(x), m, k, x.stride(0), _ptr(q), _ptr(scales), _ptr(bias), n, _ptr(y), y.stride(0), int(epilogue))
    if algo == "simt":
        _lib.call("mg_i8_linear_simt", *args, _stream())
    elif algo == "tc":
        _lib.call("mg_i8_linear_tc", *args, int(split_k), _stream())
    else:
        _lib.call("mg_i8_linear", *args, _stream())
    return y


def rope_kv_append(qkv, positions, cos_sin, slots, hq, hkv, d, k_pool, v_pool, q_out=None, k_scales=None,
                   v_scales=None):
    """RoPE on q and k, K/V into their paged slots. int8 pools (with ``k_scales`` / ``v_scales`` fp32
    [num_blocks, hkv, 16]) store each K and V vector quantized per vector (``mg_rope_kv_append_kv8``)."""
    _need(qkv, torch.float32, "qkv", contiguous=False)
    _need(slots, torch.int32, "slots")
    b = qkv.shape[0]
    if cos_sin is not None:
        _need(cos_sin, torch.float32, "cos_sin")
        _need(positions, torch.int32, "positions")
    if q_out is None:
        q_out = torch.empty((b, hq, d), dtype=torch.float32, device=qkv.device)
    if k_pool.dtype == torch.int8:
        _need(v_pool, torch.int8, "v_pool")
        _need(k_scales, torch.float32, "k_scales")
        _need(v_scales, torch.float32, "v_scales")
        _lib.call("mg_rope_kv_append_kv8", _ptr(qkv), qkv.stride(0), _ptr(positions), _ptr(cos_sin),
                  0 if cos_sin is None else cos_sin.shape[0], _ptr(slots), b, hq, hkv, d, _ptr(q_out), _ptr(k_pool),
                  _ptr(v_pool), _ptr(k_scales), _ptr(v_scales), k_pool.shape[0], _stream())
        return q_out
    _need(k_pool, torch.bfloat16, "k_pool")
    _need(v_pool, torch.bfloat16, "v_pool")
    _lib.call("mg_rope_kv_append", _ptr(qkv), qkv.stride(0), _ptr(positions), _ptr(cos_sin),
              0 if cos_sin is None else cos_sin.shape[0], _ptr(slots), b, hq, hkv, d, _ptr(q_out), _ptr(k_pool),
              _ptr(v_pool), k_pool.shape[0], _stream())
    return q_out


def attn_workspace_bytes(b, hq, hkv, d, max_blocks, n_shared_blocks=0) -> int:
    out = C.c_size_t(0)
    _lib.call("mg_paged_attn_workspace_bytes", b, hq, hkv, d, max_blocks, n_shared_blocks, C.byref(out))
    return out.value


def paged_decode_attn(q, k_pool, v_pool, block_tables, ctx_lens, scale, n_shared_blocks=0, out=None,
                      workspace=None, validate=True, k_scales=None, v_scales=None):
    """q fp32 [b, hq, d]; pools bf16 [nblk, hkv, 16, d]; tables int32 [b, max_blocks]; ctx int32 [b].
    Returns bf16 [b, hq*d]. ``workspace`` (optional) is allocated when missing or too small.

    With ``n_shared_blocks`` > 0 the first that many entries of every table must equal row 0's (the
    kernel reads the shared blocks once, from row 0); ``validate`` checks this before the launch and raises
    ValueError (a device-to-host read: skipped while a CUDA graph is being captured; callers that check
    their host copy of the tables pass False). The kernel also records MG_ERR_DEVICE when it sees a
    mismatch."""
    _need(q, torch.float32, "q")
    q8 = k_pool.dtype == torch.int8
    if q8:  # INT8 KV: codes + one fp32 scale per (block, kv head, token) vector
        _need(v_pool, torch.int8, "v_pool")
        _need(k_scales, torch.float32, "k_scales")
        _need(v_scales, torch.float32, "v_scales")
    else:
        _need(k_pool, torch.bfloat16, "k_pool")
        _need(v_pool, torch.bfloat16, "v_pool")
    _need(block_tables, torch.int32, "block_tables")
    _need(ctx_lens, torch.int32, "ctx_lens")
    b, hq, d = q.shape
    hkv = k_pool.shape[1]
    max_blocks = block_tables.shape[1]
    if validate and n_shared_blocks > 0 and b > 1 and not torch.cuda.is_current_stream_capturing():
        from .runtime.paged_kv import check_shared_prefix
        check_shared_prefix(block_tables[:, :n_shared_blocks].cpu().numpy(), n_shared_blocks)
    ws = attn_workspace_bytes(b, hq, hkv, d, max_blocks, n_shared_blocks)
    if ws and (workspace is None or workspace.numel() * workspace.element_size() < ws):
        workspace = torch.zeros(ws, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty((b, hq * d), dtype=torch.bfloat16, device=q.device)
    if q8:
        _lib.call("mg_paged_decode_attn_kv8", _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(k_scales), _ptr(v_scales),
                  k_pool.shape[0], _ptr(block_tables), max_blocks, _ptr(ctx_lens), b, hq, hkv, d, n_shared_blocks,
                  float(scale), _ptr(out), _ptr(workspace if ws else None), ws, _stream())
    else:
        _lib.call("mg_paged_decode_attn", _ptr(q), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                  _ptr(block_tables), max_blocks, _ptr(ctx_lens), b, hq, hkv, d, n_shared_blocks, float(scale),
                  _ptr(out), _ptr(workspace if ws else None), ws, _stream())
    if ws:
        _lib.LAUNCHES[0] += 1  # the split-combine kernel
    return out


def embed(tokens, positions, wte, wpe, h):
    _need(tokens, torch.int32, "tokens")
    _need(wte, torch.float32, "wte")
    _need(h, torch.float32, "h")
    max_pos = 0
    if wpe is not None:
        _need(wpe, torch.float32, "wpe")
        _need(positions, torch.int32, "positions")
        max_pos = wpe.shape[0]
    _lib.call("mg_embed", _ptr(tokens), _ptr(positions), _ptr(wte), _ptr(wpe), tokens.shape[0], wte.shape[1],
              wte.shape[0], max_pos, _ptr(h), _stream())
    return h


def rmsnorm(h, w, eps, x=None):
    _need(h, torch.float32, "h")
    _need(w, torch.float32, "w")
    if x is None:
        x = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device)
    _lib.call("mg_rmsnorm", _ptr(h), _ptr(w), h.shape[0], h.shape[1], float(eps), _ptr(x), _stream())
    return x


def layernorm(h, w, b, eps, x=None):
    _need(h, torch.float32, "h")
    if x is None:
        x = torch.empty(h.shape, dtype=torch.bfloat16, device=h.device)
    _lib.call("mg_layernorm", _ptr(h), _ptr(w), _ptr(b), h.shape[0], h.shape[1], float(eps), _ptr(x), _stream())
    return x


def argmax_rows(logits, out=None):
    _need(logits, torch.float32, "logits", contiguous=False)
    if out is None:
        out = torch.empty((logits.shape[0],), dtype=torch.int32, device=logits.device)
    _lib.call("mg_argmax_rows", _ptr(logits), logits.shape[0], logits.shape[1], logits.stride(0), _ptr(out),
              _stream())
    return out


def decode_advance(tokens, next_tokens, positions, ctx_lens, slots, block_tables):
    _lib.call("mg_decode_advance", _ptr(tokens), _ptr(next_tokens), _ptr(positions), _ptr(ctx_lens), _ptr(slots),
              _ptr(block_tables), block_tables.shape[1], tokens.shape[0], _stream())


def check_device() -> None:
    _lib.check_device(torch.cuda.current_stream().cuda_stream)


# ---- fused row-parallel all-reduce over peer memory --------------------------------------------
NORM_NONE, NORM_RMS, NORM_LAYER = 0, 1, 2


class Comm:
    """This rank's peer-memory communicator (receive area + flags, mapped into every rank).

    ``exchange(my_handle: bytes) -> list[bytes]`` returns every rank's IPC handle in rank order; by
    default it is an ``all_gather_object`` over ``group``."""

    def __init__(self, rank: int, world: int, slot_elems: int, group=None, exchange=None) -> None:
        lib = _lib.load()
        nbytes = lib.mg_comm_handle_bytes()
        self._h = C.c_void_p()
        handle = C.create_string_buffer(nbytes)
        _lib.call("mg_comm_create", rank, world, int(slot_elems), C.byref(self._h), C.cast(handle, C.c_void_p))
        mine = handle.raw
        if exchange is None:
            import torch.distributed as dist
            handles = [None] * world
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = exchange(mine)
        if len(handles) != world or any(len(h) != nbytes for h in handles):
            raise ValueError("one IPC handle per rank is needed")
        allh = C.create_string_buffer(b"".join(handles), nbytes * world)
        _lib.call("mg_comm_open", self._h, C.cast(allh, C.c_void_p))
        self.rank, self.world, self.slot = rank, world, slot_elems

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise RuntimeError("communicator is closed")
        return self._h

    def close(self) -> None:
        if self._h:
            _lib.call("mg_comm_destroy", self._h)
            self._h = C.c_void_p()


def i8_linear_rowpar(x, q: PackedWeight, scales, comm: Comm, split_k: int = 0, workspace=None) -> None:
    """This rank's partial x · (q·s)ᵀ, pushed into every rank's receive slot (no bias); with a stream-K
    ``workspace`` the stream-K kernel computes it."""
    _need(x, torch.bfloat16, "x", contiguous=False)
    _need(scales, torch.float32, "scales")
    if not isinstance(q, PackedWeight):
        raise TypeError("the row-parallel push runs on tile-packed codes")
    n, k = q.shape
    if x.dim() != 2 or x.stride(1) != 1 or x.shape[1] != k:
        raise ValueError("x must be [m, k] with unit inner stride")
    if workspace is not None:
        _lib.call("mg_i8_linear_packed_rowpar_sk", _ptr(x), x.shape[0], k, x.stride(0), _ptr(q.data), _ptr(scales),
                  n, comm.handle, _ptr(workspace), workspace.numel() * workspace.element_size(), _stream())
        return
    _lib.call("mg_i8_linear_packed_rowpar", _ptr(x), x.shape[0], k, x.stride(0), _ptr(q.data), _ptr(scales), n,
              comm.handle, int(split_k), _stream())


def rowpar_reduce_norm(comm: Comm, h, bias, norm: int, w=None, b=None, eps: float = 1e-5, x=None):
    """h += Σ_ranks partial + bias (rank order); with norm, x = bf16(norm(h)). Returns x."""
    _need(h, torch.float32, "h")
    m, n = h.shape
    if norm and x is None:
        x = torch.empty((m, n), dtype=torch.bfloat16, device=h.device)
    _lib.call("mg_rowpar_reduce_norm", comm.handle, _ptr(h), _ptr(bias), m, n, int(norm), _ptr(w), _ptr(b),
              float(eps), _ptr(x), _stream())
    return x


def vocab_argmax(comm: Comm, logits, offset: int, out=None):
    """Global greedy argmax of logits split by columns across the ranks (this rank's fp32 shard
    ``logits`` [m, n_local] holds global columns [offset, offset + n_local)): int32 [m], identical on
    every rank, torch.argmax's first maximal index over the whole row. Every rank must call it at the
    same point of the communicator's push / reduce sequence."""
    _need(logits, torch.float32, "logits", contiguous=False)
    m, n = logits.shape
    if out is None:
        out = torch.empty((m,), dtype=torch.int32, device=logits.device)
    _lib.call("mg_vocab_argmax", comm.handle, _ptr(logits), m, n, logits.stride(0), int(offset), _ptr(out),
              _stream())
    _lib.LAUNCHES[0] += 1  # the local argmax, then the exchange and merge
    return out


# ---- persistent decode layer (mg_decode_block) -----------------------------------------------------
BLK_O, BLK_MLP, BLK_N1, BLK_QKV = 1, 2, 4, 8
BLOCK_MAX_TOKENS = 32


class BlockLinear(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("bias", C.c_void_p), ("n", C.c_int64),
                ("k", C.c_int64)]


class BlockArgs(C.Structure):
    """ctypes mirror of ``mg_block_args`` (include/microgen_b200.h)."""
    _fields_ = [("m", C.c_int), ("flags", C.c_int), ("hidden", C.c_int), ("hq", C.c_int), ("hkv", C.c_int),
                ("head_dim", C.c_int), ("norm", C.c_int), ("mlp", C.c_int), ("eps", C.c_float),
                ("max_pos", C.c_int), ("o", BlockLinear), ("gate_up", BlockLinear), ("down", BlockLinear),
                ("qkv", BlockLinear), ("h", C.c_void_p), ("attn", C.c_void_p), ("n2_w", C.c_void_p),
                ("n2_b", C.c_void_p), ("x2", C.c_void_p), ("act", C.c_void_p), ("n1_w", C.c_void_p),
                ("n1_b", C.c_void_p), ("x1", C.c_void_p), ("cos_sin", C.c_void_p), ("positions", C.c_void_p),
                ("slots", C.c_void_p), ("q_out", C.c_void_p), ("k_pool", C.c_void_p), ("v_pool", C.c_void_p),
                ("num_blocks", C.c_int64)]


def block_linear(q: PackedWeight, scales: torch.Tensor, bias: torch.Tensor | None) -> BlockLinear:
    if not isinstance(q, PackedWeight):
        raise TypeError("the persistent layer kernel reads tile-packed codes (pack_weights)")
    _need(scales, torch.float32, "scales")
    if bias is not None:
        _need(bias, torch.float32, "bias")
    return BlockLinear(q.data.data_ptr(), scales.data_ptr(), 0 if bias is None else bias.data_ptr(), q.n, q.k)


def block_workspace_bytes(args: BlockArgs) -> int:
    n = C.c_size_t(0)
    _lib.call("mg_decode_block_workspace_bytes", C.byref(args), C.byref(n))
    return int(n.value)


def decode_block(args: BlockArgs, workspace: torch.Tensor, comm=None) -> None:
    """One launch of the persistent decode layer described by ``args`` (see ``mg_decode_block``).
    ``workspace``: a zero-filled uint8 device tensor of at least ``block_workspace_bytes(args)`` bytes,
    reused across launches; ``comm``: the row-parallel communicator at world > 1."""
    _lib.call("mg_decode_block", C.byref(args), comm.handle if comm is not None else None,
              _ptr(workspace), workspace.numel(), _stream())


def decode_block_diag(clear: bool = True) -> list[int]:
    """The snapshot of the first persistent-layer wait that gave up (see ``mg_decode_block_diag``)."""
    buf = (C.c_uint32 * (32 + 1024))()
    _lib.call("mg_decode_block_diag", C.cast(buf, C.c_void_p), 1 if clear else 0)
    return list(buf)


def decode_block_trace(ctas: int):
    """numpy int64 [ctas, 16]: globaltimer stamps of the latest persistent-layer launch (mg_decode_block_trace)."""
    import numpy as np
    out = np.zeros((ctas, 16), dtype=np.uint64)
    _lib.call("mg_decode_block_trace", C.c_void_p(out.ctypes.data), int(ctas))
    return out.astype(np.int64)

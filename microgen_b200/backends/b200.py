"""InferenceBackend implementations on the B200 decode engine.

Same surface as the reference backends (``microgen/backends/base.py:8-41``,
``pytorch.py:55-181``, ``quantized.py:41-80``, ``parallel.py:84-139``):
``device``, ``load_model(name, model_instance=None)``,
``prefill(input_ids, attention_mask=None, cache=None) -> (logits[B,V], cache)``,
``decode(token_ids[B,1], attention_mask=None, cache=None) -> (logits[B,V], cache)``,
``sample(logits, temperature, top_k, top_p)``, ``get_memory_usage()``.

The cache object is a ``PagedKVCache``: the block tables of the batch's sequences in
the backend's ``PagedKVCacheAllocator`` (whose device pool holds K/V). The caller
owns it and passes it back in, as with ``KVCacheState``.

Prefill runs ``prefill_chunk`` positions of every prompt per pass: each INT8 linear
on all those tokens in one launch (tcgen05 tiles of up to 256 tokens), causal
attention per prompt on the paged decode kernel (``DecodeEngine.prefill``). Prompts
that share a leading run of whole
16-token blocks are prefilled once for that prefix (batch 1) and the blocks are
shared by reference count; the attention kernel then reads them once per batch.
With ``prefix_cache_capacity`` > 0 such prefixes are also kept across calls
(``runtime/prefix_cache.py``, the paged form of the reference's ``PrefixKVCache``).

``B200TensorParallelBackend`` is SPMD: one process per GPU, every rank making the
same calls in the same order; logits are identical on every rank.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .. import kernels as K
from ..engine import DecodeEngine, WeightLoader
from ..model_spec import spec_from_hf_config
from ..runtime.paged_kv import BlockTable, PagedKVCacheAllocator, TableMirror, check_shared_prefix
from ..runtime.prefix_cache import PagedPrefixCache

BLOCK = 16


class CUDADeviceInfo:
    """The subset of the reference's ``Device`` (``microgen/devices/base.py:8-41``) the backends use."""

    def __init__(self, index: int = 0) -> None:
        self.index = index
        self.torch_device = torch.device("cuda", index)
        self.name = f"cuda:{index}"

    def to_device(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(self.torch_device)

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.torch_device)

    def get_memory_info(self) -> Dict[str, Any]:
        free, total = torch.cuda.mem_get_info(self.torch_device)
        return {"device": self.name, "allocated_bytes": torch.cuda.memory_allocated(self.torch_device),
                "reserved_bytes": torch.cuda.memory_reserved(self.torch_device), "free_bytes": free,
                "total_bytes": total}


class PagedKVCache:
    """Per-batch cache state: one BlockTable per sequence, all in the backend's allocator."""

    def __init__(self, allocator: PagedKVCacheAllocator) -> None:
        self.allocator = allocator
        self.tables: List[BlockTable] = []
        self.prefix: Optional[BlockTable] = None
        self.n_shared_blocks = 0
        self.mirror: Optional[TableMirror] = None  # host copy of the block tables for decode steps
        self.reused_prefix_tokens = 0  # prompt tokens whose K/V came from the backend's prefix cache

    def __bool__(self) -> bool:
        return True

    def __len__(self) -> int:
        return len(self.tables)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.tables[0].num_tokens if self.tables else 0

    def free(self) -> None:
        for t in self.tables:
            self.allocator.free_sequence(t)
        if self.prefix is not None:
            self.allocator.free_sequence(self.prefix)
        self.tables, self.prefix, self.n_shared_blocks = [], None, 0


def _state_dict_fp32(model: nn.Module) -> dict:
    out = {}
    for k, v in model.state_dict().items():
        out[k] = v.detach()
    return out


class B200QuantizedBackend:
    """INT8 per-channel weight-only decode on one B200 (TP = 1)."""

    def __init__(self, device=None, quant_type: str = "int8", max_batch: int = 64, max_seq_len: int = 4096,
                 num_blocks: Optional[int] = None, use_cuda_graph: bool = True, free_list_seed: Optional[int] = None,
                 world_size: int = 1, group=None, device_check_every: int = 1,
                 prefix_cache_capacity: int = 0, prefill_chunk: int = 64, quantize_kv: bool = False) -> None:
        """``device_check_every``: after every that many ``decode`` calls, read the library's device error
        word (one stream synchronisation) and raise — TimeoutError when a bounded wait gave up (a peer
        rank that never pushed its row-parallel partial), RuntimeError for a failed device-side check —
        instead of returning logits computed from incomplete data. 0 turns the check off.

        ``prefix_cache_capacity`` > 0 keeps a block-level prefix cache (``PagedPrefixCache``) of that many
        entries: a prefill whose prompts start with a cached run of whole blocks shares those blocks instead
        of recomputing them, and every prefill's whole-block common prefix is cached for later calls.

        ``quantize_kv``: keep K/V as int8 codes with one fp32 scale per (token, kv head) vector, as the
        reference's ``KVCacheState(quantize_kv=True)`` does (``kv_cache.py:30-40, 114-120``): half the KV bytes
        per decode step.

        ``prefill_chunk``: prompt positions per prefill pass (every prompt of the batch at once, the
        linears on all those tokens per launch); 0 runs the prompt through the decode step one position at
        a time."""
        if quant_type.lower() != "int8":
            raise ValueError("the B200 decode path implements INT8 per-channel weights only")
        if isinstance(device, CUDADeviceInfo):
            self._device = device
        else:
            idx = torch.cuda.current_device() if device is None else torch.device(device).index or 0
            self._device = CUDADeviceInfo(idx)
        self.quant_type = "int8"
        self.max_batch, self.max_seq_len = max_batch, max_seq_len
        self.num_blocks = num_blocks or max_batch * ((max_seq_len + BLOCK - 1) // BLOCK)
        self.use_cuda_graph = use_cuda_graph
        self.free_list_seed = free_list_seed
        self.world_size, self.group = world_size, group
        self.device_check_every = max(0, int(device_check_every))
        self._decodes = 0
        self._greedy = None
        self.prefix_cache_capacity = int(prefix_cache_capacity)
        self.prefill_chunk = max(0, int(prefill_chunk))
        self.quantize_kv = bool(quantize_kv)
        self.prefix_cache: Optional[PagedPrefixCache] = None
        self.rank = torch.distributed.get_rank(group) if world_size > 1 else 0
        self.engine: Optional[DecodeEngine] = None
        self.allocator: Optional[PagedKVCacheAllocator] = None
        self._model_name: Optional[str] = None
        self._quantized = False
        self.spec = None

    # ---- InferenceBackend --------------------------------------------------------------------
    @property
    def device(self) -> CUDADeviceInfo:
        return self._device

    def load_model(self, model_name_or_path: str, model_instance: Optional[nn.Module] = None) -> None:
        if model_instance is None:
            from transformers import AutoModelForCausalLM
            model_instance = AutoModelForCausalLM.from_pretrained(model_name_or_path, trust_remote_code=True)
        self.load_state(spec_from_hf_config(model_instance.config), _state_dict_fp32(model_instance))
        self._model_name = model_name_or_path

    def load_state(self, spec, state: dict) -> None:
        """Load from a ModelSpec and a state dict keyed by HF parameter names (any device, fp32)."""
        dev = self._device.torch_device
        with torch.cuda.device(dev):
            # lm_head split by rows across the ranks (MG_VOCAB_PARALLEL=0 replicates it, as the reference does)
            vp = self.world_size > 1 and DecodeEngine.rank0_flag("MG_VOCAB_PARALLEL", self.group)
            weights = WeightLoader(spec, dev, self.rank, self.world_size, vocab_parallel=vp).load(state)
            max_blocks = (self.max_seq_len + BLOCK - 1) // BLOCK
            self.engine = DecodeEngine(spec, weights, dev, self.max_batch, self.num_blocks, max_blocks,
                                       rank=self.rank, world=self.world_size, group=self.group,
                                       max_pos=self.max_seq_len, quantize_kv=self.quantize_kv)
        self.allocator = PagedKVCacheAllocator(num_blocks=self.num_blocks, block_size=BLOCK)
        if self.free_list_seed is not None:
            self.allocator.shuffle_free_list(self.free_list_seed)
        if self.prefix_cache_capacity > 0:
            self.prefix_cache = PagedPrefixCache(self.allocator, self.prefix_cache_capacity)
        self.spec = spec
        self._quantized = True

    def _need_model(self) -> DecodeEngine:
        if self.engine is None:
            raise RuntimeError("Model is not loaded. Call load_model() first.")
        return self.engine

    @staticmethod
    def _ids(t) -> List[List[int]]:
        t = torch.as_tensor(t)
        if t.dim() == 1:
            t = t[None]
        return t.detach().to("cpu", torch.int64).tolist()

    def _run(self, tables: List[BlockTable], tokens: List[int], positions: List[int], n_shared: int,
             logits: bool, cache_mirror: Optional[TableMirror] = None) -> None:
        eng = self.engine
        b = len(tables)
        if max(t.num_blocks() for t in tables) > eng.max_blocks:
            width = max(t.num_blocks() for t in tables)
            raise ValueError(f"context of {width * BLOCK} tokens exceeds max_seq_len {self.max_seq_len}")
        if cache_mirror is None:
            cache_mirror = TableMirror(b, eng.max_blocks)
        tab = cache_mirror.update(tables)
        key = (cache_mirror.rebuilds, b, n_shared)
        if cache_mirror.prefix_checked != key:  # rows only grew since the last check: leading entries kept
            check_shared_prefix(tab, n_shared)
            cache_mirror.prefix_checked = key
        pos = np.asarray(positions, dtype=np.int64)
        slots = tab[np.arange(b), pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK
        eng.set_inputs(tokens, pos, slots, pos + 1, tab)
        if self.use_cuda_graph:
            eng.capture(b, n_shared, compute_logits=logits).replay()
        else:
            eng.forward(b, n_shared, compute_logits=logits)

    def prefill(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                cache: Optional[PagedKVCache] = None) -> Tuple[torch.Tensor, PagedKVCache]:
        eng = self._need_model()
        if attention_mask is not None and not bool(torch.as_tensor(attention_mask).bool().all()):
            raise NotImplementedError("padded prompts are not supported: pass equal-length prompts")
        ids = self._ids(input_ids)
        b, T = len(ids), len(ids[0])
        if b > self.max_batch:
            raise ValueError(f"batch {b} > max_batch {self.max_batch}")
        with torch.cuda.device(self._device.torch_device):
            if cache is None or not cache.tables:
                cache = cache or PagedKVCache(self.allocator)
                start = 0
                # longest common prefix in whole blocks (keep >= 1 private token per sequence)
                lcp = T
                for row in ids[1:]:
                    lcp = min(lcp, next((i for i, (a, c) in enumerate(zip(ids[0], row)) if a != c), T))
                n_prefix = min(lcp, T - 1) // BLOCK
                if not (b > 1 or self.prefix_cache is not None):
                    n_prefix = 0
                if n_prefix:
                    # the prefix's blocks: those a cached prefix already holds, then computed ones (batch 1)
                    toks = ids[0][:n_prefix * BLOCK]
                    hit = self.prefix_cache.match_prefix(toks) if self.prefix_cache is not None else None
                    reused = hit[0] // BLOCK if hit is not None else 0
                    if reused:
                        cache.prefix = self.allocator.share_prefix(hit[1], reused, "prefix", n_prefix * BLOCK)
                    else:
                        cache.prefix = self.allocator.allocate_sequence("prefix", n_prefix * BLOCK)
                    prefix_mirror = TableMirror(1, eng.max_blocks)
                    if self.prefill_chunk and n_prefix > reused:
                        eng.prefill([ids[0]], prefix_mirror.update([cache.prefix]), reused * BLOCK, n_prefix * BLOCK,
                                    compute_logits=False, chunk=self.prefill_chunk)
                    else:
                        for p in range(reused * BLOCK, n_prefix * BLOCK):
                            self._run([cache.prefix], [ids[0][p]], [p], 0, logits=False, cache_mirror=prefix_mirror)
                    if self.prefix_cache is not None:
                        self.prefix_cache.insert(toks, cache.prefix)
                    cache.tables = [self.allocator.share_prefix(cache.prefix, n_prefix, f"seq{i}", T)
                                    for i in range(b)]
                    cache.reused_prefix_tokens = reused * BLOCK
                    start = n_prefix * BLOCK
                else:
                    cache.tables = [self.allocator.allocate_sequence(f"seq{i}", T) for i in range(b)]
                # the attention kernel's shared-prefix CTAs serve a batch; one sequence reads its blocks itself
                cache.n_shared_blocks = n_prefix if b > 1 else 0
            else:
                if len(cache.tables) != b:
                    raise ValueError("cache holds a different batch size")
                start = cache.tables[0].num_tokens
                for t in cache.tables:
                    for _ in range(T):
                        self.allocator.append_token(t)
                ids = [[0] * start + r for r in ids]
                T = start + T
            if cache.mirror is None or cache.mirror.arr.shape[0] < b:
                cache.mirror = TableMirror(b, eng.max_blocks)
            if self.prefill_chunk:
                width = max(t.num_blocks() for t in cache.tables)
                if width > eng.max_blocks:
                    raise ValueError(f"context of {width * BLOCK} tokens exceeds max_seq_len {self.max_seq_len}")
                eng.prefill(ids, cache.mirror.update(cache.tables), start, T, compute_logits=True,
                            chunk=self.prefill_chunk)
            else:
                for p in range(start, T):
                    self._run(cache.tables, [r[p] for r in ids], [p] * b, cache.n_shared_blocks,
                              logits=(p == T - 1), cache_mirror=cache.mirror)
            return self._logits_out(b), cache

    def _logits_out(self, b: int) -> torch.Tensor:
        """The step's full logits for the caller, remembering the greedy tokens the step already computed
        on the device (as int64 [b, 1], sample's return type) so that the first ``sample`` of these
        unmodified logits needs no second argmax."""
        eng = self.engine
        out = eng.full_logits(b)
        self._greedy = (out, out._version, eng.next_tokens[:b, None].to(torch.int64))
        return out

    def decode(self, token_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
               cache: Optional[PagedKVCache] = None) -> Tuple[torch.Tensor, PagedKVCache]:
        eng = self._need_model()
        if cache is None or not cache.tables:
            raise ValueError("decode needs the cache returned by prefill")
        toks = [r[-1] for r in self._ids(token_ids)]
        b = len(toks)
        if b != len(cache.tables):
            raise ValueError(f"{b} tokens for a cache of {len(cache.tables)} sequences")
        with torch.cuda.device(self._device.torch_device):
            positions = []
            for t in cache.tables:
                positions.append(t.num_tokens)
                self.allocator.append_token(t)
            if cache.mirror is None or cache.mirror.arr.shape[0] < b:
                cache.mirror = TableMirror(b, eng.max_blocks)
            self._run(cache.tables, toks, positions, cache.n_shared_blocks, logits=True, cache_mirror=cache.mirror)
            out = self._logits_out(b)  # the copies queue behind the step, ahead of the check's synchronisation
            self._decodes += 1
            if self.device_check_every and self._decodes % self.device_check_every == 0:
                K.check_device()
            return out, cache

    def sample(self, logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0,
               top_p: float = 0.0) -> torch.Tensor:
        """Greedy on the device argmax kernel; otherwise the reference's sampling (``pytorch.py:145-177``)."""
        if temperature <= 0.0 or (top_k == 0 and top_p == 0.0 and temperature == 1.0):
            g = self._greedy
            if g is not None and logits is g[0] and logits._version == g[1]:
                self._greedy = None  # handed out once: a later call returns a new tensor, as torch.argmax does
                return g[2]  # the device argmax of exactly these logits
            lg = logits.to(torch.float32).contiguous()
            return K.argmax_rows(lg).to(torch.int64)[:, None]
        logits = logits / max(temperature, 1e-5)
        if top_k > 0:
            top_k = min(top_k, logits.size(-1))
            logits[logits < torch.topk(logits, top_k)[0][..., -1, None]] = -float("Inf")
        if top_p > 0.0:
            sorted_logits, sorted_indices = torch.sort(logits, descending=True)
            cum = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
            remove = cum > top_p
            remove[..., 1:] = remove[..., :-1].clone()
            remove[..., 0] = 0
            logits[remove.scatter(dim=-1, index=sorted_indices, src=remove)] = -float("Inf")
        return torch.multinomial(torch.softmax(logits, dim=-1), num_samples=1)

    def get_memory_usage(self) -> Dict[str, Any]:
        info = self._device.get_memory_info()
        info["quant_type"] = self.quant_type
        info["is_quantized"] = self._quantized
        if self.engine is not None:
            info["weight_bytes"] = self.engine.w.nbytes()
            info["kv_pool_bytes"] = self.engine.pool.nbytes()
            info["free_blocks"] = self.allocator.get_num_free_blocks()
        return info


class B200TensorParallelBackend(B200QuantizedBackend):
    """INT8 tensor-parallel decode, one process per GPU (SPMD over ``group``)."""

    def __init__(self, world_size: int = 2, devices: Optional[list] = None, group=None, **kw) -> None:
        if world_size > 1 and not torch.distributed.is_initialized():
            raise RuntimeError("tensor parallelism runs one process per GPU: initialise torch.distributed first")
        rank = torch.distributed.get_rank(group) if world_size > 1 else 0
        dev = devices[rank] if devices else torch.cuda.current_device()
        super().__init__(device=dev, world_size=world_size, group=group, **kw)
        self._is_parallel = world_size > 1

    def get_memory_usage(self) -> Dict[str, Any]:
        info = super().get_memory_usage()
        info["world_size"] = self.world_size
        info["is_tensor_parallel"] = self._is_parallel
        info["rank"] = self.rank
        return info

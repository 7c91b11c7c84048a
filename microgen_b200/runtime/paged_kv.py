"""Paged KV cache: the reference's block allocator plus the device pool it indexes.

``PhysicalBlock``, ``BlockTable`` and ``PagedKVCacheAllocator`` keep the reference's
interface and behaviour (``microgen/runtime/paged_kv.py:7-110``): 16-token blocks,
a FIFO free list (``pop(0)``, freed blocks appended), ``allocate_sequence`` takes
``ceil(n/16)`` blocks, ``append_token`` allocates when the last block is full,
``MemoryError`` on exhaustion, and ``free_block`` decrements ``ref_count``.

Additions for the device path (the reference allocator is bookkeeping only):

* ``shuffle_free_list(seed)`` — seeded shuffle of the free list (block ids drawn
  from a shuffled free list, as the workloads specify);
* ``share_prefix(src, n_blocks, sequence_id)`` — a new table whose first
  ``n_blocks`` entries are ``src``'s blocks (``ref_count`` incremented), the
  block-level prefix sharing the attention kernel reads once per batch;
* ``block_table_tensor`` / ``slot`` — the int32 block table and slot ids the
  kernels consume;
* ``PagedKVPool`` — per-layer bf16 pools ``[num_blocks, kv_heads, 16, head_dim]``.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

BLOCK_SIZE = 16


@dataclass
class PhysicalBlock:
    """A fixed-size block of the KV pool (``paged_kv.py:7-12``)."""
    block_id: int
    block_size: int = BLOCK_SIZE
    ref_count: int = 0


@dataclass
class BlockTable:
    """Logical-to-physical block map of one sequence (``paged_kv.py:15-31``)."""
    sequence_id: str
    block_size: int = BLOCK_SIZE
    physical_blocks: List[PhysicalBlock] = field(default_factory=list)
    num_tokens: int = 0
    version: int = 0  # bumped whenever blocks are removed (rollback, free): mirrors rebuild their row

    def num_blocks(self) -> int:
        return len(self.physical_blocks)

    def is_last_block_full(self) -> bool:
        if not self.physical_blocks:
            return True
        return (self.num_tokens % self.block_size) == 0

    def block_ids(self) -> List[int]:
        return [b.block_id for b in self.physical_blocks]

    def slot(self, position: int) -> int:
        """Pool slot (block_id * block_size + offset) of token ``position``."""
        return self.physical_blocks[position // self.block_size].block_id * self.block_size + position % self.block_size


class PagedKVCacheAllocator:
    """Pool of fixed-size blocks (``paged_kv.py:34-110``)."""

    def __init__(self, num_blocks: int = 64, block_size: int = BLOCK_SIZE) -> None:
        if block_size != BLOCK_SIZE:
            raise ValueError("the decode kernels use 16-token blocks")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free_blocks: List[PhysicalBlock] = [PhysicalBlock(block_id=i, block_size=block_size)
                                                  for i in range(num_blocks)]
        self._allocated_blocks: Dict[int, PhysicalBlock] = {}

    def get_num_free_blocks(self) -> int:
        return len(self._free_blocks)

    def get_num_allocated_blocks(self) -> int:
        return len(self._allocated_blocks)

    def shuffle_free_list(self, seed: int) -> None:
        random.Random(seed).shuffle(self._free_blocks)

    def allocate_block(self) -> PhysicalBlock:
        if not self._free_blocks:
            raise MemoryError(f"PagedKVCacheAllocator out of physical memory blocks (max={self.num_blocks}).")
        block = self._free_blocks.pop(0)
        block.ref_count = 1
        self._allocated_blocks[block.block_id] = block
        return block

    def free_block(self, block: PhysicalBlock) -> None:
        if block.block_id not in self._allocated_blocks:
            return
        block.ref_count -= 1
        if block.ref_count <= 0:
            block.ref_count = 0
            del self._allocated_blocks[block.block_id]
            self._free_blocks.append(block)

    def allocate_sequence(self, sequence_id: str, prompt_token_count: int) -> BlockTable:
        num_blocks_needed = (prompt_token_count + self.block_size - 1) // self.block_size
        if prompt_token_count == 0:
            num_blocks_needed = 0
        if self.get_num_free_blocks() < num_blocks_needed:
            raise MemoryError(f"Insufficient free physical blocks: needed {num_blocks_needed}, "
                              f"available {self.get_num_free_blocks()}.")
        table = BlockTable(sequence_id=sequence_id, block_size=self.block_size, num_tokens=prompt_token_count)
        for _ in range(num_blocks_needed):
            table.physical_blocks.append(self.allocate_block())
        return table

    def append_token(self, block_table: BlockTable) -> None:
        if block_table.is_last_block_full():
            block_table.physical_blocks.append(self.allocate_block())
        block_table.num_tokens += 1

    def free_sequence(self, block_table: BlockTable) -> None:
        for block in block_table.physical_blocks:
            self.free_block(block)
        block_table.physical_blocks.clear()
        block_table.num_tokens = 0
        block_table.version += 1

    # ---- additions for the device path -------------------------------------------------------
    def rollback(self, block_table: BlockTable, num_tokens: int) -> None:
        """Drop the last ``num_tokens`` tokens of a sequence, freeing blocks left empty
        (the paged form of ``KVCacheState.rollback``, ``kv_cache.py:180-210``)."""
        if num_tokens <= 0:
            return
        keep = max(0, block_table.num_tokens - num_tokens)
        need = (keep + self.block_size - 1) // self.block_size
        while block_table.num_blocks() > need:
            self.free_block(block_table.physical_blocks.pop())
            block_table.version += 1
        block_table.num_tokens = keep

    def share_prefix(self, src: BlockTable, n_blocks: int, sequence_id: str, prompt_token_count: int) -> BlockTable:
        """Table for a sequence of ``prompt_token_count`` tokens whose first ``n_blocks`` full
        blocks are ``src``'s (shared, ref-counted); the rest are freshly allocated."""
        if n_blocks > src.num_blocks() or n_blocks * self.block_size > min(src.num_tokens, prompt_token_count):
            raise ValueError("a shared prefix must consist of full blocks of both sequences")
        rest = (prompt_token_count + self.block_size - 1) // self.block_size - n_blocks
        if self.get_num_free_blocks() < rest:
            raise MemoryError(f"Insufficient free physical blocks: needed {rest}, "
                              f"available {self.get_num_free_blocks()}.")
        table = BlockTable(sequence_id=sequence_id, block_size=self.block_size, num_tokens=prompt_token_count)
        for b in src.physical_blocks[:n_blocks]:
            b.ref_count += 1
            table.physical_blocks.append(b)
        for _ in range(rest):
            table.physical_blocks.append(self.allocate_block())
        return table


class TableMirror:
    """Host int32 copy of a batch's block tables, [rows, max_blocks], kept up to date incrementally.

    A decode step appends at most one block per sequence, so rebuilding the whole table in Python
    every step (hundreds of microseconds for a batch of 32) is replaced by writing the new entries.
    A row is rebuilt when its table object changes, its ``version`` changes (blocks removed), or its
    last mirrored entry no longer matches. Entries past a row's block count are zero. ``rebuilds`` counts
    row rebuilds: while it is unchanged, every row's existing entries are unchanged (rows only grew)."""

    def __init__(self, rows: int, max_blocks: int) -> None:
        self.arr = np.zeros((rows, max_blocks), np.int32)
        self._tabs: List[Optional[BlockTable]] = [None] * rows
        self._ver = [0] * rows
        self._n = [0] * rows
        self.rebuilds = 0
        self.prefix_checked = None  # (rebuilds, rows, shared blocks) of the last shared-prefix check passed

    def update(self, tables: Sequence[BlockTable]) -> np.ndarray:
        """The mirror's rows for ``tables`` (a view, [len(tables), widest table])."""
        if len(tables) > self.arr.shape[0]:
            raise ValueError(f"{len(tables)} tables > {self.arr.shape[0]} mirror rows")
        width = 0
        for i, t in enumerate(tables):
            blocks = t.physical_blocks
            nb = len(blocks)
            if nb > self.arr.shape[1]:
                raise ValueError(f"block table of {nb} blocks > {self.arr.shape[1]}")
            n = self._n[i]
            if (self._tabs[i] is not t or self._ver[i] != t.version or nb < n
                    or (n and self.arr[i, n - 1] != blocks[n - 1].block_id)):
                self.arr[i, :n] = 0
                self._tabs[i], self._ver[i], n = t, t.version, 0
                self._n[i] = 0
                self.rebuilds += 1
            if nb > n:
                self.arr[i, n:nb] = [b.block_id for b in blocks[n:nb]]
            self._n[i] = nb
            width = max(width, nb)
        return self.arr[:len(tables), :width]


def check_shared_prefix(tables: np.ndarray, n_shared_blocks: int) -> None:
    """Raise ValueError unless the first ``n_shared_blocks`` entries of every row of ``tables`` equal
    row 0's: the attention kernel reads shared-prefix blocks once, from row 0's table."""
    if n_shared_blocks <= 0 or len(tables) == 0:
        return
    t = np.asarray(tables)
    if n_shared_blocks > t.shape[1]:
        raise ValueError(f"{n_shared_blocks} shared blocks > table width {t.shape[1]}")
    lead = t[:, :n_shared_blocks]
    bad = np.nonzero((lead != lead[:1]).any(axis=1))[0]
    if len(bad):
        raise ValueError(f"n_shared_blocks={n_shared_blocks}, but the leading block ids of sequence {int(bad[0])} "
                         "differ from sequence 0's: shared-prefix blocks must be the same in every table")


def block_table_tensor(tables: Sequence[BlockTable], max_blocks: int, device=None) -> torch.Tensor:
    """int32 [len(tables), max_blocks] of block ids (unused entries 0)."""
    out = torch.zeros((len(tables), max_blocks), dtype=torch.int32)
    for i, t in enumerate(tables):
        ids = t.block_ids()
        if len(ids) > max_blocks:
            raise ValueError(f"sequence {t.sequence_id} holds {len(ids)} blocks > max_blocks {max_blocks}")
        if ids:
            out[i, : len(ids)] = torch.tensor(ids, dtype=torch.int32)
    return out if device is None else out.to(device)


class PagedKVPool:
    """Per-layer K and V pools ``[num_blocks, kv_heads, 16, head_dim]`` on one device: bf16, or with
    ``quantize`` int8 codes plus one fp32 scale per (block, kv head, token) vector in ``k_scale`` /
    ``v_scale`` ``[layers, num_blocks, kv_heads, 16]`` (the paged form of ``KVCacheState(quantize_kv=True)``,
    ``kv_cache.py:30-40``)."""

    def __init__(self, layers: int, num_blocks: int, kv_heads: int, head_dim: int, device,
                 dtype: torch.dtype = torch.bfloat16, quantize: bool = False) -> None:
        shape = (layers, num_blocks, kv_heads, BLOCK_SIZE, head_dim)
        self.quantize = bool(quantize)
        dtype = torch.int8 if self.quantize else dtype
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.k_scale = self.v_scale = None
        if self.quantize:
            self.k_scale = torch.zeros(shape[:4], dtype=torch.float32, device=device)
            self.v_scale = torch.zeros(shape[:4], dtype=torch.float32, device=device)
        self.num_blocks = num_blocks

    def scales(self, layer: int) -> dict:
        """Keyword arguments naming layer ``layer``'s scale arrays for the KV kernels (none for bf16)."""
        if not self.quantize:
            return {}
        return {"k_scales": self.k_scale[layer], "v_scales": self.v_scale[layer]}

    def nbytes(self) -> int:
        n = 2 * self.k.numel() * self.k.element_size()
        if self.quantize:
            n += 2 * self.k_scale.numel() * 4
        return n

"""Block-level prefix cache over the paged KV allocator (the paged form of
``microgen/caching/prefix_cache.py``).

The reference's ``PrefixKVCache`` stores whole ``KVCacheState`` objects under the SHA-256 of the
comma-joined token ids (``prefix_cache.py:8-11``) and finds the longest cached prefix of a prompt by a
linear scan (``:49-70``), evicting the oldest entry first when full (``:26-42``). Here an entry is a
``BlockTable`` whose whole 16-token blocks hold the prefix's K/V in the device pool: the cache keeps a
reference (``ref_count``) on each of those blocks, a prefill that matches the entry shares the blocks by
reference instead of recomputing them, and eviction drops the cache's references (a block returns to
the free list once no sequence holds it either). Prefix lengths are whole blocks: a partly filled block
cannot be shared, because the sequence that reuses it writes its own next tokens into it.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import List, Optional, Tuple

from .paged_kv import BlockTable, PagedKVCacheAllocator


def compute_token_hash(token_ids: List[int]) -> str:
    """SHA-256 hex digest of the comma-joined token ids (the reference's key, ``prefix_cache.py:8-11``)."""
    import hashlib
    return hashlib.sha256(",".join(str(int(t)) for t in token_ids).encode("utf-8")).hexdigest()


class PagedPrefixCache:
    """Token prefix -> shared block table, FIFO-evicted at ``max_capacity`` entries."""

    def __init__(self, allocator: PagedKVCacheAllocator, max_capacity: int = 100) -> None:
        if max_capacity < 1:
            raise ValueError("max_capacity must be >= 1")
        self.allocator = allocator
        self.max_capacity = max_capacity
        self._cache: "OrderedDict[str, Tuple[List[int], BlockTable]]" = OrderedDict()

    @property
    def size(self) -> int:
        return len(self._cache)

    @property
    def block_size(self) -> int:
        return self.allocator.block_size

    def _release(self, table: BlockTable) -> None:
        self.allocator.free_sequence(table)

    def insert(self, token_ids: List[int], table: BlockTable) -> str:
        """Cache the K/V of ``token_ids`` held by the first len(token_ids) / block_size blocks of ``table``
        (``len(token_ids)`` must be a positive multiple of the block size and ``table`` must hold at least
        that many tokens). The cache takes its own reference on those blocks. Returns the key."""
        n = len(token_ids)
        bs = self.block_size
        if n == 0:
            raise ValueError("Cannot cache empty token sequence.")
        if n % bs:
            raise ValueError(f"a cached prefix is whole {bs}-token blocks ({n} tokens given)")
        if table.num_tokens < n:
            raise ValueError("the table holds fewer tokens than the prefix")
        key = compute_token_hash(token_ids)
        if len(self._cache) >= self.max_capacity and key not in self._cache:
            _, (_, old) = self._cache.popitem(last=False)  # oldest entry first
            self._release(old)
        held = BlockTable(sequence_id=f"prefix:{key[:12]}", block_size=bs, num_tokens=n)
        for b in table.physical_blocks[:n // bs]:
            b.ref_count += 1
            held.physical_blocks.append(b)
        prev = self._cache.get(key)
        # a present key keeps its place in the eviction order and takes the new blocks (as a dict update does)
        self._cache[key] = (list(int(t) for t in token_ids), held)
        if prev is not None:
            self._release(prev[1])
        return key

    def get(self, cache_key: str) -> Optional[BlockTable]:
        entry = self._cache.get(cache_key)
        return entry[1] if entry is not None else None

    def match_prefix(self, token_ids: List[int]) -> Optional[Tuple[int, BlockTable]]:
        """(length, table) of the longest cached prefix of ``token_ids``, or None (the reference's scan,
        ``prefix_cache.py:49-70``)."""
        if not token_ids:
            return None
        ids = [int(t) for t in token_ids]
        best_len, best = 0, None
        for cached, table in self._cache.values():
            n = len(cached)
            if best_len < n <= len(ids) and ids[:n] == cached:
                best_len, best = n, table
        return (best_len, best) if best is not None else None

    def clear(self) -> None:
        for _, table in self._cache.values():
            self._release(table)
        self._cache.clear()

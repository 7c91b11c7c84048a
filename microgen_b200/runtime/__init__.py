"""Runtime memory: the paged block allocator and its device KV pool."""

from microgen_b200.runtime.paged_kv import (BlockTable, PagedKVCacheAllocator, PagedKVPool,  # noqa: F401
                                            PhysicalBlock, block_table_tensor)
from microgen_b200.runtime.prefix_cache import PagedPrefixCache, compute_token_hash  # noqa: F401

__all__ = ["BlockTable", "PagedKVCacheAllocator", "PagedKVPool", "PhysicalBlock", "block_table_tensor",
           "PagedPrefixCache", "compute_token_hash"]

"""Runtime memory: the paged block allocator and its device KV pool."""

from microgen_b200.runtime.paged_kv import (BlockTable, PagedKVCacheAllocator, PagedKVPool,  # noqa: F401
                                            PhysicalBlock, block_table_tensor)

__all__ = ["BlockTable", "PagedKVCacheAllocator", "PagedKVPool", "PhysicalBlock", "block_table_tensor"]

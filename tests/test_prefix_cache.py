"""Block-level prefix cache (CPU): the reference PrefixKVCache's keys, longest-prefix matches and FIFO
eviction (tests/golden/prefix_trace.json, written by running the reference), and the block reference
counts the paged form adds."""

import json
import os

import pytest

from microgen_b200.runtime.paged_kv import PagedKVCacheAllocator
from microgen_b200.runtime.prefix_cache import PagedPrefixCache, compute_token_hash

G = os.path.join(os.path.dirname(__file__), "golden")


def test_replays_reference_prefix_trace():
    d = json.load(open(os.path.join(G, "prefix_trace.json")))
    seqs = {k: v for k, v in d["seqs"].items()}
    seqs["b2"] = seqs["b"]
    a = PagedKVCacheAllocator(num_blocks=64)
    pc = PagedPrefixCache(a, max_capacity=3)
    label_of = {}
    keys = {}
    for op in d["trace"]:
        kind = op[0]
        if kind == "insert":
            _, lab, key, size = op
            t = a.allocate_sequence(lab, len(seqs[lab]))
            keys[lab] = pc.insert(seqs[lab], t)
            label_of[id(pc.get(keys[lab]))] = lab
            a.free_sequence(t)  # the cache keeps its own reference
            assert keys[lab] == key and pc.size == size
        elif kind == "match":
            _, probe, want = op
            m = pc.match_prefix(probe)
            got = None if m is None else [m[0], label_of[id(m[1])]]
            assert got == want, probe
        elif kind == "get":
            _, lab, want = op
            t = pc.get(keys[lab])
            assert (None if t is None else label_of[id(t)]) == want
        elif kind == "hash":
            assert compute_token_hash(op[1]) == op[2]


def test_cache_holds_block_references():
    a = PagedKVCacheAllocator(num_blocks=16)
    pc = PagedPrefixCache(a, max_capacity=1)
    t = a.allocate_sequence("s", 40)            # 3 blocks, the first 2 cacheable
    key = pc.insert(list(range(32)), t)
    held = pc.get(key)
    assert [b.block_id for b in held.physical_blocks] == [b.block_id for b in t.physical_blocks[:2]]
    assert [b.ref_count for b in t.physical_blocks] == [2, 2, 1]
    a.free_sequence(t)
    assert a.get_num_allocated_blocks() == 2    # still held by the cache
    m = pc.match_prefix(list(range(40)))
    assert m is not None and m[0] == 32
    u = a.share_prefix(m[1], 2, "u", 40)        # a new sequence shares them
    assert [b.ref_count for b in u.physical_blocks[:2]] == [2, 2]
    pc.insert(list(range(100, 116)), u)         # capacity 1: evicts the first entry
    assert pc.match_prefix(list(range(40))) is None
    assert [b.ref_count for b in u.physical_blocks[:2]] == [2, 1]  # block 0 also held by the new entry
    a.free_sequence(u)
    pc.clear()
    assert a.get_num_allocated_blocks() == 0 and a.get_num_free_blocks() == 16


def test_insert_rejects_partial_blocks_and_empty():
    a = PagedKVCacheAllocator(num_blocks=8)
    pc = PagedPrefixCache(a)
    t = a.allocate_sequence("s", 20)
    with pytest.raises(ValueError):
        pc.insert([], t)
    with pytest.raises(ValueError):
        pc.insert(list(range(20)), t)
    with pytest.raises(ValueError):
        pc.insert(list(range(32)), t)          # the table holds only 20 tokens

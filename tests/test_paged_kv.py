"""Paged block allocator (CPU): the reference's block-id order, its error behaviour, the additions for
the device path (rollback, shared prefixes) and the incremental host mirror of the block tables."""

import json
import os
import random

import numpy as np
import pytest

from microgen_b200.runtime.paged_kv import PagedKVCacheAllocator, TableMirror, block_table_tensor

G = os.path.join(os.path.dirname(__file__), "golden")


def test_allocator_replays_reference_trace():
    """Same operations as tests/golden/make_golden.py ran on the reference allocator: identical block
    ids at every step, identical free list after a free, identical out-of-memory message."""
    want = json.load(open(os.path.join(G, "alloc_trace.json")))
    a = PagedKVCacheAllocator(num_blocks=12, block_size=16)
    got = []
    t1 = a.allocate_sequence("a", 35)
    got.append(["alloc", "a", 35, [b.block_id for b in t1.physical_blocks]])
    t2 = a.allocate_sequence("b", 16)
    got.append(["alloc", "b", 16, [b.block_id for b in t2.physical_blocks]])
    for _ in range(13):
        a.append_token(t1)
    got.append(["append13", "a", t1.num_tokens, [b.block_id for b in t1.physical_blocks]])
    a.append_token(t2)
    got.append(["append1", "b", t2.num_tokens, [b.block_id for b in t2.physical_blocks]])
    a.free_sequence(t1)
    got.append(["free", "a", a.get_num_free_blocks(), [b.block_id for b in a._free_blocks]])
    t3 = a.allocate_sequence("c", 70)
    got.append(["alloc", "c", 70, [b.block_id for b in t3.physical_blocks]])
    t4 = a.allocate_sequence("d", 0)
    got.append(["alloc", "d", 0, [b.block_id for b in t4.physical_blocks]])
    with pytest.raises(MemoryError) as e:
        a.allocate_sequence("e", 16 * 20)
    got.append(["oom", "e", 320, str(e.value)])
    assert got == want


def test_block_counts_overflow_and_oom():
    a = PagedKVCacheAllocator(num_blocks=4)
    t = a.allocate_sequence("s", 16)
    assert t.num_blocks() == 1 and a.get_num_free_blocks() == 3
    a.append_token(t)  # 17th token opens a second block
    assert t.num_blocks() == 2 and t.slot(16) == t.physical_blocks[1].block_id * 16
    a.allocate_sequence("u", 32)
    with pytest.raises(MemoryError):
        a.allocate_sequence("v", 1)
    a.free_sequence(t)
    assert a.get_num_free_blocks() == 2 and t.num_blocks() == 0


def test_rollback_and_shared_prefix_refcounts():
    a = PagedKVCacheAllocator(num_blocks=16)
    src = a.allocate_sequence("p", 40)  # 3 blocks, 2 full
    s1 = a.share_prefix(src, 2, "s1", 40)
    s2 = a.share_prefix(src, 2, "s2", 50)
    assert s1.block_ids()[:2] == s2.block_ids()[:2] == src.block_ids()[:2]
    assert src.physical_blocks[0].ref_count == 3
    v = s2.version
    a.rollback(s2, 30)  # 50 -> 20 tokens: two blocks left, the shared ones
    assert s2.num_tokens == 20 and s2.num_blocks() == 2 and s2.version > v
    a.free_sequence(s1)
    a.free_sequence(s2)
    assert src.physical_blocks[0].ref_count == 1  # still held by the source
    with pytest.raises(ValueError):
        a.share_prefix(src, 3, "bad", 48)  # the third block is not full


def test_table_mirror_tracks_appends_rollbacks_and_replacements():
    rng = random.Random(0)
    a = PagedKVCacheAllocator(num_blocks=4000)
    a.shuffle_free_list(1)
    tables = [a.allocate_sequence(f"s{i}", rng.randint(1, 300)) for i in range(12)]
    m = TableMirror(12, 64)
    for step in range(400):
        op = rng.random()
        i = rng.randrange(len(tables))
        if op < 0.85:
            for t in tables:
                a.append_token(t)
        elif op < 0.93:
            a.rollback(tables[i], rng.randint(1, 60))
        elif op < 0.97:
            a.free_sequence(tables[i])
            tables[i] = a.allocate_sequence(f"r{step}", rng.randint(1, 200))
        else:
            a.free_sequence(tables[i])
            a.append_token(tables[i])
        got = m.update(tables)
        width = max(t.num_blocks() for t in tables)
        want = block_table_tensor(tables, 64).numpy()[:, :width]
        assert got.shape == want.shape and np.array_equal(got, want), f"step {step}"


def test_table_mirror_rejects_oversized_input():
    a = PagedKVCacheAllocator(num_blocks=64)
    m = TableMirror(2, 4)
    with pytest.raises(ValueError):
        m.update([a.allocate_sequence("x", 16 * 5)])
    with pytest.raises(ValueError):
        m.update([a.allocate_sequence(f"y{i}", 1) for i in range(3)])


def test_table_mirror_row_reused_by_an_empty_table_then_block_zero():
    """A row that held 3 blocks gets a new empty table, which then grows to 3 blocks whose last id is 0:
    the mirror must hold the new ids, not the zeros left by the rebuild."""
    a = PagedKVCacheAllocator(num_blocks=8, block_size=16)
    old = a.allocate_sequence("old", 40)  # blocks 0, 1, 2
    m = TableMirror(1, 8)
    assert m.update([old])[0].tolist() == [0, 1, 2]
    a.free_sequence(old)
    a._free_blocks.sort(key=lambda b: -b.block_id)  # hand out 7, 6, ..., 0 so the third block is 0
    a._free_blocks = [b for b in a._free_blocks if b.block_id in (5, 3, 0)]
    new = a.allocate_sequence("new", 0)
    assert m.update([new]).shape == (1, 0)
    for _ in range(33):
        a.append_token(new)
    assert [b.block_id for b in new.physical_blocks] == [5, 3, 0]
    assert m.update([new])[0].tolist() == [5, 3, 0]


def test_check_shared_prefix():
    from microgen_b200.runtime.paged_kv import check_shared_prefix
    t = np.array([[4, 7, 1, 0], [4, 7, 2, 3], [4, 7, 5, 6]], np.int32)
    check_shared_prefix(t, 2)
    check_shared_prefix(t, 0)
    with pytest.raises(ValueError):
        check_shared_prefix(t, 3)
    t[2, 1] = 9
    with pytest.raises(ValueError, match="sequence 2"):
        check_shared_prefix(t, 2)


def test_mirror_rebuild_count_tracks_changed_rows():
    """Rows that only grow keep ``rebuilds``; a rollback that frees blocks or a replaced table raises it.
    The decode step re-checks the shared-prefix contract only when ``rebuilds`` moved."""
    a = PagedKVCacheAllocator(num_blocks=64)
    s0, s1 = a.allocate_sequence("s0", 40), a.allocate_sequence("s1", 20)
    m = TableMirror(2, 16)
    m.update([s0, s1])
    r0 = m.rebuilds
    for _ in range(40):
        a.append_token(s0)
        a.append_token(s1)
        tab = m.update([s0, s1])
    assert m.rebuilds == r0
    assert tab[0, :s0.num_blocks()].tolist() == s0.block_ids()
    assert tab[1, :s1.num_blocks()].tolist() == s1.block_ids()
    a.rollback(s0, 3)                      # frees no block: entries unchanged, no rebuild
    m.update([s0, s1])
    assert m.rebuilds == r0
    a.rollback(s0, 30)                     # frees blocks
    assert m.update([s0, s1])[0, :s0.num_blocks()].tolist() == s0.block_ids()
    assert m.rebuilds == r0 + 1
    s2 = a.allocate_sequence("s2", 5)
    assert m.update([s2, s1])[0].tolist()[:2] == s2.block_ids() + [0]
    assert m.rebuilds == r0 + 2

"""Control plane on the CPU: ports of the reference's CPU tests
(tests/{block_table,sequence_state,slot_mapping,batch_block_table,
physical_block_pool,prefix_cache,copy_on_write,paged_kv_layout,oom,
fragmentation}_test.cpp in KVFlux) against kvflux_b200's C++ API, plus A/B
traces against the reference's own control plane (golden fixtures, and live
when oracle/_ref is built)."""
import json
from pathlib import Path

import numpy as np
import pytest

import kvflux_b200 as kv
import scenarios

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "control_plane.json").read_text())


# ------------------------------------------------------------- A/B traces ---

@pytest.mark.parametrize("fn", scenarios.ALL, ids=lambda f: f.__name__)
def test_trace_matches_reference_golden(fn):
    assert fn(kv) == GOLDEN[fn.__name__]


def test_known_answers_from_reference_tests():
    assert GOLDEN["occupy_slots"]["slots"] == [173, 522, 944]
    assert GOLDEN["read_27_3_91"]["blocks"] == [27, 3, 91]
    assert GOLDEN["slot_mapping_recipe"] == {"slots": [1298, 513, 2208], "later": [2216]}
    pad = 2**64 - 1
    assert GOLDEN["batch_table_recipe"]["table"] == [0, 3, 6, pad, 1, 4, 7, 8, 2, 5, pad, pad, pad, pad, pad, pad]
    assert GOLDEN["batch_table_recipe"]["lens"] == [35, 61, 28, 0]


def test_live_trace_against_compiled_reference():
    from oracle import refapi

    if not refapi.available():
        pytest.skip("reference CPU library not built")
    for fn in scenarios.ALL:
        assert fn(kv) == fn(refapi), fn.__name__


# ------------------------------------------------------ physical block pool ---

def test_pool_lifo_reuse_and_stale_handles():
    with pytest.raises(ValueError):
        kv.PhysicalBlockPool(0, 16)
    with pytest.raises(ValueError):
        kv.PhysicalBlockPool(1024, 0)
    pool = kv.PhysicalBlockPool(1024, 16)
    assert (pool.capacity(), pool.block_size(), pool.available()) == (1024, 16, 1024)
    first, middle, third = pool.allocate(), pool.allocate(), pool.allocate()
    assert [pool.id(h) for h in (first, middle, third)] == [0, 1, 2]
    pool.free(middle)
    reused = pool.allocate()
    assert pool.id(reused) == middle.id and reused.generation != middle.generation
    with pytest.raises(ValueError):
        pool.id(middle)
    with pytest.raises(ValueError):
        pool.free(middle)
    pool.retain(first)
    assert pool.ref_count(first) == 2
    pool.free(first)
    assert pool.ref_count(first) == 1 and pool.available() == 1021


def test_pool_capacity_error():
    pool = kv.PhysicalBlockPool(2, 4)
    pool.allocate()
    pool.allocate()
    with pytest.raises(kv.CapacityError):
        pool.allocate()


# -------------------------------------------------------------- block table ---

def test_block_table_mapping_and_sharing():
    pool = kv.PhysicalBlockPool(100, 16)
    initial = [pool.allocate() for _ in range(92)]
    a = kv.BlockTable(pool)
    for pid in (27, 91, 3, 48):
        a.append_existing(initial[pid])
    assert [a.physical_id(i) for i in range(4)] == [27, 91, 3, 48] and a[0] == 27
    with pytest.raises(IndexError):
        a.physical_id(4)
    for h in initial:
        pool.free(h)
    assert pool.available() == 96
    b = kv.BlockTable(pool)
    b.append_shared(a, 1)
    b.append_shared(a, 3)
    assert (b.physical_id(0), b.physical_id(1), pool.available()) == (91, 48, 96)
    a.pop_back()
    assert a.size() == 3 and b.physical_id(1) == 48
    a.clear()
    assert a.empty() and pool.available() == 98
    b.clear()
    assert pool.available() == pool.capacity()
    with pytest.raises(IndexError):
        b.pop_back()


def test_block_table_capacity_move_and_invalid_inputs():
    pool = kv.PhysicalBlockPool(2, 16)
    a = kv.BlockTable(pool)
    assert a.append_new() == 0 and a.append_new() == 1
    with pytest.raises(kv.CapacityError):
        a.append_new()
    moved = kv.BlockTable(pool)
    moved.move_from(a)
    assert a.empty() and moved.physical_id(0) == 0
    with pytest.raises(kv.LogicError):
        a.append_new()
    moved.append_shared(moved, 0)
    assert moved.size() == 3 and pool.available() == 0
    moved.pop_back()
    assert pool.available() == 0
    moved.clear()
    assert pool.available() == 2

    other_pool = kv.PhysicalBlockPool(2, 16)
    t, other = kv.BlockTable(pool), kv.BlockTable(other_pool)
    stale = pool.allocate()
    pool.free(stale)
    with pytest.raises(ValueError):
        t.append_existing(stale)
    t.append_new()
    with pytest.raises(IndexError):
        t.append_shared(t, 1)
    with pytest.raises(ValueError):
        t.append_shared(other, 0)
    assert t.size() == 1 and pool.available() == 1


# ----------------------------------------------------------- sequence state ---

def test_sequence_virtual_blocks_and_growth():
    pool = kv.PhysicalBlockPool(100, 16)
    held = []

    def occupy(n):
        while len(held) < n:
            held.append(pool.allocate())

    r = kv.SequenceState(1001, pool)
    assert (r.request_id(), r.block_size(), r.num_tokens(), r.last_block_num_tokens()) == (1001, 16, 0, 0)
    occupy(7)
    r.append_tokens(16)
    occupy(32)
    r.append_tokens(16)
    occupy(89)
    r.append_tokens(3)
    assert r.num_tokens() == 35 and r.num_allocated_blocks() == 3 and r.last_block_num_tokens() == 3
    assert [r.physical_block_id(i) for i in range(3)] == [7, 33, 91]
    loc = r.token_location(34)
    assert (loc.physical_block, loc.offset_in_block) == (91, 2)
    with pytest.raises(IndexError):
        r.token_location(35)
    for h in held:
        pool.free(h)
    assert pool.available() == 97


def test_sequence_rollback_on_capacity_and_overflow():
    pool = kv.PhysicalBlockPool(2, 16)
    r = kv.SequenceState(42, pool)
    r.append_tokens(15)
    r.append_tokens(1)
    r.append_tokens(0)
    assert r.num_tokens() == 16 and pool.available() == 1
    with pytest.raises(kv.CapacityError):
        r.append_tokens(32)
    assert r.num_tokens() == 16 and r.num_allocated_blocks() == 1 and pool.available() == 1
    with pytest.raises(OverflowError):
        r.append_tokens(2**64 - 1)
    loc = r.append_token()
    assert (loc.physical_block, loc.offset_in_block) == (1, 0)
    r.append_tokens(15)
    with pytest.raises(kv.CapacityError):
        r.append_token()
    assert r.num_tokens() == 32


# -------------------------------------------------------------- slot mapping ---

def test_slot_mapping_rejects_invalid_batches():
    p1, p2 = kv.PhysicalBlockPool(2, 16), kv.PhysicalBlockPool(2, 16)
    a, b = kv.SequenceState(1, p1), kv.SequenceState(2, p2)
    a.append_tokens(16)
    b.append_tokens(1)
    assert kv.build_slot_mapping([]) == []
    assert kv.build_slot_mapping([(a, 15), (a, 0)]) == [15, 0]
    with pytest.raises(ValueError):
        kv.build_slot_mapping([(None, 0)])
    with pytest.raises(IndexError):
        kv.build_slot_mapping([(a, 16)])
    with pytest.raises(ValueError):
        kv.build_slot_mapping([(a, 0), (b, 0)])
    assert a.num_tokens() == 16 and p1.available() == 1


def test_batch_table_errors():
    assert kv.build_batch_block_table([]).num_sequences() == 0
    pool, other_pool = kv.PhysicalBlockPool(16, 16), kv.PhysicalBlockPool(2, 16)
    a, o = kv.SequenceState(1, pool), kv.SequenceState(5, other_pool)
    a.append_tokens(35)
    t = kv.build_batch_block_table([a])
    assert t.physical_id(0, 2) == 2
    with pytest.raises(IndexError):
        t.physical_id(1, 0)
    with pytest.raises(ValueError):
        kv.build_batch_block_table([a, None])
    with pytest.raises(ValueError):
        kv.build_batch_block_table([a, o])


# ---------------------------------------------------------- copy-on-write ---

def test_cow_shared_partial_page_and_rollback():
    pool = kv.PhysicalBlockPool(3, 4)
    pages = [[0, 0, 0, 0] for _ in range(3)]
    a = kv.SequenceState(1, pool)
    a.append_tokens(3)
    old = a.physical_block_id(0)
    pages[old] = [11, 22, 33, -1]
    b = a.fork_shared(2)
    assert b.num_tokens() == 3 and pool.ref_count(a.block_table().handle(0)) == 2
    with pytest.raises(kv.LogicError):
        a.append_token()
    copies = []

    def copier(src, dst):
        pages[dst.id] = list(pages[src.id])
        copies.append((src.id, dst.id))

    loc = a.append_token_with_copy(copier)
    assert len(copies) == 1 and loc.physical_block != old and loc.offset_in_block == 3
    assert pages[loc.physical_block] == [11, 22, 33, -1]
    assert pool.ref_count(b.block_table().handle(0)) == 1

    pool2 = kv.PhysicalBlockPool(2, 4)
    x = kv.SequenceState(1, pool2)
    x.append_tokens(2)
    y = x.fork_shared(2)

    def failing(src, dst):
        raise RuntimeError("copy failed")

    with pytest.raises(RuntimeError):
        x.append_token_with_copy(failing)
    assert x.num_tokens() == 2 and pool2.available() == 1
    with pytest.raises(ValueError):
        x.append_token_with_copy(None)
    assert y.physical_block_id(0) == x.physical_block_id(0)


# ------------------------------------------------------------ prefix cache ---

def test_prefix_cache_share_collision_and_eviction():
    pool = kv.PhysicalBlockPool(6, 2)
    cache = kv.PrefixCache(pool)
    a = kv.SequenceState(1, pool)
    a.append_tokens(5)
    cache.publish_computed_block(a, 0, [10, 20])
    cache.publish_computed_block(a, 1, [10, 20, 30, 40])
    with pytest.raises(ValueError):
        cache.publish_computed_block(a, 2, [10, 20, 30, 40, 50])
    b = kv.SequenceState(2, pool)
    assert cache.attach_cached_prefix(b, [10, 20, 30, 40, 60]) == 4
    assert b.physical_block_id(0) == 0 and b.physical_block_id(1) == 1

    pool2 = kv.PhysicalBlockPool(4, 2, lambda toks: 7)  # every prefix collides
    c2 = kv.PrefixCache(pool2)
    x, y = kv.SequenceState(1, pool2), kv.SequenceState(2, pool2)
    x.append_tokens(4)
    y.append_tokens(4)
    c2.publish_computed_block(x, 0, [1, 2])
    c2.publish_computed_block(x, 1, [1, 2, 3, 4])
    c2.publish_computed_block(y, 0, [5, 6])
    c2.publish_computed_block(y, 1, [5, 6, 3, 4])
    hit = kv.SequenceState(3, pool2)
    assert c2.attach_cached_prefix(hit, [5, 6, 3, 4]) == 4
    assert hit.physical_block_id(1) == y.physical_block_id(1)

    pool3 = kv.PhysicalBlockPool(2, 2)
    c3 = kv.PrefixCache(pool3)
    s = kv.SequenceState(1, pool3)
    s.append_tokens(4)
    c3.publish_computed_block(s, 0, [1, 2])
    c3.publish_computed_block(s, 1, [1, 2, 3, 4])
    cached = pool3.lookup([1, 2])
    pool3.free(cached)
    del s
    assert pool3.available() == 2
    reused = pool3.allocate()  # evicts the oldest idle cached page
    assert reused.id == cached.id and reused.generation != cached.generation
    assert pool3.lookup([1, 2]) is None


# ---------------------------------------------------------------- layout ---

@pytest.mark.parametrize("dtype,elem", [(kv.DType.Float16, 2), (kv.DType.BFloat16, 2), (kv.DType.Float32, 4)])
def test_layout_offsets_exhaustive(dtype, elem):
    lay = kv.PagedKVLayout(3, 2, 4, 3, dtype)
    assert lay.page_bytes() == 2 * 4 * 3 * elem and lay.cache_bytes() == 3 * lay.page_bytes()
    assert lay.total_bytes() == 2 * lay.cache_bytes() and lay.slot_count() == 12
    expected = 0
    for kind in (kv.KVKind.Key, kv.KVKind.Value):
        for block in range(3):
            assert lay.page_byte_offset(kind, block) == expected
            for head in range(2):
                for tok in range(4):
                    for d in range(3):
                        assert lay.byte_offset(kind, block, head, tok, d) == expected
                        assert lay.slot_byte_offset(kind, block * 4 + tok, head, d) == expected
                        expected += elem
    assert expected == lay.total_bytes()
    with pytest.raises(IndexError):
        lay.page_byte_offset(kv.KVKind.Key, 3)
    with pytest.raises(IndexError):
        lay.slot_byte_offset(kv.KVKind.Key, 12, 0, 0)
    with pytest.raises(OverflowError):
        kv.PagedKVLayout(2**64 - 1, 1, 1, 1, kv.DType.Float16)
    with pytest.raises(ValueError):
        kv.PagedKVLayout(0, 1, 1, 1, kv.DType.Float16)


def test_fragmented_pool_hands_out_permutation_order():
    from kvflux_b200 import workloads as w

    pool = kv.PhysicalBlockPool(64, 16)
    ids = np.array([5, 9, 33, 2, 60])
    held = w.fragment_pool(pool, ids)
    assert [pool.allocate().id for _ in range(5)] == ids.tolist()
    with pytest.raises(kv.CapacityError):
        pool.allocate()
    assert len(held) == 59

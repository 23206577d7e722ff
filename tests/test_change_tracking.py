"""Change tracking that lets paged_attention_batch keep its page table on the
GPU between calls: BlockTable's lineage / revision / first_changed_since and
the pool's log of pages whose references fell to zero. Host-only."""
import kvflux_b200 as kv


def test_appends_keep_revision_edits_change_it():
    pool = kv.PhysicalBlockPool(32, 4)
    t = kv.BlockTable(pool)
    lin, rev = t.lineage(), t.revision()
    t.append_new()
    t.append_new()
    assert t.lineage() == lin and t.revision() == rev
    assert t.first_changed_since(rev) == 2  # only appends since
    t.pop_back()
    assert t.revision() != rev and t.lineage() == lin
    assert t.first_changed_since(rev) == 1  # entry 1 was removed
    r2 = t.revision()
    t.append_new()
    assert t.first_changed_since(r2) == 2
    assert t.first_changed_since(rev) == 1


def test_replace_last_and_clear():
    pool = kv.PhysicalBlockPool(32, 4)
    t = kv.BlockTable(pool)
    for _ in range(5):
        t.append_new()
    rev = t.revision()
    fresh = pool.allocate()
    t.replace_last_owned(fresh)
    assert t.first_changed_since(rev) == 4
    r2 = t.revision()
    t.clear()
    assert t.first_changed_since(r2) == 0 and t.first_changed_since(rev) == 0


def test_old_revisions_beyond_the_edit_ring_are_unknown():
    pool = kv.PhysicalBlockPool(64, 4)
    t = kv.BlockTable(pool)
    for _ in range(20):
        t.append_new()
    rev = t.revision()
    for _ in range(5):  # more edits than the ring keeps
        t.pop_back()
    assert t.first_changed_since(rev) == 0
    recent = t.revision()
    t.pop_back()
    assert t.first_changed_since(recent) == t.size()


def test_moves_start_new_lineages_on_both_ends():
    pool = kv.PhysicalBlockPool(16, 4)
    a = kv.BlockTable(pool)
    a.append_new()
    b = kv.BlockTable(pool)
    la, lb = a.lineage(), b.lineage()
    b.move_from(a)
    assert b.size() == 1 and a.size() == 0
    assert b.lineage() not in (la, lb) and a.lineage() not in (la, lb)
    assert b.first_changed_since(b.revision()) == 1


def test_sequences_expose_their_table_tracking():
    pool = kv.PhysicalBlockPool(32, 4)
    s = kv.SequenceState(1, pool)
    s.append_tokens(5)
    rev = s.block_table().revision()
    s.append_tokens(4)  # grows by pages: an append
    assert s.block_table().revision() == rev
    child = s.fork_shared(2)
    assert child.block_table().lineage() != s.block_table().lineage()


def test_zero_reference_log():
    pool = kv.PhysicalBlockPool(8, 4)
    e0 = pool.zero_ref_events()
    h = [pool.allocate() for _ in range(3)]
    pool.retain(h[1])
    pool.free(h[1])  # 2 -> 1: not an event
    assert pool.zero_ref_events() == e0
    pool.free(h[1])
    pool.free(h[2])
    assert pool.zero_ref_events() == e0 + 2
    assert pool.zero_ref_ids_since(e0) == [h[1].id, h[2].id]
    assert pool.zero_ref_ids_since(e0 + 1) == [h[2].id]
    assert pool.zero_ref_ids_since(pool.zero_ref_events()) == []
    # More events than the log holds: it cannot tell.
    start = pool.zero_ref_events()
    for _ in range(8200):
        pool.free(pool.allocate())
    assert pool.zero_ref_ids_since(start) is None
    assert pool.zero_ref_ids_since(pool.zero_ref_events() - 10) is not None

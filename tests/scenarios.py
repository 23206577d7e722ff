"""Control-plane scenarios written against the binding's names, so the same
script drives kvflux_b200._C and the reference's compiled control plane
(oracle.refapi). Each returns a JSON-serialisable trace of page ids and slots.

The recipes are the reference tests' own (file:line in KVFlux).
"""
import numpy as np

from kvflux_b200 import workloads as w


def occupy_slots(api):
    # tests/paged_kv_write_test.cpp:36-55 -> slots {173, 522, 944}
    pool = api.PhysicalBlockPool(64, 16)
    held = []

    def occupy(n):
        while pool.capacity() - pool.available() < n:
            held.append(pool.allocate())

    occupy(10)
    a = api.SequenceState(1001, pool)
    a.append_tokens(14)
    occupy(32)
    b = api.SequenceState(1002, pool)
    b.append_tokens(11)
    occupy(59)
    c = api.SequenceState(1003, pool)
    c.append_tokens(1)
    return {"slots": list(api.build_slot_mapping([(a, 13), (b, 10), (c, 0)]))}


def read_27_3_91(api):
    # tests/paged_kv_read_test.cpp:39-51 -> table [27, 3, 91], 40 tokens
    pool = api.PhysicalBlockPool(96, 16)
    held = [pool.allocate() for _ in range(27)]
    r = api.SequenceState(1001, pool)
    r.append_tokens(16)
    held += [pool.allocate() for _ in range(28, 91)]
    pool.free(held[3])
    r.append_tokens(16)
    r.append_tokens(8)
    slots = api.build_slot_mapping([(r, t) for t in range(40)])
    return {"blocks": [r.physical_block_id(j) for j in range(r.num_allocated_blocks())], "slots": list(slots)}


def slot_mapping_recipe(api):
    # tests/slot_mapping_test.cpp:23-55 -> {1298, 513, 2208}, then 2216
    pool = api.PhysicalBlockPool(160, 16)
    held = []

    def occupy(n):
        while pool.capacity() - pool.available() < n:
            held.append(pool.allocate())

    occupy(31)
    b = api.SequenceState(1002, pool)
    b.append_tokens(18)
    occupy(79)
    a = api.SequenceState(1001, pool)
    a.append_tokens(35)
    occupy(133)
    c = api.SequenceState(1003, pool)
    c.append_tokens(81)
    first = list(api.build_slot_mapping([(a, 34), (b, 17), (c, 80)]))
    c.append_tokens(8)
    return {"slots": first, "later": list(api.build_slot_mapping([(c, 88)]))}


def batch_table_recipe(api):
    # tests/batch_block_table_test.cpp:24-42
    pool = api.PhysicalBlockPool(16, 16)
    a, b, c, e = (api.SequenceState(i, pool) for i in (1, 2, 3, 4))
    a.append_tokens(16)
    b.append_tokens(16)
    c.append_tokens(16)
    a.append_tokens(16)
    b.append_tokens(16)
    c.append_tokens(12)
    a.append_tokens(3)
    b.append_tokens(29)
    t = api.build_batch_block_table([a, b, c, e])
    return {"table": [int(x) for x in t.block_table()], "lens": [int(x) for x in t.sequence_lengths()],
            "width": int(t.max_blocks_per_sequence())}


def odd_fragmented(api):
    # benchmark/v2_paged_benchmark.cpp:66-84: 2B pages taken, odd ones freed in reverse
    requests, tokens, bs = 4, 37, 16
    blocks = requests * ((tokens + bs - 1) // bs)
    pool = api.PhysicalBlockPool(2 * blocks, bs)
    holders = [pool.allocate() for _ in range(2 * blocks)]
    for nxt in range(2 * blocks, 0, -2):
        pool.free(holders[nxt - 1])
    seqs = []
    for r in range(requests):
        s = api.SequenceState(r + 1, pool)
        s.append_tokens(tokens)
        seqs.append(s)
    return {"rows": [[s.physical_block_id(j) for j in range(s.num_allocated_blocks())] for s in seqs]}


def seeded_random_fragmentation(api):
    pool = api.PhysicalBlockPool(256, 16)
    ids = w.permutation(77, np.arange(256))[:90]
    held = w.fragment_pool(pool, ids, seed=1234)
    lens = [1, 15, 16, 17, 200, 33, 900]
    seqs = []
    for i, L in enumerate(lens):
        s = api.SequenceState(i, pool)
        s.append_tokens(L)
        seqs.append(s)
    t = api.build_batch_block_table(seqs)
    return {"table": [int(x) for x in t.block_table()], "width": int(t.max_blocks_per_sequence()),
            "available": int(pool.available())}


def fork_and_cow(api):
    # tests/copy_on_write_test.cpp:21-58 and the config-4 prefix-sharing shape
    pool = api.PhysicalBlockPool(64, 16)
    base = api.SequenceState(0, pool)
    base.append_tokens(40)  # 2 full pages + a shared partial page of 8 tokens
    forks = [base.fork_shared(i) for i in range(1, 4)]
    trace = []
    for f in forks:
        copies = []
        loc = f.append_token_with_copy(lambda s, d: copies.append([int(s.id), int(d.id)]))
        trace.append({"loc": [int(loc.physical_block), int(loc.offset_in_block)], "copies": copies})
        f.append_tokens(100)
    own = base.append_token()
    rows = [[s.physical_block_id(j) for j in range(s.num_allocated_blocks())] for s in [base] + forks]
    return {"trace": trace, "base_append": [int(own.physical_block), int(own.offset_in_block)], "rows": rows}


ALL = [occupy_slots, read_27_3_91, slot_mapping_recipe, batch_table_recipe, odd_fragmented,
       seeded_random_fragmentation, fork_and_cow]

"""Host logic of the multi-GPU decode on CPU ranks (gloo, world size 2):
each rank keeps only its KV heads' pages (its own pool, its own page ids),
computes its Q heads' outputs (the CPU oracle stands in for the kernel here),
the outputs are all-gathered and reassembled, and the result equals the
single-rank computation over all heads."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from kvflux_b200 import sharding


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


KVH, QH, HD, BS = 4, 8, 16, 4
LENS = [5, 17, 33]


def _full_inputs():
    from kvflux_b200 import workloads as w

    total = sum(LENS)
    k = w.normal(1, total * KVH * HD).reshape(total, KVH, HD)
    v = w.normal(2, total * KVH * HD).reshape(total, KVH, HD)
    q = w.normal(3, len(LENS) * QH * HD).reshape(len(LENS), QH, HD)
    return k, v, q


def _rank_output(shard, seed):
    """Builds this rank's own pool/tables for its heads and runs the oracle decode."""
    import oracle
    from kvflux_b200 import workloads as w

    k, v, q = _full_inputs()
    b = w.decode_batch_on_pool(64, BS, LENS, seed=seed, mode="random")
    table, width = b.table()
    h = shard.kv_heads
    cache_k = np.zeros((64, h, BS, HD), np.float32)
    cache_v = np.zeros_like(cache_k)
    off = 0
    for r, L in enumerate(LENS):
        for t in range(L):
            page, slot = int(table[r, t // BS]), t % BS
            cache_k[page, :, slot] = k[off + t, shard.kv_begin:shard.kv_end]
            cache_v[page, :, slot] = v[off + t, shard.kv_begin:shard.kv_end]
        off += L
    qs = np.ascontiguousarray(q[:, shard.q_begin:shard.q_end]).reshape(-1)
    out = oracle.decode_batch(cache_k.reshape(-1).view(np.uint8), cache_v.reshape(-1).view(np.uint8), 2, 64, h,
                              BS, HD, table, np.array(LENS, np.uint64), shard.q_heads, qs)
    return out, b


def _worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = sharding.shard_heads(KVH, QH, world, rank)
        out, _ = _rank_output(shard, seed=100 + rank)  # each rank fragments its own pool
        t = torch.from_numpy(out)
        gathered = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        if rank == 0:
            full = sharding.assemble(gathered, len(LENS), QH, HD)
            np.save(result_path, full.numpy())
    finally:
        dist.destroy_process_group()


def test_shard_heads_partition():
    shards = [sharding.shard_heads(8, 64, 8, r) for r in range(8)]
    assert [(s.kv_begin, s.kv_end) for s in shards] == [(r, r + 1) for r in range(8)]
    assert [(s.q_begin, s.q_end) for s in shards] == [(8 * r, 8 * r + 8) for r in range(8)]
    assert sharding.shard_heads(8, 32, 2, 1).q_heads == 16
    with pytest.raises(ValueError):
        sharding.shard_heads(8, 64, 3, 0)


def test_two_rank_gloo_matches_single_rank(tmp_path):
    import oracle

    result = tmp_path / "out.npy"
    mp.start_processes(_worker, args=(2, _free_port(), str(result)), nprocs=2, join=True, start_method="spawn")
    got = np.load(result)
    k, v, q = _full_inputs()
    off = 0
    for r, L in enumerate(LENS):
        exp = oracle.reference_attention(q[r].reshape(-1), k[off:off + L].reshape(-1), v[off:off + L].reshape(-1),
                                         (1, L, QH, KVH, HD))
        assert np.array_equal(got[r].reshape(-1), exp)
        off += L

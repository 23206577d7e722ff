"""Seeded synthetic workloads for the paged-KV path (the configs of the
benchmark and their small parity variants).

Inputs are synthetic: no dataset is involved. Host-side values come from a
splitmix64 stream through Box-Muller (identical on every machine); device-side
bulk values come from torch's seeded generator on the GPU.

Fragmented pools follow the reference's recipe (allocate every page, then
free a chosen subset): the pool's free list is LIFO, so freeing a permutation
in reverse hands the pages out in permutation order
(reference: benchmark/v2_paged_benchmark.cpp:69-74, src/block_manager.cpp:75-86).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import _C

from .synth import (CONFIG2, CONFIG3, CONFIG4, CONFIG5, DTYPE_CODE, ELEM_BYTES,  # noqa: F401
                    bf16_bits_to_f32, config_lengths, decode, encode, f32_to_bf16_bits, normal,
                    permutation, splitmix64, uniform, uniform_ints)

DTYPES = {"float16": _C.DType.Float16, "bfloat16": _C.DType.BFloat16, "float32": _C.DType.Float32}


def fragment_pool(pool, free_ids, seed: int | None = None) -> list:
    """Allocates every page of `pool`, then frees `free_ids` so that the next
    allocations return them in the given order (shuffled first when `seed` is
    set). Returns the handles still held (to be freed by the caller)."""
    cap = pool.capacity()
    handles = [pool.allocate() for _ in range(cap)]
    order = np.asarray(free_ids, dtype=np.int64)
    if seed is not None:
        order = permutation(seed, order)
    freed = np.zeros(cap, bool)
    for pid in order[::-1]:
        pool.free(handles[int(pid)])
        freed[int(pid)] = True
    return [h for h, f in zip(handles, freed) if not f]


@dataclass
class Batch:
    """A set of sequences on one pool, with their host-side tables."""

    pool: object
    sequences: list
    holders: list = field(default_factory=list)

    def lengths(self) -> np.ndarray:
        return np.array([s.num_tokens() for s in self.sequences], np.uint64)

    def table(self) -> tuple[np.ndarray, int]:
        t = _C.build_batch_block_table(self.sequences)
        width = t.max_blocks_per_sequence()
        return np.array(t.block_table(), np.uint64).reshape(len(self.sequences), width), width

    def release(self) -> None:
        self.sequences.clear()
        for h in self.holders:
            self.pool.free(h)
        self.holders.clear()


def decode_batch_on_pool(capacity: int, block_size: int, lengths, seed: int, mode: str = "random",
                         request_base: int = 1) -> Batch:
    """Sequences of the given lengths on a fresh pool whose free pages are a
    seeded random subset (mode 'random') or the odd ids (mode 'odd'), handed
    out in seeded random order."""
    pool = _C.PhysicalBlockPool(capacity, block_size)
    need = int(sum((int(l) + block_size - 1) // block_size for l in lengths))
    if need > capacity:
        raise ValueError(f"pool of {capacity} pages cannot hold {need}")
    if mode == "odd":
        ids = np.arange(1, capacity, 2)
        if len(ids) < need:
            raise ValueError("odd pages do not cover the workload")
    else:
        ids = permutation(seed ^ 0x5EED, np.arange(capacity))[:need]
    holders = fragment_pool(pool, ids, seed=seed)
    seqs = []
    for i, l in enumerate(lengths):
        s = _C.SequenceState(request_base + i, pool)
        s.append_tokens(int(l))
        seqs.append(s)
    return Batch(pool, seqs, holders)



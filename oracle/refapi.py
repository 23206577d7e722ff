"""The reference's own control plane (compiled, via ref_shim) behind the same
Python names as kvflux_b200's binding, so one scenario script can drive both
and their page ids, slots and tables can be compared. TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import OracleError, ref

_CODES = {1: ValueError, 2: IndexError, 3: OverflowError, 4: RuntimeError, 5: RuntimeError, 6: RuntimeError}


def _raise(rc: int, what: str) -> None:
    if rc != 0:
        raise _CODES.get(rc, RuntimeError)(f"reference {what} failed ({rc})")


def available() -> bool:
    return ref() is not None


class Handle:
    def __init__(self, id_: int, gen: int):
        self.id = id_
        self.generation = gen

    def __eq__(self, other):
        return self.id == other.id and self.generation == other.generation


class PhysicalBlockPool:
    def __init__(self, capacity: int, block_size: int):
        self._R = ref()
        if self._R is None:
            raise OracleError("reference CPU library not built")
        self._p = self._R.ref_pool_new(capacity, block_size)
        if not self._p:
            raise ValueError("invalid pool")
        self._block_size = block_size
        self._capacity = capacity

    def __del__(self):
        if getattr(self, "_p", None):
            self._R.ref_pool_delete(self._p)
            self._p = None

    def allocate(self) -> Handle:
        i, g = ctypes.c_uint64(), ctypes.c_uint64()
        _raise(self._R.ref_pool_allocate(self._p, ctypes.byref(i), ctypes.byref(g)), "allocate")
        return Handle(i.value, g.value)

    def free(self, h: Handle) -> None:
        _raise(self._R.ref_pool_free(self._p, h.id, h.generation), "free")

    def retain(self, h: Handle) -> None:
        _raise(self._R.ref_pool_retain(self._p, h.id, h.generation), "retain")

    def ref_count(self, h: Handle) -> int:
        out = ctypes.c_uint64()
        _raise(self._R.ref_pool_ref_count(self._p, h.id, h.generation, ctypes.byref(out)), "ref_count")
        return out.value

    def available(self) -> int:
        return int(self._R.ref_pool_available(self._p))

    def capacity(self) -> int:
        return self._capacity

    def block_size(self) -> int:
        return self._block_size


class _Loc:
    def __init__(self, b, o):
        self.physical_block = b
        self.offset_in_block = o


class SequenceState:
    def __init__(self, request_id: int, pool: PhysicalBlockPool, _raw=None):
        self._R = pool._R
        self._pool = pool
        self._s = _raw if _raw is not None else self._R.ref_seq_new(pool._p, request_id)

    def __del__(self):
        if getattr(self, "_s", None):
            self._R.ref_seq_delete(self._s)
            self._s = None

    def append_tokens(self, n: int) -> None:
        _raise(self._R.ref_seq_append_tokens(self._s, n), "append_tokens")

    def append_token(self) -> _Loc:
        b, o = ctypes.c_uint64(), ctypes.c_uint64()
        _raise(self._R.ref_seq_append_token(self._s, ctypes.byref(b), ctypes.byref(o)), "append_token")
        return _Loc(b.value, o.value)

    def fork_shared(self, request_id: int) -> "SequenceState":
        raw = self._R.ref_seq_fork(self._s, request_id)
        if not raw:
            raise RuntimeError("reference fork failed")
        return SequenceState(request_id, self._pool, _raw=raw)

    def append_token_with_copy(self, copier) -> _Loc:
        b, o, f, t = (ctypes.c_uint64() for _ in range(4))
        _raise(self._R.ref_seq_append_token_with_copy(self._s, ctypes.byref(b), ctypes.byref(o), ctypes.byref(f),
                                                      ctypes.byref(t)), "append_token_with_copy")
        if copier is not None and f.value != 2**64 - 1:
            copier(Handle(f.value, 0), Handle(t.value, 0))
        return _Loc(b.value, o.value)

    def num_tokens(self) -> int:
        return int(self._R.ref_seq_num_tokens(self._s))

    def num_allocated_blocks(self) -> int:
        return int(self._R.ref_seq_num_blocks(self._s))

    def physical_block_id(self, j: int) -> int:
        return int(self.block_ids()[j])

    def block_ids(self) -> list[int]:
        n = self.num_allocated_blocks()
        out = np.zeros(max(n, 1), np.uint64)
        _raise(self._R.ref_seq_block_ids(self._s, out.ctypes.data_as(ctypes.c_void_p)), "block_ids")
        return [int(x) for x in out[:n]]


def build_slot_mapping(batch) -> list[int]:
    R = ref()
    n = len(batch)
    seqs = (ctypes.c_void_p * max(n, 1))(*[s._s for s, _ in batch])
    pos = np.array([p for _, p in batch] or [0], np.uint64)
    out = np.zeros(max(n, 1), np.uint64)
    _raise(R.ref_slot_mapping(seqs, pos.ctypes.data_as(ctypes.c_void_p), n, out.ctypes.data_as(ctypes.c_void_p)),
           "build_slot_mapping")
    return [int(x) for x in out[:n]]


class _Batch:
    def __init__(self, table, lens, width):
        self._t, self._l, self._w = table, lens, width

    def block_table(self):
        return self._t

    def sequence_lengths(self):
        return self._l

    def max_blocks_per_sequence(self):
        return self._w

    def num_sequences(self):
        return len(self._l)


def build_batch_block_table(seqs) -> _Batch:
    R = ref()
    n = len(seqs)
    arr = (ctypes.c_void_p * max(n, 1))(*[s._s for s in seqs])
    width = ctypes.c_uint64()
    _raise(R.ref_batch_table(arr, n, ctypes.byref(width), None, None), "build_batch_block_table")
    table = np.zeros(max(n * width.value, 1), np.uint64)
    lens = np.zeros(max(n, 1), np.uint64)
    _raise(R.ref_batch_table(arr, n, ctypes.byref(width), table.ctypes.data_as(ctypes.c_void_p),
                             lens.ctypes.data_as(ctypes.c_void_p)), "build_batch_block_table")
    return _Batch([int(x) for x in table[: n * width.value]], [int(x) for x in lens[:n]], width.value)

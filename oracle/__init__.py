"""CPU oracles for the paged-KV path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, and only as the checker or the timed CPU baseline; the product
(kvflux_b200) never imports it.

  kvo_*  : oracle/kvoracle.c, a C restatement of the reference's CPU path
           (write/gather index math, FP64 three-pass reference_attention).
  ref_*  : oracle/_ref/libkvflux_ref.so, the reference's own CPU sources
           compiled unchanged plus a C shim (absent when no reference checkout
           was available to build it; callers then skip).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_lib = None
_ref = None

u64 = ctypes.c_uint64
u32 = ctypes.c_uint32
vp = ctypes.c_void_p
fp = ctypes.POINTER(ctypes.c_float)


class OracleError(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        path = HERE / "libkvoracle.so"
        if not path.exists():
            from . import build as _b  # noqa: F401  (relative import of oracle/build.py)
            _b.build()
        L = ctypes.CDLL(str(path))
        L.kvo_write.argtypes = [vp, vp, u64, u32, u32, u64, vp, vp, vp, u64]
        L.kvo_gather.argtypes = [vp, vp, u64, u32, u32, u64, vp, u64, vp, vp]
        L.kvo_to_f32.argtypes = [vp, ctypes.c_int, u64, vp]
        L.kvo_to_f32.restype = None
        L.kvo_reference_attention.argtypes = [vp, vp, vp, u64, u64, u64, u64, u64, vp]
        L.kvo_decode_batch.argtypes = [vp, vp, ctypes.c_int, u64, u32, u32, u32, vp, u64, vp, u64, u64, u32, vp, vp,
                                       ctypes.c_int]
        L.kvo_attention_rows.argtypes = [vp, vp, ctypes.c_int, u64, u32, u32, u32, vp, u64, u64, u32, vp, u64, u64,
                                         vp, ctypes.c_int]
        _lib = L
    return _lib


def ref():
    """The reference's own CPU library, or None if it was not built."""
    global _ref
    if _ref is None:
        path = HERE / "_ref" / "libkvflux_ref.so"
        if not path.exists():
            return None
        R = ctypes.CDLL(str(path))
        R.ref_pool_new.argtypes = [u64, u64]
        R.ref_pool_new.restype = vp
        R.ref_pool_delete.argtypes = [vp]
        R.ref_pool_delete.restype = None
        R.ref_pool_allocate.argtypes = [vp, ctypes.POINTER(u64), ctypes.POINTER(u64)]
        R.ref_pool_free.argtypes = [vp, u64, u64]
        R.ref_pool_retain.argtypes = [vp, u64, u64]
        R.ref_pool_available.argtypes = [vp]
        R.ref_pool_available.restype = u64
        R.ref_pool_ref_count.argtypes = [vp, u64, u64, ctypes.POINTER(u64)]
        R.ref_seq_new.argtypes = [vp, u64]
        R.ref_seq_new.restype = vp
        R.ref_seq_delete.argtypes = [vp]
        R.ref_seq_delete.restype = None
        R.ref_seq_append_tokens.argtypes = [vp, u64]
        R.ref_seq_append_token.argtypes = [vp, ctypes.POINTER(u64), ctypes.POINTER(u64)]
        R.ref_seq_fork.argtypes = [vp, u64]
        R.ref_seq_fork.restype = vp
        R.ref_seq_append_token_with_copy.argtypes = [vp] + [ctypes.POINTER(u64)] * 4
        R.ref_seq_num_tokens.argtypes = [vp]
        R.ref_seq_num_tokens.restype = u64
        R.ref_seq_num_blocks.argtypes = [vp]
        R.ref_seq_num_blocks.restype = u64
        R.ref_seq_block_ids.argtypes = [vp, vp]
        R.ref_slot_mapping.argtypes = [vp, vp, u64, vp]
        R.ref_batch_table.argtypes = [vp, u64, ctypes.POINTER(u64), vp, vp]
        R.ref_reference_attention.argtypes = [vp, vp, vp, u64, u64, u64, u64, u64, vp]
        R.ref_decode_batch.argtypes = [vp, vp, ctypes.c_int, u64, u64, u64, vp, u64, vp, u64, u64, u64, vp, vp,
                                       ctypes.c_int]
        _ref = R
    return _ref


def _p(a: np.ndarray):
    return a.ctypes.data_as(vp)


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise OracleError(f"{what} failed with code {rc}")


# ------------------------------------------------------------------ oracle ---

def write(k_cache: np.ndarray, v_cache: np.ndarray, num_blocks: int, heads: int, bs: int, row_bytes: int,
          k_new: np.ndarray, v_new: np.ndarray, slots: np.ndarray) -> None:
    """In-place byte write into host copies of the caches (kvo_write)."""
    slots = np.ascontiguousarray(slots, dtype=np.uint64)
    _check(lib().kvo_write(_p(k_cache), _p(v_cache), num_blocks, heads, bs, row_bytes,
                           _p(np.ascontiguousarray(k_new)), _p(np.ascontiguousarray(v_new)), _p(slots),
                           len(slots)), "kvo_write")


def gather(k_cache: np.ndarray, v_cache: np.ndarray, num_blocks: int, heads: int, bs: int, row_bytes: int,
           blocks: np.ndarray, num_tokens: int) -> tuple[np.ndarray, np.ndarray]:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint64)
    k_out = np.zeros(num_tokens * heads * row_bytes, np.uint8)
    v_out = np.zeros_like(k_out)
    _check(lib().kvo_gather(_p(k_cache), _p(v_cache), num_blocks, heads, bs, row_bytes, _p(blocks), num_tokens,
                            _p(k_out), _p(v_out)), "kvo_gather")
    return k_out, v_out


def to_f32(raw: np.ndarray, dtype: int) -> np.ndarray:
    elem = 4 if dtype == 2 else 2
    n = raw.nbytes // elem
    out = np.empty(n, np.float32)
    lib().kvo_to_f32(_p(np.ascontiguousarray(raw)), dtype, n, _p(out))
    return out


def reference_attention(q, k, v, shape) -> np.ndarray:
    """kvoracle's reference_attention; shape = (Lq, Lkv, Hq, Hkv, hd)."""
    lq, lkv, hq, hkv, hd = shape
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    if q.size != lq * hq * hd or k.size != lkv * hkv * hd or v.size != k.size:
        raise OracleError("tensor size does not match shape")
    out = np.empty(max(q.size, 1), np.float32)
    _check(lib().kvo_reference_attention(_p(q), _p(k), _p(v), lq, lkv, hq, hkv, hd, _p(out)),
           "kvo_reference_attention")
    return out[: q.size]


def decode_batch(k_cache, v_cache, dtype, num_blocks, kv_heads, bs, hd, table, lens, q_heads, q,
                 first=0, count=None, threads=1) -> np.ndarray:
    """Reference CPU path of batch decode (gather + reference_attention) for
    requests [first, first+count); other rows of the returned array are 0."""
    table = np.ascontiguousarray(table, np.uint64)
    lens = np.ascontiguousarray(lens, np.uint64)
    q = np.ascontiguousarray(q, np.float32)
    batch = len(lens)
    count = batch - first if count is None else count
    max_blocks = table.size // batch
    out = np.zeros(batch * q_heads * hd, np.float32)
    _check(lib().kvo_decode_batch(_p(k_cache), _p(v_cache), dtype, num_blocks, kv_heads, bs, hd, _p(table),
                                  max_blocks, _p(lens), first, count, q_heads, _p(q), _p(out), threads),
           "kvo_decode_batch")
    return out


def attention_rows(k_cache, v_cache, dtype, num_blocks, kv_heads, bs, hd, blocks, q_tokens, kv_tokens, q_heads, q,
                   row_begin=0, row_end=None, threads=1) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, np.uint64)
    q = np.ascontiguousarray(q, np.float32)
    row_end = q_tokens if row_end is None else row_end
    out = np.zeros(q_tokens * q_heads * hd, np.float32)
    _check(lib().kvo_attention_rows(_p(k_cache), _p(v_cache), dtype, num_blocks, kv_heads, bs, hd, _p(blocks),
                                    q_tokens, kv_tokens, q_heads, _p(q), row_begin, row_end, _p(out), threads),
           "kvo_attention_rows")
    return out


# --------------------------------------------------- reference (compiled) ---

def ref_reference_attention(q, k, v, shape) -> np.ndarray:
    R = ref()
    if R is None:
        raise OracleError("reference CPU library not built")
    lq, lkv, hq, hkv, hd = shape
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty(max(q.size, 1), np.float32)
    _check(R.ref_reference_attention(_p(q), _p(k), _p(v), lq, lkv, hq, hkv, hd, _p(out)), "ref_reference_attention")
    return out[: q.size]


def ref_decode_batch(k_cache, v_cache, dtype, kv_heads, bs, hd, table, lens, q_heads, q, first=0, count=None,
                     threads=1) -> np.ndarray:
    R = ref()
    if R is None:
        raise OracleError("reference CPU library not built")
    table = np.ascontiguousarray(table, np.uint64)
    lens = np.ascontiguousarray(lens, np.uint64)
    q = np.ascontiguousarray(q, np.float32)
    batch = len(lens)
    count = batch - first if count is None else count
    out = np.zeros(batch * q_heads * hd, np.float32)
    _check(R.ref_decode_batch(_p(k_cache), _p(v_cache), dtype, kv_heads, bs, hd, _p(table), table.size // batch,
                              _p(lens), first, count, q_heads, _p(q), _p(out), threads), "ref_decode_batch")
    return out


# ------------------------------------------------ reference GPU (compiled) ---

_ref_gpu = None


def ref_gpu():
    """The reference's own GPU path (its CUDA kernels for sm_100a behind its
    public API), or None if it was not built."""
    global _ref_gpu
    if _ref_gpu is None:
        path = HERE / "_ref" / "libkvflux_ref_gpu.so"
        if not path.exists():
            return None
        G = ctypes.CDLL(str(path))
        G.kvref_gpu_decode.argtypes = [ctypes.c_int, u64, ctypes.c_uint32, vp, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_uint32, vp, u64, vp, vp, vp, vp, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        _ref_gpu = G
    return _ref_gpu


def ref_gpu_decode(device, num_blocks, block_size, page_order, kv_heads, q_heads, head_size, dtype, lens, k_rows,
                   v_rows, q, reps=3):
    """Batch decode through the reference's public GPU API (write_paged_kv of
    every token, then paged_attention_batch `reps` times) on a pool whose free
    list hands out `page_order`. Returns (O, (first write ms, median ms of
    `reps` repeated writes), median decode ms)."""
    G = ref_gpu()
    if G is None:
        raise OracleError("reference GPU library not built")
    page_order = np.ascontiguousarray(page_order, np.uint64)
    lens = np.ascontiguousarray(lens, np.uint64)
    k_rows = np.ascontiguousarray(k_rows)
    v_rows = np.ascontiguousarray(v_rows)
    q = np.ascontiguousarray(q, np.float32)
    o = np.zeros(q.size, np.float32)
    w_ms, d_ms = (ctypes.c_double * 2)(0.0, 0.0), ctypes.c_double(0.0)
    _check(G.kvref_gpu_decode(device, num_blocks, block_size, _p(page_order), kv_heads, q_heads, head_size, dtype,
                              _p(lens), len(lens), _p(k_rows), _p(v_rows), _p(q), _p(o), reps, w_ms,
                              ctypes.byref(d_ms)), "kvref_gpu_decode")
    return o, (w_ms[0], w_ms[1]), d_ms.value

"""kvflux_b200: KVFlux's v2 paged-KV data path on B200 (sm_100a).

Two native surfaces, both built in-tree by ``python kvflux_b200/build.py``:

* ``kvflux_b200.lib`` - ctypes binding of the C ABI in include/kvfx.h
  (libkvflux_b200.so): stream-ordered kernels taking plain device pointers.
* ``kvflux_b200._C`` (re-exported here) - the reference's C++ v2 API
  (PhysicalBlockPool, SequenceState, PagedKVStorage, write_paged_kv,
  read_paged_kv, paged_attention, paged_attention_batch, append_token_cow,
  PrefixCache, SequenceLifecycle, ...) running on those kernels, plus
  BatchDecodeSession (batched decode steps over a device-resident block table)
  and write_paged_kv_layers / read_paged_kv_layers (one launch for all layers).

There is no fallback: importing fails loudly if the extension is not built.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "libkvflux_b200.so"

if not _LIB_PATH.exists():
    raise ImportError(
        f"kvflux_b200 native library missing ({_LIB_PATH.name}); build it with `python kvflux_b200/build.py`")

from ._C import *  # noqa: E402,F401,F403  (the C++ v2 API)
from . import _C  # noqa: E402

u64 = ctypes.c_uint64
u32 = ctypes.c_uint32
vp = ctypes.c_void_p

KVFX_OK, KVFX_EINVAL, KVFX_ERANGE, KVFX_EOVERFLOW, KVFX_ECUDA, KVFX_ETIMEOUT, KVFX_ENOSPACE = range(7)
KVFX_F16, KVFX_BF16, KVFX_F32 = 0, 1, 2
KVFX_FLAG_BAD_INDEX, KVFX_FLAG_TIMEOUT = 1, 2
KVFX_MAX_LAYERS = 128
KVFX_MAX_PREFILL_SEQS = 32


class KvfxCache(ctypes.Structure):
    """Mirror of ``kvfx_cache`` (include/kvfx.h)."""

    _fields_ = [
        ("k_base", vp),
        ("v_base", vp),
        ("num_blocks", u64),
        ("num_kv_heads", u32),
        ("block_size", u32),
        ("head_size", u32),
        ("dtype", u32),
        ("device", ctypes.c_int32),
        ("reserved", u32),
    ]


def _load():
    L = ctypes.CDLL(str(_LIB_PATH))
    C = ctypes.POINTER(KvfxCache)
    L.kvfx_write.argtypes = [C, vp, vp, vp, u64, vp]
    L.kvfx_gather.argtypes = [C, vp, u64, vp, vp, vp]
    L.kvfx_gather_batch.argtypes = [C, vp, vp, u64, u64, vp, vp, vp]
    L.kvfx_copy_page.argtypes = [C, u64, u64, vp]
    L.kvfx_write_layers.argtypes = [C, u32, vp, vp, u64, vp, u64, vp]
    L.kvfx_gather_layers.argtypes = [C, u32, vp, vp, u64, u64, vp, vp, u64, vp]
    L.kvfx_decode_workspace_bytes.argtypes = [C, u64, u32, u64, u32]
    L.kvfx_decode_workspace_bytes.restype = u64
    L.kvfx_decode_pages_per_split.argtypes = [C, u64, u32, u64, u64]
    L.kvfx_decode_pages_per_split.restype = u32
    L.kvfx_decode.argtypes = [C, vp, vp, vp, vp, u64, u64, u32, u64, u32, vp, u64, vp]
    L.kvfx_decode_append.argtypes = [C, vp, vp, vp, vp, vp, vp, vp, u64, u64, u32, u64, u32, vp, u64, vp]
    L.kvfx_decode_noalloc.argtypes = [C, vp, vp, vp, vp, u64, u64, u32, u64, vp]
    L.kvfx_attention_workspace_bytes.argtypes = [C, u64, u64, u32]
    L.kvfx_attention_workspace_bytes.restype = u64
    L.kvfx_attention.argtypes = [C, vp, vp, vp, u64, u64, u32, vp, u64, vp]
    L.kvfx_attention_batch.argtypes = [C, u32, vp, vp, vp, u64, vp, vp, u32, vp, u64, vp]
    L.kvfx_last_error.restype = ctypes.c_char_p
    L.kvfx_last_error.argtypes = []
    L.kvfx_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(u32), ctypes.c_int]
    L.kvfx_selftest_wait_timeout.argtypes = [ctypes.c_int]
    L.kvfx_version.restype = ctypes.c_char_p
    L.kvfx_version.argtypes = []
    return L


lib = _load()

#: Every symbol include/kvfx.h declares (checked by the tests).
KVFX_SYMBOLS = (
    "kvfx_write", "kvfx_gather", "kvfx_gather_batch", "kvfx_write_layers", "kvfx_gather_layers", "kvfx_copy_page", "kvfx_decode_workspace_bytes",
    "kvfx_decode_pages_per_split", "kvfx_decode", "kvfx_decode_append", "kvfx_decode_noalloc", "kvfx_attention_workspace_bytes",
    "kvfx_attention", "kvfx_attention_batch",
    "kvfx_last_error", "kvfx_device_status", "kvfx_selftest_wait_timeout", "kvfx_version",
)

DTYPE_CODE = {"float16": KVFX_F16, "bfloat16": KVFX_BF16, "float32": KVFX_F32}


class KvfxError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: kvfx error {code}: {lib.kvfx_last_error().decode()}")
        self.code = code


def check(code: int, what: str) -> None:
    if code != KVFX_OK:
        raise KvfxError(code, what)


def cache_descriptor(storage) -> KvfxCache:
    """The kvfx_cache of a PagedKVStorage (all fields from its public API)."""
    lay = storage.layout()
    return KvfxCache(storage.key_base(), storage.value_base(), lay.num_blocks(), lay.num_kv_heads(),
                     lay.block_size(), lay.head_size(), int(lay.dtype()), storage.device(), 0)


def device_status(device: int = 0, clear: bool = True) -> int:
    flags = u32(0)
    check(lib.kvfx_device_status(device, ctypes.byref(flags), int(clear)), "kvfx_device_status")
    return flags.value

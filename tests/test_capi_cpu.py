"""C-ABI checks that need no GPU: the library loads, exports every function
include/kvfx.h declares, and rejects bad arguments before touching CUDA."""
import ctypes
import re
from pathlib import Path

import kvflux_b200 as kv

HEADER = Path(__file__).resolve().parent.parent / "include" / "kvfx.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:const char\*|int|uint64_t|uint32_t)\s+(kvfx_\w+)\(", text, re.M)))


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(kv.lib, name), name
    assert set(names) == set(kv.KVFX_SYMBOLS)


def test_version_string():
    assert kv.lib.kvfx_version().decode().startswith("kvflux-b200")


def _cache(**kw):
    d = dict(k_base=4096, v_base=8192, num_blocks=4, num_kv_heads=2, block_size=16, head_size=8, dtype=kv.KVFX_BF16,
             device=0, reserved=0)
    d.update(kw)
    return kv.KvfxCache(**d)


def test_bad_descriptors_rejected_before_cuda():
    assert kv.lib.kvfx_write(None, None, None, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_write(ctypes.byref(_cache(num_blocks=0)), None, None, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_write(ctypes.byref(_cache(dtype=7)), None, None, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_write(ctypes.byref(_cache(reserved=1)), None, None, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_write(ctypes.byref(_cache(k_base=None)), None, None, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_write(ctypes.byref(_cache(num_blocks=2**63, head_size=2**31)), 1, 1, 1, 1, None) \
        == kv.KVFX_EOVERFLOW
    kv.lib.kvfx_write(ctypes.byref(_cache(reserved=1)), None, None, None, 1, None)
    assert b"reserved" in kv.lib.kvfx_last_error()


def test_empty_calls_return_ok_without_pointers():
    c = ctypes.byref(_cache())
    assert kv.lib.kvfx_write(c, None, None, None, 0, None) == kv.KVFX_OK
    assert kv.lib.kvfx_gather(c, None, 0, None, None, None) == kv.KVFX_OK
    assert kv.lib.kvfx_gather_batch(c, None, None, 0, 0, None, None, None) == kv.KVFX_OK
    assert kv.lib.kvfx_decode(c, None, None, None, None, 0, 0, 8, 0, 0, None, 0, None) == kv.KVFX_OK
    assert kv.lib.kvfx_attention(c, None, None, None, 0, 5, 4, None, 0, None) == kv.KVFX_OK


def test_argument_errors():
    c = ctypes.byref(_cache())
    assert kv.lib.kvfx_write(c, None, 1, 1, 3, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_gather(c, 1, 3, None, 1, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_decode(c, 1, 1, 1, 1, 1, 1, 3, 10, 0, None, 0, None) == kv.KVFX_EINVAL  # 3 % 2 != 0
    assert kv.lib.kvfx_decode(c, 1, 1, 1, 1, 1, 1, 4, 100, 0, None, 0, None) == kv.KVFX_EINVAL  # table too narrow
    assert kv.lib.kvfx_attention(c, 1, 1, 1, 6, 5, 4, None, 0, None) == kv.KVFX_EINVAL  # Lq > kv
    assert kv.lib.kvfx_copy_page(c, 0, 4, None) == kv.KVFX_ERANGE
    kv.lib.kvfx_decode(c, 1, 1, 1, 1, 1, 1, 3, 10, 0, None, 0, None)
    assert b"q_heads" in kv.lib.kvfx_last_error()


def test_workspace_sizes():
    c = ctypes.byref(_cache(num_blocks=1024, num_kv_heads=8, head_size=128))
    pps = kv.lib.kvfx_decode_pages_per_split(c, 64, 32, 8192, 64 * 4352)
    assert pps >= 4 and pps % 4 == 0
    ws = kv.lib.kvfx_decode_workspace_bytes(c, 64, 32, 8192, pps)
    splits = -(-(8192 // 16) // pps)
    assert ws >= 64 * 8 * splits * 8 * 130 * 4
    # generic shapes need no workspace
    assert kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(_cache(head_size=3)), 4, 4, 100, 0) == 0


def test_new_entry_points_validate_before_cuda():
    c = ctypes.byref(_cache())
    # kvfx_decode_append: head ratio, null inputs, narrow table, empty batch
    f = kv.lib.kvfx_decode_append
    assert f(c, 1, 1, 1, 1, 1, 1, 1, 1, 1, 3, 10, 0, None, 0, None) == kv.KVFX_EINVAL   # 3 % 2 != 0
    assert f(c, None, 1, 1, 1, 1, 1, 1, 1, 1, 4, 10, 0, None, 0, None) == kv.KVFX_EINVAL
    assert f(c, 1, 1, 1, 1, 1, 1, 1, 1, 1, 4, 100, 0, None, 0, None) == kv.KVFX_EINVAL  # 1 block < 100 tokens
    assert f(c, None, None, None, None, None, None, None, 0, 0, 4, 0, 0, None, 0, None) == kv.KVFX_OK
    # layer batches: descriptors must agree, at most KVFX_MAX_LAYERS, strides cover a layer
    two = (kv.KvfxCache * 2)(_cache(), _cache(k_base=16384, v_base=20480))
    odd = (kv.KvfxCache * 2)(_cache(), _cache(head_size=16))
    w_ = kv.lib.kvfx_write_layers
    assert w_(None, 2, 1, 1, 1024, 1, 1, None) == kv.KVFX_EINVAL
    assert w_(two, kv.KVFX_MAX_LAYERS + 1, 1, 1, 1024, 1, 1, None) == kv.KVFX_EINVAL
    assert w_(odd, 2, 1, 1, 1024, 1, 1, None) == kv.KVFX_EINVAL
    assert w_(two, 2, 1, 1, 16, 1, 1, None) == kv.KVFX_EINVAL                      # stride < 2 x 8 x 2 B x 1 token
    assert w_(two, 2, None, None, 0, None, 0, None) == kv.KVFX_OK                  # no tokens
    assert w_(two, 0, None, None, 0, None, 5, None) == kv.KVFX_OK                  # no layers
    g = kv.lib.kvfx_gather_layers
    assert g(odd, 2, 1, 1, 1, 1, 1, 1, 4096, None) == kv.KVFX_EINVAL
    assert g(two, 2, None, 1, 1, 1, 1, 1, 4096, None) == kv.KVFX_EINVAL
    assert g(two, 2, 1, 1, 70000, 1, 1, 1, 4096, None) == kv.KVFX_EINVAL          # batch above 65535
    assert g(two, 2, None, None, 0, 0, None, None, 0, None) == kv.KVFX_OK
    # batched attention: sequence count, head ratio, shapes, table width, null arrays
    a = kv.lib.kvfx_attention_batch
    n = kv.KVFX_MAX_PREFILL_SEQS + 1
    ptrs = (ctypes.c_void_p * n)(*[64] * n)
    ones = (ctypes.c_uint64 * n)(*[4] * n)
    assert a(c, n, ptrs, ptrs, 1, 1, ones, ones, 4, None, 0, None) == kv.KVFX_EINVAL
    assert a(c, 2, ptrs, ptrs, 1, 1, ones, ones, 3, None, 0, None) == kv.KVFX_EINVAL      # 3 % 2 != 0
    qt, kt = (ctypes.c_uint64 * 2)(4, 9), (ctypes.c_uint64 * 2)(4, 8)
    assert a(c, 2, ptrs, ptrs, 1, 1, qt, kt, 4, None, 0, None) == kv.KVFX_EINVAL         # 9 queries > 8 tokens
    kt2 = (ctypes.c_uint64 * 2)(4, 40)
    assert a(c, 2, ptrs, ptrs, 1, 2, qt, kt2, 4, None, 0, None) == kv.KVFX_EINVAL        # 40 tokens > 2 blocks of 16
    assert a(c, 2, None, ptrs, 1, 1, ones, ones, 4, None, 0, None) == kv.KVFX_EINVAL
    zero = (ctypes.c_uint64 * 2)(0, 0)
    assert a(c, 2, ptrs, ptrs, None, 0, zero, kt, 4, None, 0, None) == kv.KVFX_OK         # no queries
    assert a(c, 0, None, None, None, 0, None, None, 4, None, 0, None) == kv.KVFX_OK
    # the failure-detection self-test refuses a negative ordinal before CUDA
    assert kv.lib.kvfx_selftest_wait_timeout(-1) == kv.KVFX_EINVAL

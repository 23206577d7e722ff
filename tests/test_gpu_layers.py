"""Layer batches: kvfx_write_layers / kvfx_gather_layers (C ABI) and
write_paged_kv_layers / read_paged_kv_layers (C++ API over one
PagedKVStorage per layer on one pool). Byte-exact against the oracle's
single-layer write and gather applied to each layer, on the 16-byte kernels
(head_size 64/128 16-bit, FP32 32) and on the per-layer fallback (rows that are
not 16-byte multiples, padded layer strides); sentinels past each output stay
untouched."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from gpu_util import d2h
from kvflux_b200 import workloads as w
from test_gpu_capi import Cache, call, u64

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def clear_status(cuda):
    kv.device_status(0, clear=True)
    yield


def _layers(n, nb, heads, bs, hd, dtype, seed):
    caches = [Cache(nb, heads, bs, hd, dtype, seed=seed + 17 * l) for l in range(n)]
    arr = (kv.KvfxCache * n)(*[c.desc for c in caches])
    return caches, arr


@pytest.mark.parametrize("dtype,hd,bs,heads,layers,pad", [
    ("bfloat16", 128, 16, 8, 6, 0),      # 16-byte kernel, packed layers
    ("float16", 64, 16, 2, 3, 48),       # 16-byte kernel, padded layer stride
    ("float32", 32, 8, 2, 2, 0),
    ("bfloat16", 3, 4, 2, 4, 6),         # 6-byte rows: one launch per layer
    ("float32", 5, 2, 3, 1, 0),
])
def test_write_layers_byte_exact(dtype, hd, bs, heads, layers, pad):
    caches, arr = _layers(layers, 40, heads, bs, hd, dtype, seed=hd + layers)
    n = 29
    slots = w.permutation(9 + hd, np.arange(40 * bs))[:n].astype(np.uint64)
    row = hd * w.ELEM_BYTES[dtype]
    per_layer = n * heads * row
    stride = per_layer + pad
    kn = np.zeros(stride * layers, np.uint8)
    vn = np.zeros_like(kn)
    for l in range(layers):
        kn[l * stride:l * stride + per_layer] = w.encode(w.normal(100 + l, n * heads * hd), dtype).view(np.uint8)
        vn[l * stride:l * stride + per_layer] = w.encode(w.normal(200 + l, n * heads * hd), dtype).view(np.uint8)
    dk, dv = torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda()
    call(kv.lib.kvfx_write_layers, arr, layers, dk.data_ptr(), dv.data_ptr(), stride, u64(slots), n, None)
    assert kv.device_status(0) == 0
    for l, c in enumerate(caches):
        hk, hv = c.host_k.copy(), c.host_v.copy()
        oracle.write(hk, hv, c.nb, c.h, c.bs, c.row, kn[l * stride:l * stride + per_layer],
                     vn[l * stride:l * stride + per_layer], slots)
        gk, gv = c.device_bytes()
        assert np.array_equal(gk, hk) and np.array_equal(gv, hv), f"layer {l}"


@pytest.mark.parametrize("dtype,hd,bs,heads,layers,pad", [
    ("bfloat16", 128, 16, 8, 5, 0),
    ("float16", 64, 16, 2, 3, 32),
    ("float32", 32, 16, 1, 2, 0),
    ("bfloat16", 3, 4, 2, 3, 10),        # per-layer fallback
])
def test_gather_layers_byte_exact_with_sentinels(dtype, hd, bs, heads, layers, pad):
    lens = [1, bs - 1, bs, 3 * bs + 5, 100]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    caches, arr = _layers(layers, nb, heads, bs, hd, dtype, seed=3 * hd + layers)
    ids = w.permutation(hd + 1, np.arange(nb))
    width = max((l + bs - 1) // bs for l in lens)
    table = np.full((len(lens), width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (l + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    row = hd * w.ELEM_BYTES[dtype]
    strides = [l * heads * row + pad for l in lens]
    stride = max(strides)
    seq_bytes = stride * layers + 64
    ko = torch.full((len(lens) * seq_bytes + 16,), 0xA5, dtype=torch.uint8, device="cuda")
    vo = torch.full_like(ko, 0x5A)
    base = (ko.data_ptr() + 15) // 16 * 16 - ko.data_ptr()
    kp = np.array([ko.data_ptr() + base + r * seq_bytes for r in range(len(lens))], np.uint64)
    vp = np.array([vo.data_ptr() + base + r * seq_bytes for r in range(len(lens))], np.uint64)
    call(kv.lib.kvfx_gather_layers, arr, layers, u64(table), u64(np.array(lens, np.uint64)), len(lens), width,
         u64(kp), u64(vp), stride, None)
    assert kv.device_status(0) == 0
    gk, gv = ko.cpu().numpy(), vo.cpu().numpy()
    for r, L in enumerate(lens):
        for l, c in enumerate(caches):
            ek, ev = oracle.gather(c.host_k, c.host_v, c.nb, c.h, c.bs, c.row, table[r], L)
            o = base + r * seq_bytes + l * stride
            n = L * heads * row
            assert np.array_equal(gk[o:o + n], ek) and np.array_equal(gv[o:o + n], ev), (r, l)
            assert (gk[o + n:o + stride] == 0xA5).all() and (gv[o + n:o + stride] == 0x5A).all(), "padding written"


def test_layers_argument_errors():
    caches, arr = _layers(2, 8, 2, 16, 128, "bfloat16", seed=1)
    x = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = x.data_ptr()
    f = kv.lib.kvfx_write_layers
    assert f(arr, 2, p, p, 16, p, 1, None) == kv.KVFX_EINVAL            # stride below one layer's rows
    assert f(arr, 129, p, p, 1024, p, 1, None) == kv.KVFX_EINVAL        # above KVFX_MAX_LAYERS
    assert f(arr, 0, p, p, 0, p, 1, None) == kv.KVFX_OK                 # no layers: nothing to do
    bad = (kv.KvfxCache * 2)(caches[0].desc, kv.KvfxCache(caches[1].base, caches[1].base + caches[1].cache_bytes,
                                                          8, 2, 16, 64, kv.KVFX_BF16, 0, 0))
    assert f(bad, 2, p, p, 8192, p, 1, None) == kv.KVFX_EINVAL          # head sizes differ
    g = kv.lib.kvfx_gather_layers
    assert g(arr, 2, None, p, 1, 1, p, p, 4096, None) == kv.KVFX_EINVAL
    assert g(bad, 2, p, p, 1, 1, p, p, 4096, None) == kv.KVFX_EINVAL


# -------------------------------------------------------------- C++ API ---

@pytest.mark.parametrize("dtype,hd", [("bfloat16", 128), ("float32", 3)])
def test_layer_api_roundtrip_matches_single_layer_calls(dtype, hd):
    layers, heads, bs = 4, 2, 16
    pool = kv.PhysicalBlockPool(64, bs)
    w.fragment_pool(pool, np.arange(64), seed=5)
    stores = [kv.PagedKVStorage(pool, heads, hd, w.DTYPES[dtype], 0) for _ in range(layers)]
    seq = kv.SequenceState(1, pool)
    seq.append_tokens(77)
    row = heads * hd * w.ELEM_BYTES[dtype]
    kn = np.concatenate([w.encode(w.normal(10 + l, 77 * heads * hd), dtype).view(np.uint8) for l in range(layers)])
    vn = np.concatenate([w.encode(w.normal(20 + l, 77 * heads * hd), dtype).view(np.uint8) for l in range(layers)])
    slots = kv.build_slot_mapping([(seq, t) for t in range(77)])
    kv.write_paged_kv_layers(stores, torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda(), slots)
    ko = torch.empty(layers * 77 * row, dtype=torch.uint8, device="cuda")
    vo = torch.empty_like(ko)
    kv.read_paged_kv_layers(stores, seq, ko, vo)
    assert np.array_equal(ko.cpu().numpy(), kn) and np.array_equal(vo.cpu().numpy(), vn)
    for l, st in enumerate(stores):  # each layer also reads back alone
        k1 = torch.empty(77 * row, dtype=torch.uint8, device="cuda")
        v1 = torch.empty_like(k1)
        kv.read_paged_kv(st, seq, k1, v1)
        assert np.array_equal(k1.cpu().numpy(), kn[l * 77 * row:(l + 1) * 77 * row])
        assert np.array_equal(v1.cpu().numpy(), vn[l * 77 * row:(l + 1) * 77 * row])


def test_layer_api_errors_in_reference_order():
    pool = kv.PhysicalBlockPool(16, 16)
    other = kv.PhysicalBlockPool(16, 16)
    a = kv.PagedKVStorage(pool, 2, 64, kv.DType.BFloat16, 0)
    b = kv.PagedKVStorage(pool, 2, 64, kv.DType.BFloat16, 0)
    odd = kv.PagedKVStorage(pool, 2, 32, kv.DType.BFloat16, 0)
    foreign = kv.PagedKVStorage(other, 2, 64, kv.DType.BFloat16, 0)
    seq = kv.SequenceState(1, pool)
    seq.append_tokens(20)
    x = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        kv.write_paged_kv_layers([], x, x, [0])
    with pytest.raises(ValueError):
        kv.write_paged_kv_layers([a, odd], x, x, [0])
    kv.write_paged_kv_layers([a, b], None, None, [])          # empty mapping returns first
    with pytest.raises(ValueError):
        kv.write_paged_kv_layers([a, b], None, x, [0])
    with pytest.raises(IndexError):
        kv.write_paged_kv_layers([a, b], x, x, [16 * 16])
    with pytest.raises(ValueError):
        kv.write_paged_kv_layers([a, b], x, x, [3, 3])
    with pytest.raises(ValueError):
        kv.write_paged_kv_layers([a, b], np.zeros(8192, np.uint8), x, [3])
    with pytest.raises(ValueError):
        kv.read_paged_kv_layers([a, foreign], seq, x, x)
    with pytest.raises(ValueError):
        kv.read_paged_kv_layers([a, b], seq, x, x)             # K and V outputs overlap
    empty = kv.SequenceState(2, pool)
    kv.read_paged_kv_layers([a, b], empty, None, None)        # empty sequence returns first
    assert kv.device_status(0) == 0

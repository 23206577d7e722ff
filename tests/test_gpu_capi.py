"""Parity of every C-ABI entry point (include/kvfx.h) against the CPU oracle
on seeded inputs: byte-exact for write, gather and page copy; attention within
max_abs_err 1e-5 for FP32 caches and 2e-3 for FP16/BF16 caches (the stated
tolerances of the path), against the FP64 reference_attention restatement.
Shapes cover the fast kernels (16-bit caches, head_size 64/128, block 16,
GQA group <= 8) and the generic ones (FP32, head_size 1..32, block 2..8,
group 16), ragged and single-token sequences, partial last pages over
poisoned (NaN) cache bytes, many split-K splits, and out-of-range ids."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from gpu_util import d2h, h2d, memset
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 2e-3}


class Cache:
    """A raw paged cache on the GPU plus its host mirror."""

    def __init__(self, num_blocks, heads, bs, hd, dtype, seed, poison=None):
        self.nb, self.h, self.bs, self.hd, self.dtype = num_blocks, heads, bs, hd, dtype
        self.elem = w.ELEM_BYTES[dtype]
        self.row = hd * self.elem
        self.page = heads * bs * self.row
        self.cache_bytes = num_blocks * self.page
        self.buf = torch.empty(2 * self.cache_bytes + 256, dtype=torch.uint8, device="cuda")
        self.base = (self.buf.data_ptr() + 255) // 256 * 256
        n = num_blocks * heads * bs * hd
        if poison is None:
            hk = w.encode(w.normal(seed, n), dtype).view(np.uint8)
            hv = w.encode(w.normal(seed + 1, n), dtype).view(np.uint8)
        else:
            hk = np.full(self.cache_bytes, poison, np.uint8)
            hv = hk.copy()
        self.host_k, self.host_v = hk.copy(), hv.copy()
        h2d(self.base, hk)
        h2d(self.base + self.cache_bytes, hv)
        self.desc = kv.KvfxCache(self.base, self.base + self.cache_bytes, num_blocks, heads, bs, hd,
                                 kv.DTYPE_CODE[dtype], 0, 0)

    def device_bytes(self):
        return d2h(self.base, self.cache_bytes), d2h(self.base + self.cache_bytes, self.cache_bytes)


def u64(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint64).view(np.int64)).cuda()


def call(fn, *args):
    """Calls a C-ABI entry point; tensor arguments pass their device address and
    stay referenced (alive) until the launch has completed."""
    keep = [a for a in args if isinstance(a, torch.Tensor)]
    rc = fn(*[a.data_ptr() if isinstance(a, torch.Tensor) else a for a in args])
    torch.cuda.synchronize()
    del keep
    kv.check(rc, fn.__name__)


@pytest.fixture(autouse=True)
def clear_status(cuda):
    kv.device_status(0, clear=True)
    yield


@pytest.mark.parametrize("dtype,hd,bs,heads", [("bfloat16", 128, 16, 8), ("float16", 64, 16, 2), ("float32", 3, 4, 2),
                                               ("bfloat16", 1, 2, 1), ("float32", 32, 16, 2), ("float16", 5, 8, 3)])
def test_write_byte_exact(dtype, hd, bs, heads):
    c = Cache(48, heads, bs, hd, dtype, seed=11)
    n = 37
    slots = w.permutation(5 + hd, np.arange(c.nb * bs))[:n].astype(np.uint64)
    kn = w.encode(w.normal(21, n * heads * hd), dtype).view(np.uint8)
    vn = w.encode(w.normal(22, n * heads * hd), dtype).view(np.uint8)
    dk, dv = torch.from_numpy(kn.copy()).cuda(), torch.from_numpy(vn.copy()).cuda()
    call(kv.lib.kvfx_write, ctypes.byref(c.desc), dk.data_ptr(), dv.data_ptr(), u64(slots), n, None)
    oracle.write(c.host_k, c.host_v, c.nb, heads, bs, c.row, kn, vn, slots)
    gk, gv = c.device_bytes()
    assert np.array_equal(gk, c.host_k) and np.array_equal(gv, c.host_v)
    assert kv.device_status(0) == 0


# Rows of 16-byte multiples take the direct page kernel (16 heads of 128 bf16:
# a 64 KiB page), other rows the SIMT one.
@pytest.mark.parametrize("dtype,hd,bs,heads", [("bfloat16", 128, 16, 8), ("float16", 64, 16, 4), ("float32", 3, 4, 2),
                                               ("float32", 32, 16, 2), ("bfloat16", 5, 8, 3), ("bfloat16", 128, 16, 16)])
@pytest.mark.parametrize("length", [1, 15, 16, 17, 333])
def test_gather_byte_exact_with_sentinel(dtype, hd, bs, heads, length):
    c = Cache(128, heads, bs, hd, dtype, seed=31)
    pages = (length + bs - 1) // bs
    blocks = w.permutation(length * 7 + hd, np.arange(c.nb))[:pages].astype(np.uint64)
    out_bytes = length * heads * c.row
    ko = torch.full((out_bytes + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    vo = torch.full((out_bytes + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    call(kv.lib.kvfx_gather, ctypes.byref(c.desc), u64(blocks), length, ko.data_ptr(), vo.data_ptr(),
         None)
    ek, ev = oracle.gather(c.host_k, c.host_v, c.nb, heads, bs, c.row, blocks, length)
    gk, gv = ko.cpu().numpy(), vo.cpu().numpy()
    assert np.array_equal(gk[:out_bytes], ek) and np.array_equal(gv[:out_bytes], ev)
    assert (gk[out_bytes:] == 0xA5).all() and (gv[out_bytes:] == 0xA5).all()


@pytest.mark.parametrize("dtype,hd", [("bfloat16", 128), ("float32", 3)])
def test_gather_batch_byte_exact(dtype, hd):
    heads, bs = 4, 16
    c = Cache(256, heads, bs, hd, dtype, seed=41)
    lens = np.array([1, 16, 17, 250, 0, 64], np.uint64)
    width = int(max((int(l) + bs - 1) // bs for l in lens))
    ids = w.permutation(3, np.arange(c.nb))
    table = np.full((len(lens), width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (int(l) + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    outs_k = [torch.full((max(int(l), 1) * heads * c.row + 32,), 0xA5, dtype=torch.uint8, device="cuda") for l in lens]
    outs_v = [torch.full_like(t, 0xA5) for t in outs_k]
    pk = u64(np.array([t.data_ptr() for t in outs_k], np.uint64))
    pv = u64(np.array([t.data_ptr() for t in outs_v], np.uint64))
    call(kv.lib.kvfx_gather_batch, ctypes.byref(c.desc), u64(table), u64(lens), len(lens),
         width, pk.data_ptr(), pv.data_ptr(), None)
    for r, l in enumerate(lens):
        l = int(l)
        ek, ev = oracle.gather(c.host_k, c.host_v, c.nb, heads, bs, c.row, table[r], l)
        gk, gv = outs_k[r].cpu().numpy(), outs_v[r].cpu().numpy()
        nb = l * heads * c.row
        assert np.array_equal(gk[:nb], ek) and np.array_equal(gv[:nb], ev)
        assert (gk[nb:] == 0xA5).all() and (gv[nb:] == 0xA5).all()
    assert kv.device_status(0) == 0


@pytest.mark.parametrize("dtype,hd,bs,heads", [("bfloat16", 128, 16, 8), ("float32", 3, 4, 2)])
def test_copy_page_byte_exact(dtype, hd, bs, heads):
    c = Cache(16, heads, bs, hd, dtype, seed=51)
    call(kv.lib.kvfx_copy_page, ctypes.byref(c.desc), 3, 11, None)
    gk, gv = c.device_bytes()
    ek, ev = c.host_k.copy(), c.host_v.copy()
    ek[11 * c.page:12 * c.page] = ek[3 * c.page:4 * c.page]
    ev[11 * c.page:12 * c.page] = ev[3 * c.page:4 * c.page]
    assert np.array_equal(gk, ek) and np.array_equal(gv, ev)
    assert kv.lib.kvfx_copy_page(ctypes.byref(c.desc), 3, 3, None) == kv.KVFX_EINVAL
    assert kv.lib.kvfx_copy_page(ctypes.byref(c.desc), 3, 16, None) == kv.KVFX_ERANGE


def _page_order(order, nb, seed):
    """Physical page ids handed out in order: "perm" (fragmented), "seq" (one
    run from page 0, as a fresh free list gives them), "mixed" (runs ending on
    the pool's last page, some broken by a swapped pair, some reversed)."""
    if order == "perm":
        return w.permutation(seed, np.arange(nb))
    ids = np.arange(nb)
    if order == "mixed":
        ids = np.roll(ids, -8)  # the runs that reach the end of the pool wrap to page 0
        for t in range(0, nb // 8):
            if t % 3 == 1:
                ids[8 * t + 3], ids[8 * t + 4] = ids[8 * t + 4], ids[8 * t + 3]
            elif t % 3 == 2:
                ids[8 * t:8 * t + 8] = ids[8 * t:8 * t + 8][::-1].copy()
    return ids


def _decode_case(dtype, hd, bs, kvh, group, lens, seed, pps=0, poison_tail=True, order="perm"):
    c = Cache(int(sum((l + bs - 1) // bs for l in lens)) + 8, kvh, bs, hd, dtype, seed=seed)
    qh = kvh * group
    batch = len(lens)
    width = max((l + bs - 1) // bs for l in lens)
    ids = _page_order(order, c.nb, seed + 3)
    table = np.full((batch, width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (l + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    if poison_tail:
        # Token slots past each sequence's end hold NaN bit patterns.
        nan = {"bfloat16": 0xFFFF, "float16": 0xFFFF, "float32": 0xFFFFFFFF}[dtype]
        hk = c.host_k.view(np.uint16 if c.elem == 2 else np.uint32)
        hv = c.host_v.view(np.uint16 if c.elem == 2 else np.uint32)
        for r, l in enumerate(lens):
            last = int(table[r, (l - 1) // bs])
            for t in range(l % bs or bs, bs):
                for h in range(kvh):
                    o = ((last * kvh + h) * bs + t) * hd
                    hk[o:o + hd] = nan
                    hv[o:o + hd] = nan
        h2d(c.base, c.host_k)
        h2d(c.base + c.cache_bytes, c.host_v)
    q = w.normal(seed + 9, batch * qh * hd)
    return c, table, np.array(lens, np.uint64), q, qh


@pytest.mark.parametrize("dtype,hd,bs,kvh,group", [
    ("bfloat16", 128, 16, 8, 4), ("bfloat16", 128, 16, 2, 8), ("float16", 128, 16, 4, 2), ("bfloat16", 64, 16, 4, 1),
    ("float16", 64, 16, 2, 8), ("float32", 64, 16, 2, 4), ("float32", 3, 4, 2, 2), ("bfloat16", 32, 8, 2, 16),
    ("float16", 1, 2, 1, 3)])
def test_decode_matches_oracle(dtype, hd, bs, kvh, group):
    lens = [1, 15, 16, 17, 100, 513, 1000, 2049]
    c, table, lens_np, q, qh = _decode_case(dtype, hd, bs, kvh, group, lens, seed=hd * 31 + group)
    batch = len(lens)
    max_len = int(lens_np.max())
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), batch, qh, max_len, 0)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q).cuda()
    out = torch.full((batch * qh * hd + 1,), 12345.0, device="cuda")
    for _ in range(2):  # the second call reuses the workspace (counters must have been reset)
        call(kv.lib.kvfx_decode, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(table),
             u64(lens_np), batch, table.shape[1], qh, max_len, 0, ws.data_ptr(), ws.numel(), None)
        got = out.cpu().numpy()
        exp = oracle.decode_batch(c.host_k, c.host_v, w.DTYPE_CODE[dtype], c.nb, kvh, bs, hd, table, lens_np, qh, q,
                                  threads=8)
        assert np.isfinite(got[:-1]).all()
        err = float(np.abs(got[:-1] - exp).max())
        assert err < TOL[dtype], err
        assert got[-1] == 12345.0
    assert kv.device_status(0) == 0


@pytest.mark.parametrize("pps", [4, 8, 64, 4096])
def test_decode_split_k_merge(pps):
    lens = [5000, 33, 4097, 777]
    c, table, lens_np, q, qh = _decode_case("bfloat16", 128, 16, 4, 4, lens, seed=77)
    batch, max_len = len(lens), int(lens_np.max())
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), batch, qh, max_len, pps)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q).cuda()
    out = torch.empty(batch * qh * 128, device="cuda")
    call(kv.lib.kvfx_decode, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(table),
         u64(lens_np), batch, table.shape[1], qh, max_len, pps, ws.data_ptr(), ws.numel(), None)
    exp = oracle.decode_batch(c.host_k, c.host_v, 1, c.nb, 4, 16, 128, table, lens_np, qh, q, threads=8)
    assert float(np.abs(out.cpu().numpy() - exp).max()) < TOL["bfloat16"]


def test_decode_workspace_serves_changing_shapes_without_clearing():
    """One workspace, zero-filled once, through launches whose batch, lengths
    and split sizes change (so each launch's partials cover bytes that other
    launches' layouts never use as counters only if the counters sit apart):
    every launch matches the oracle, and the counters it used end at zero."""
    lens_all = [5000, 33, 4097, 777, 1, 2500, 16, 9000, 300, 4100, 64, 1999]
    c, table, lens_np, q, qh = _decode_case("bfloat16", 128, 16, 4, 4, lens_all, seed=13)
    big = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), len(lens_all), qh, int(lens_np.max()), 4)
    ws = torch.zeros(int(big), dtype=torch.uint8, device="cuda")
    hd = 128
    for rows, pps in [(list(range(12)), 4), ([0, 2], 8), (list(range(12)), 64), ([7, 9, 0, 3, 5], 4),
                      (list(range(12)), 0), ([1], 0), (list(range(12)), 4)]:
        t = table[rows]
        ln = lens_np[rows]
        qq = q.reshape(len(lens_all), -1)[rows].reshape(-1).copy()
        qd = torch.from_numpy(qq).cuda()
        out = torch.full((len(rows) * qh * hd,), float("nan"), device="cuda")
        call(kv.lib.kvfx_decode, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(t), u64(ln), len(rows),
             t.shape[1], qh, int(ln.max()), pps, ws.data_ptr(), ws.numel(), None)
        exp = oracle.decode_batch(c.host_k, c.host_v, 1, c.nb, 4, 16, hd, t, ln, qh, qq, threads=8)
        got = out.cpu().numpy()
        assert np.isfinite(got).all(), (rows, pps)
        assert float(np.abs(got - exp).max()) < TOL["bfloat16"], (rows, pps)
        counters = ws[:65536 * 4 * 2].view(torch.int32)
        assert int(counters.abs().sum()) == 0, (rows, pps)
    assert kv.device_status(0) == 0


@pytest.mark.parametrize("dtype,pps", [("bfloat16", 8), ("bfloat16", 0), ("float16", 64)])
def test_decode_rescale_path(dtype, pps):
    """Q scaled by 8 (scores with ~8x the spread): running maxima rise by more
    than the lazy-rescale threshold inside splits, and splits with very
    different maxima are merged."""
    lens = [3000, 700, 129, 4100]
    c, table, lens_np, q, qh = _decode_case(dtype, 128, 16, 4, 4, lens, seed=91)
    q = q * np.float32(8.0)
    batch, max_len = len(lens), int(lens_np.max())
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), batch, qh, max_len, pps)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q).cuda()
    out = torch.empty(batch * qh * 128, device="cuda")
    call(kv.lib.kvfx_decode, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(table),
         u64(lens_np), batch, table.shape[1], qh, max_len, pps, ws.data_ptr(), ws.numel(), None)
    exp = oracle.decode_batch(c.host_k, c.host_v, w.DTYPE_CODE[dtype], c.nb, 4, 16, 128, table, lens_np, qh, q,
                              threads=8)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert float(np.abs(got - exp).max()) < TOL[dtype]
    assert kv.device_status(0) == 0


@pytest.mark.parametrize("dtype,hd,bs,kvh,group,lq,kvlen", [
    ("bfloat16", 128, 16, 2, 4, 1, 300), ("bfloat16", 128, 16, 2, 4, 37, 300), ("float32", 4, 4, 2, 2, 10, 10),
    ("float16", 64, 16, 1, 8, 64, 64), ("float32", 3, 2, 3, 1, 5, 9)])
def test_attention_single_sequence(dtype, hd, bs, kvh, group, lq, kvlen):
    c, table, _, _, qh = _decode_case(dtype, hd, bs, kvh, group, [kvlen], seed=lq + kvlen)
    blocks = table[0]
    q = w.normal(lq * 3 + hd, lq * qh * hd)
    ws_bytes = kv.lib.kvfx_attention_workspace_bytes(ctypes.byref(c.desc), lq, kvlen, qh)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    qd = torch.from_numpy(q).cuda()
    out = torch.full((lq * qh * hd + 1,), 12345.0, device="cuda")
    call(kv.lib.kvfx_attention, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(blocks), lq,
         kvlen, qh, ws.data_ptr(), ws.numel(), None)
    exp = oracle.attention_rows(c.host_k, c.host_v, w.DTYPE_CODE[dtype], c.nb, kvh, bs, hd, blocks, lq, kvlen, qh, q,
                                threads=8)
    got = out.cpu().numpy()
    assert float(np.abs(got[:-1] - exp).max()) < TOL[dtype]
    assert got[-1] == 12345.0


def test_out_of_range_ids_are_flagged_not_followed():
    c = Cache(8, 2, 4, 8, "float32", seed=3)
    bad = np.array([1, 99], np.uint64)  # page 99 does not exist
    ko = torch.zeros(8 * 2 * 8, dtype=torch.float32, device="cuda")
    vo = torch.zeros_like(ko)
    call(kv.lib.kvfx_gather, ctypes.byref(c.desc), u64(bad), 8, ko.data_ptr(), vo.data_ptr(), None)
    assert kv.device_status(0) & kv.KVFX_FLAG_BAD_INDEX
    slots = np.array([0, 8 * 4 + 5], np.uint64)  # second slot is beyond the cache
    kn = torch.ones(2 * 2 * 8, device="cuda")
    call(kv.lib.kvfx_write, ctypes.byref(c.desc), kn.data_ptr(), kn.data_ptr(), u64(slots), 2, None)
    assert kv.device_status(0) & kv.KVFX_FLAG_BAD_INDEX
    # Only slot 0 (page 0, offset 0) changed: both of its head rows hold the new ones.
    gk, _ = c.device_bytes()
    page_rows = gk.view(np.float32).reshape(8, 2, 4, 8)
    assert (page_rows[0, :, 0, :] == 1.0).all()
    assert np.array_equal(page_rows[1:], c.host_k.view(np.float32).reshape(8, 2, 4, 8)[1:])


def test_workspace_too_small_is_rejected():
    c = Cache(64, 2, 16, 128, "bfloat16", seed=4)
    lens = np.array([1000], np.uint64)
    table = np.arange(63, dtype=np.uint64)[None, :]
    need = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), 1, 8, 1000, 4)
    assert need > 0
    q = torch.zeros(8 * 128, device="cuda")
    td, ld = u64(table), u64(lens)
    rc = kv.lib.kvfx_decode(ctypes.byref(c.desc), q.data_ptr(), q.data_ptr(), td.data_ptr(), ld.data_ptr(), 1, 63, 8,
                            1000, 4, None, 0, None)
    assert rc == kv.KVFX_ENOSPACE


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("kvh,group,lq,kvlen,qmul", [
    (2, 4, 2, 2, 1.0), (1, 8, 127, 127, 1.0), (2, 1, 128, 128, 1.0), (2, 4, 129, 129, 1.0), (1, 4, 300, 300, 1.0),
    (2, 4, 100, 333, 1.0), (1, 2, 64, 1000, 1.0), (2, 3, 200, 517, 1.0), (2, 2, 256, 256, 1.0),
    # Scores with ~8x the spread: running row maxima rise by more than 8
    # (base 2) after the first tile, so O is rescaled in TMEM.
    (1, 4, 300, 300, 8.0), (2, 3, 96, 700, 8.0)])
@pytest.mark.parametrize("order", ["perm", "seq", "mixed"])
def test_prefill_tensor_core_path(dtype, kvh, group, lq, kvlen, qmul, order):
    """Causal prefill on the tcgen05 kernel (16-bit cache, head_size 128,
    block 16): suffix-aligned queries, partial query and KV tiles, NaN-poisoned
    slots past the sequence end, GQA groups 1..8, pages fragmented or in
    consecutive runs as a free list hands them out; max |err| against the
    FP64 oracle."""
    c, table, _, _, qh = _decode_case(dtype, 128, 16, kvh, group, [kvlen], seed=lq * 7 + kvlen + group,
                                      order=order)
    blocks = table[0]
    q = w.normal(lq + 11 * kvlen, lq * qh * 128) * np.float32(qmul)
    qd = torch.from_numpy(q).cuda()
    out = torch.full((lq * qh * 128 + 1,), 12345.0, device="cuda")
    call(kv.lib.kvfx_attention, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(blocks), lq, kvlen, qh,
         None, 0, None)
    exp = oracle.attention_rows(c.host_k, c.host_v, w.DTYPE_CODE[dtype], c.nb, kvh, 16, 128, blocks, lq, kvlen, qh,
                                q, threads=8)
    got = out.cpu().numpy()
    assert np.isfinite(got[:-1]).all()
    err = float(np.abs(got[:-1] - exp).max())
    assert err < TOL[dtype], err
    assert got[-1] == 12345.0
    assert kv.device_status(0) == 0
    if qmul > 1:
        assert _rescaled_rows(c, dtype, blocks, lq, kvlen, kvh, group, q) > 0


def _rescaled_rows(c, dtype, blocks, lq, kvlen, kvh, group, q, tile=64):
    """Rows (x heads) whose score maximum over some later 64-token tile exceeds
    the first tile's by more than 8 in base 2: the cases that take the
    kernel's O-rescale path."""
    raw = c.host_k.view(np.uint16).reshape(c.nb, kvh, 16, 128)
    f = (raw.astype(np.uint32) << 16).view(np.float32) if dtype == "bfloat16" else \
        raw.view(np.float16).astype(np.float32)
    npg = (kvlen + 15) // 16
    keys = f[blocks[:npg].astype(np.int64)].transpose(1, 0, 2, 3).reshape(kvh, -1, 128)[:, :kvlen]
    qh = kvh * group
    qs = q.reshape(lq, qh, 128).astype(np.float64)
    pos = kvlen - lq + np.arange(lq)
    count = 0
    for h in range(qh):
        s = qs[:, h] @ keys[h // group].T.astype(np.float64) * (1.4426950408889634 / np.sqrt(128.0))
        s[np.arange(kvlen)[None, :] > pos[:, None]] = -np.inf
        first = s[:, :tile].max(axis=1)
        later = s[:, tile:].max(axis=1) if kvlen > tile else np.full(lq, -np.inf)
        count += int((later > first + 8).sum())
    return count


def test_prefill_long_sequence_sampled_rows():
    """4096-token causal prefill (config 4's per-sequence shape, 32/8 heads):
    first 192 rows, rows across the middle and the last 64 rows checked in
    full against the oracle."""
    kvh, group, L = 8, 4, 4096
    c, table, _, _, qh = _decode_case("bfloat16", 128, 16, kvh, group, [L], seed=4096)
    blocks = table[0]
    q = w.normal(77, L * qh * 128)
    qd = torch.from_numpy(q).cuda()
    out = torch.empty(L * qh * 128, device="cuda")
    call(kv.lib.kvfx_attention, ctypes.byref(c.desc), qd.data_ptr(), out.data_ptr(), u64(blocks), L, L, qh,
         None, 0, None)
    got = out.cpu().numpy().reshape(L, -1)
    for lo, hi in [(0, 192), (2000, 2056), (L - 64, L)]:
        exp = oracle.attention_rows(c.host_k, c.host_v, 1, c.nb, kvh, 16, 128, blocks, L, L, qh, q, row_begin=lo,
                                    row_end=hi, threads=16).reshape(L, -1)
        err = float(np.abs(got[lo:hi] - exp[lo:hi]).max())
        assert err < TOL["bfloat16"], (lo, err)

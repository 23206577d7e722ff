"""kvfx_decode_noalloc: batch decode for callers that cannot allocate device
memory (engines that give all device memory to their KV pool up front, loops
that cannot take cudaMalloc's implicit synchronisation, embedders whose
allocator policy forbids it). Its split-K scratch is a static device array
inside the library instead of a caller workspace.

Called through the C ABI twice in a row (the second call finds the previous
call's contents in the shared array) and compared with kvfx_decode, the
entry point with a caller workspace, and with the oracle's decode, within the
tolerance of the decode tests (2e-3 for bf16/fp16 caches, 1e-5 for FP32
caches). A batch large enough that the static array forces longer splits
than kvfx_decode would choose is checked the same way, interleaved with
calls of other shapes and head counts (the array's counters must be zero at
every call), and an out-of-range page id is reported through
kvfx_device_status. This file sorts last so that a run stopping at the first
failure has run every other test before it."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from gpu_util import d2h, h2d
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu


def _case(dtype, hd, kvh, group, lens, seed):
    bs = 16
    elem = w.ELEM_BYTES[dtype]
    nb = int(sum((l + bs - 1) // bs for l in lens)) + 4
    cache_bytes = nb * kvh * bs * hd * elem
    buf = torch.empty(2 * cache_bytes + 256, dtype=torch.uint8, device="cuda")
    base = (buf.data_ptr() + 255) // 256 * 256
    n = nb * kvh * bs * hd
    hk = w.encode(w.normal(seed, n), dtype).view(np.uint8)
    hv = w.encode(w.normal(seed + 1, n), dtype).view(np.uint8)
    h2d(base, hk)
    h2d(base + cache_bytes, hv)
    desc = kv.KvfxCache(base, base + cache_bytes, nb, kvh, bs, hd, w.DTYPE_CODE[dtype], 0, 0)
    width = max((l + bs - 1) // bs for l in lens)
    ids = w.permutation(seed + 2, np.arange(nb))
    table = np.full((len(lens), width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (l + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    qh = kvh * group
    q = w.normal(seed + 3, len(lens) * qh * hd)
    return dict(buf=buf, desc=desc, table=table, lens=np.array(lens, np.uint64), q=q, qh=qh, hd=hd, kvh=kvh, nb=nb,
                hk=hk, hv=hv, dtype=dtype)


def _decode(c, rows=None):
    """kvfx_decode (caller workspace, zero-filled) on rows of the case."""
    rows = list(range(len(c["lens"]))) if rows is None else rows
    t, ln = c["table"][rows], c["lens"][rows]
    q = c["q"].reshape(len(c["lens"]), -1)[rows].reshape(-1)
    batch, max_len, qh, hd = len(rows), int(ln.max()), c["qh"], c["hd"]
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c["desc"]), batch, qh, max_len, 0)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    td = torch.from_numpy(t.view(np.int64)).cuda()
    ld = torch.from_numpy(ln.view(np.int64)).cuda()
    qd = torch.from_numpy(q).cuda()
    out = torch.empty(batch * qh * hd, device="cuda")
    kv.check(kv.lib.kvfx_decode(ctypes.byref(c["desc"]), qd.data_ptr(), out.data_ptr(), td.data_ptr(), ld.data_ptr(),
                                batch, t.shape[1], qh, max_len, 0, ws.data_ptr(), ws.numel(), None), "kvfx_decode")
    torch.cuda.synchronize()
    return out.cpu().numpy(), (td, ld, qd, batch, t.shape[1], max_len)


def _noalloc(c, args):
    td, ld, qd, batch, width, max_len = args
    out = torch.full((batch * c["qh"] * c["hd"],), float("nan"), device="cuda")
    kv.check(kv.lib.kvfx_decode_noalloc(ctypes.byref(c["desc"]), qd.data_ptr(), out.data_ptr(), td.data_ptr(),
                                        ld.data_ptr(), batch, width, c["qh"], max_len, None), "kvfx_decode_noalloc")
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("dtype,hd,kvh,group,tol", [("bfloat16", 128, 8, 8, 2e-3), ("float16", 64, 4, 4, 2e-3),
                                                    ("float32", 32, 2, 2, 1e-5)])
def test_noalloc_decode_matches_workspace_decode(cuda, dtype, hd, kvh, group, tol):
    lens = [1, 17, 700, 4100, 9000, 33]
    c = _case(dtype, hd, kvh, group, lens, seed=hd + group)
    expected, args = _decode(c)
    ref = oracle.decode_batch(c["hk"], c["hv"], w.DTYPE_CODE[dtype], c["nb"], kvh, 16, hd, c["table"], c["lens"],
                              c["qh"], c["q"], threads=8)
    assert float(np.abs(expected - ref).max()) < tol
    for call in range(2):
        out = _noalloc(c, args)
        assert np.isfinite(out).all(), call
        assert float(np.abs(out - expected).max()) < tol, call
        assert float(np.abs(out - ref).max()) < tol, call
    assert kv.device_status(0) == 0


def test_noalloc_scratch_forces_longer_splits(cuda):
    """200 sequences x 8 KV heads of up to 9,000 tokens: the partials of the
    three splits per row kvfx_decode would choose do not fit the static
    array, so the no-allocation path takes two longer splits per row; its
    rows agree with kvfx_decode and, sampled, with the oracle. Calls of other
    shapes and of a cache with another head count run in between, on the
    same shared array."""
    kvh, hd, bs = 8, 128, 16
    lens = [int(x) for x in w.uniform_ints(0x5EE, 200, 16, 9000)]
    nb = int(sum((l + bs - 1) // bs for l in lens)) + 4
    cache_bytes = nb * kvh * bs * hd * 2
    # K then V, cache_bytes each (bf16 elements: cache_bytes in all)
    buf = torch.empty(cache_bytes, dtype=torch.bfloat16, device="cuda").normal_(generator=torch.Generator(
        device="cuda").manual_seed(5))
    base = buf.data_ptr()
    desc = kv.KvfxCache(base, base + cache_bytes, nb, kvh, bs, hd, kv.KVFX_BF16, 0, 0)
    width = max((l + bs - 1) // bs for l in lens)
    ids = w.permutation(77, np.arange(nb))
    table = np.full((len(lens), width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (l + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    big = dict(desc=desc, table=table, lens=np.array(lens, np.uint64), q=w.normal(78, len(lens) * kvh * hd), qh=kvh,
               hd=hd)
    small = _case("float16", 64, 4, 4, [1, 17, 700, 4100], seed=5)

    expected, args = _decode(big)
    # The default split of the longest row vs. what fits the 16 MiB array.
    default_pps = kv.lib.kvfx_decode_pages_per_split(ctypes.byref(desc), len(lens), kvh, max(lens), 0)
    pairs = len(lens) * kvh
    fit = (16 * 2**20 - 65536 * kvh * 2 - 256) // (pairs * 8 * (hd + 2) * 4)
    assert -(-width // default_pps) > fit >= 2, (default_pps, fit)

    sample = [0, 1, 100, 199, int(np.argmax(lens))]
    page = kvh * bs * hd * 2
    pids = np.unique(np.concatenate([table[r, :(lens[r] + bs - 1) // bs] for r in sample]))
    remap = {int(p): i for i, p in enumerate(pids)}
    hk = np.concatenate([d2h(base + int(p) * page, page) for p in pids])
    hv = np.concatenate([d2h(base + cache_bytes + int(p) * page, page) for p in pids])
    ctab = np.zeros((len(sample), width), np.uint64)
    for j, r in enumerate(sample):
        row = table[r, :(lens[r] + bs - 1) // bs]
        ctab[j, :len(row)] = [remap[int(p)] for p in row]
    qs = big["q"].reshape(len(lens), -1)[sample].reshape(-1)
    ref = oracle.decode_batch(hk, hv, 1, len(pids), kvh, bs, hd, ctab, big["lens"][sample], kvh, qs, threads=8)
    rows = np.concatenate([np.arange(r * kvh * hd, (r + 1) * kvh * hd) for r in sample])

    s_expected, s_args = _decode(small)
    for rnd in range(2):
        out = _noalloc(big, args)
        assert np.isfinite(out).all(), rnd
        assert float(np.abs(out - expected).max()) < 2e-3, rnd
        assert float(np.abs(out[rows] - ref).max()) < 2e-3, rnd
        # another cache (4 KV heads, other shapes) on the same array
        s_out = _noalloc(small, s_args)
        assert float(np.abs(s_out - s_expected).max()) < 2e-3, rnd
        # a different batch of the same cache
        part, p_args = _decode(big, rows=[5, 6, 7])
        assert float(np.abs(_noalloc(big, p_args) - part).max()) < 2e-3, rnd
    assert kv.device_status(0) == 0
    del buf


def test_noalloc_reports_out_of_range_pages(cuda):
    c = _case("bfloat16", 128, 2, 4, [40, 300], seed=9)
    c["table"][1, 3] = c["nb"] + 7  # beyond the cache: read as page 0 and flagged
    _, args = _decode(c)
    assert kv.device_status(0, clear=True) & kv.KVFX_FLAG_BAD_INDEX
    _noalloc(c, args)
    assert kv.device_status(0, clear=True) & kv.KVFX_FLAG_BAD_INDEX
    assert kv.device_status(0) == 0


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    # 65535 sequences x 64 KV heads: the counters and one split per sequence
    # need more than the static scratch, so the call is refused up front.
    desc = kv.KvfxCache(1 << 20, 1 << 21, 1 << 20, 64, 16, 128, kv.KVFX_BF16, 0, 0)
    rc = kv.lib.kvfx_decode_noalloc(ctypes.byref(desc), 16, 16, 16, 16, 65535, 1, 64, 16, None)
    assert rc == kv.KVFX_ENOSPACE
    assert b"16 MiB" in kv.lib.kvfx_last_error()

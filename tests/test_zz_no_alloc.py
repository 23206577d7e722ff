"""kvfx_decode_noalloc: batch decode for callers that cannot allocate device
memory (engines that give all device memory to their KV pool up front, loops
that cannot take cudaMalloc's implicit synchronisation, embedders whose
allocator policy forbids it). Its split-K scratch is a static device array
inside the library instead of a caller workspace.

Called through the C ABI twice in a row (the second call finds the previous
call's contents in the shared array) and compared with kvfx_decode, the
entry point with a caller workspace, within the tolerance of the decode tests
(2e-3 for bf16 caches, 1e-5 for FP32 caches). This file sorts last so that a
run stopping at the first failure has run every other test before it."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
from gpu_util import h2d
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
    h2d(base, w.encode(w.normal(seed, n), dtype).view(np.uint8))
    h2d(base + cache_bytes, w.encode(w.normal(seed + 1, n), dtype).view(np.uint8))
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
    q = torch.from_numpy(w.normal(seed + 3, len(lens) * qh * hd)).cuda()
    td = torch.from_numpy(table.view(np.int64)).cuda()
    ld = torch.from_numpy(np.array(lens, np.uint64).view(np.int64)).cuda()
    return buf, desc, td, ld, q, qh, width


@pytest.mark.parametrize("dtype,hd,kvh,group,tol", [("bfloat16", 128, 8, 8, 2e-3), ("float16", 64, 4, 4, 2e-3),
                                                    ("float32", 32, 2, 2, 1e-5)])
def test_noalloc_decode_matches_workspace_decode(cuda, dtype, hd, kvh, group, tol):
    lens = [1, 17, 700, 4100, 9000, 33]
    buf, desc, td, ld, q, qh, width = _case(dtype, hd, kvh, group, lens, seed=hd + group)
    batch, max_len = len(lens), max(lens)
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(desc), batch, qh, max_len, 0)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    expected = torch.empty(batch * qh * hd, device="cuda")
    kv.check(kv.lib.kvfx_decode(ctypes.byref(desc), q.data_ptr(), expected.data_ptr(), td.data_ptr(),
                                ld.data_ptr(), batch, width, qh, max_len, 0, ws.data_ptr(), ws.numel(), None),
             "kvfx_decode")
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full((batch * qh * hd,), float("nan"), device="cuda")
        kv.check(kv.lib.kvfx_decode_noalloc(ctypes.byref(desc), q.data_ptr(), out.data_ptr(), td.data_ptr(),
                                            ld.data_ptr(), batch, width, qh, max_len, None),
                 "kvfx_decode_noalloc")
        torch.cuda.synchronize()
        err = float((out - expected).abs().max())
        assert torch.isfinite(out).all(), call
        assert err < tol, (call, err)
    del buf


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    # 65535 sequences x 64 KV heads: the counters and one split per sequence
    # need more than the static scratch, so the call is refused up front.
    desc = kv.KvfxCache(1 << 20, 1 << 21, 1 << 20, 64, 16, 128, kv.KVFX_BF16, 0, 0)
    rc = kv.lib.kvfx_decode_noalloc(ctypes.byref(desc), 16, 16, 16, 16, 65535, 1, 64, 16, None)
    assert rc == kv.KVFX_ENOSPACE
    assert b"16 MiB" in kv.lib.kvfx_last_error()

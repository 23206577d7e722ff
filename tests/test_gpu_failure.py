"""Device-side failure detection without a GPU fault: the bounded barrier
waits of the TMA/tensor-core kernels, run on a barrier that nothing completes
(kvfx_selftest_wait_timeout), give up after their limit, report
KVFX_FLAG_TIMEOUT and return; the context keeps working afterwards (a decode
launched next matches the oracle). Host-side failure paths (bad slots,
duplicates, wrong-device and host pointers, pool exhaustion, a throwing
copier) are covered with the API tests."""
import time

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda):
    kv.device_status(0, clear=True)
    t = time.perf_counter()
    rc = kv.lib.kvfx_selftest_wait_timeout(0)
    secs = time.perf_counter() - t
    assert rc == kv.KVFX_ETIMEOUT, kv.lib.kvfx_last_error().decode()
    assert b"gave up" in kv.lib.kvfx_last_error()
    assert 1.5 < secs < 30.0, secs          # the 2 s limit, both waits in parallel
    assert kv.device_status(0) == 0         # the self-test leaves the status word as it was
    assert kv.lib.kvfx_selftest_wait_timeout(-1) == kv.KVFX_EINVAL

    # The context is usable: a small decode right after matches the oracle.
    lens = [33, 70]
    batch = w.decode_batch_on_pool(32, 16, lens, seed=3)
    st = kv.PagedKVStorage(batch.pool, 2, 128, kv.DType.BFloat16, 0)
    total = sum(lens)
    k = w.encode(w.normal(1, total * 2 * 128), "bfloat16")
    v = w.encode(w.normal(2, total * 2 * 128), "bfloat16")
    writes = [(s, p) for s in batch.sequences for p in range(s.num_tokens())]
    kv.write_paged_kv(st, torch.from_numpy(k.view(np.int16)).cuda(), torch.from_numpy(v.view(np.int16)).cuda(),
                      kv.build_slot_mapping(writes))
    q = w.normal(3, 2 * 8 * 128)
    o = torch.empty(2 * 8 * 128, device="cuda")
    kv.paged_attention_batch(st, batch.sequences, torch.from_numpy(q).cuda(), o, 8)
    kf, vf = w.decode(k, "bfloat16"), w.decode(v, "bfloat16")
    got = o.cpu().numpy()
    off = 0
    for r, L in enumerate(lens):
        rows = slice(off * 256, (off + L) * 256)
        exp = oracle.reference_attention(q[r * 1024:(r + 1) * 1024], kf[rows], vf[rows], (1, L, 8, 2, 128))
        assert float(np.abs(got[r * 1024:(r + 1) * 1024] - exp).max()) < 2e-3
        off += L

"""paged_attention_batch_host: batch decode with Q and O in page-locked host
memory. Its output is bit-identical to paged_attention_batch on device
buffers (same kernels, same split size, same row chunks) and within
max_abs_err 2e-3 (BF16/FP16 caches) / 1e-5 (FP32) of the FP64 oracle; batches
of 16 rows and more take the two-chunk path (Q uploaded per chunk, O written
by the kernels through the host buffer's device mapping). Pageable host
memory and device memory are refused."""
import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 2e-3}


def _case(dtype, kvh, hd, lens, seed):
    bs = 16
    batch = w.decode_batch_on_pool(sum((l + bs - 1) // bs for l in lens) + 16, bs, lens, seed=seed)
    st = kv.PagedKVStorage(batch.pool, kvh, hd, w.DTYPES[dtype], 0)
    total = sum(lens)
    k_host = w.encode(w.normal(seed + 1, total * kvh * hd), dtype)
    v_host = w.encode(w.normal(seed + 2, total * kvh * hd), dtype)
    view = np.int16 if dtype != "float32" else np.float32
    writes = [(s, t) for s in batch.sequences for t in range(s.num_tokens())]
    kv.write_paged_kv(st, torch.from_numpy(k_host.view(view)).cuda(), torch.from_numpy(v_host.view(view)).cuda(),
                      kv.build_slot_mapping(writes))
    return batch, st, k_host, v_host


@pytest.mark.parametrize("dtype,kvh,group,hd,nrows", [
    ("bfloat16", 8, 4, 128, 40),     # fast kernel, two chunks
    ("float16", 2, 8, 64, 5),        # fast kernel, one chunk
    ("float32", 2, 2, 32, 17),       # generic kernel, two chunks
])
def test_host_buffers_bit_identical_to_device_buffers(cuda, dtype, kvh, group, hd, nrows):
    lens = [int(x) for x in w.uniform_ints(7 + nrows, nrows, 1, 3000)]
    batch, st, k_host, v_host = _case(dtype, kvh, hd, lens, seed=11 + hd)
    qh = kvh * group
    q = w.normal(99, nrows * qh * hd)
    q_pin = torch.from_numpy(q).pin_memory()
    o_pin = torch.full((nrows * qh * hd,), 7.0).pin_memory()
    kv.paged_attention_batch_host(st, batch.sequences, q_pin, o_pin, qh)
    o_dev = torch.empty(nrows * qh * hd, device="cuda")
    kv.paged_attention_batch(st, batch.sequences, q_pin.cuda(), o_dev, qh)
    got = o_pin.numpy()
    assert np.array_equal(got.view(np.uint32), o_dev.cpu().numpy().view(np.uint32))
    kf, vf = w.decode(k_host, dtype), w.decode(v_host, dtype)
    off = 0
    for r, L in enumerate(lens):
        rows = slice(off * kvh * hd, (off + L) * kvh * hd)
        exp = oracle.reference_attention(q[r * qh * hd:(r + 1) * qh * hd], kf[rows], vf[rows], (1, L, qh, kvh, hd))
        err = float(np.abs(got[r * qh * hd:(r + 1) * qh * hd] - exp).max())
        assert err < TOL[dtype], (r, err)
        off += L


def test_host_buffers_must_be_page_locked(cuda):
    batch, st, _, _ = _case("bfloat16", 2, 128, [20, 40], seed=5)
    n = 2 * 8 * 128
    pinned = torch.zeros(n).pin_memory()
    with pytest.raises(ValueError):
        kv.paged_attention_batch_host(st, batch.sequences, np.zeros(n, np.float32), pinned, 8)  # pageable Q
    with pytest.raises(ValueError):
        kv.paged_attention_batch_host(st, batch.sequences, pinned, torch.zeros(n, device="cuda"), 8)  # device O
    with pytest.raises(ValueError):
        kv.paged_attention_batch_host(st, batch.sequences, pinned, pinned, 8)  # overlap
    kv.paged_attention_batch_host(st, [], None, None, 8)  # empty batch returns first

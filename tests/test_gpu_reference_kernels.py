"""This build's batch decode against the reference's own GPU implementation:
KVFlux's CUDA write and paged_attention_batch kernels (compiled from its
sources for sm_100a into oracle/_ref/libkvflux_ref_gpu.so) run through its
public API on the same B200, on the same page ids (the same free-list order)
and the same inputs. Outputs agree within max_abs_err 2e-3 (BF16 caches) /
1e-5 (FP32 caches); both are checked against the FP64 oracle as well.
Skipped when the reference library was not built."""
import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 2e-3}


@pytest.fixture(scope="module", autouse=True)
def need_reference():
    if oracle.ref_gpu() is None:
        pytest.skip("reference GPU library not built")


@pytest.mark.parametrize("dtype,kvh,group,hd", [("bfloat16", 2, 4, 128), ("float32", 2, 2, 64),
                                                ("float16", 1, 8, 32)])
def test_decode_matches_reference_gpu_kernels(cuda, dtype, kvh, group, hd):
    bs, qh = 16, kvh * group
    lens = [1, 17, 300, 1000, 33]
    nb = sum((l + bs - 1) // bs for l in lens) + 16
    order = w.permutation(hd + kvh, np.arange(nb))
    total = sum(lens)
    k = w.encode(w.normal(11, total * kvh * hd), dtype)
    v = w.encode(w.normal(12, total * kvh * hd), dtype)
    q = w.normal(13, len(lens) * qh * hd)

    o_ref, _, _ = oracle.ref_gpu_decode(0, nb, bs, order, kvh, qh, hd, w.DTYPE_CODE[dtype], lens, k, v, q, reps=1)

    pool = kv.PhysicalBlockPool(nb, bs)
    held = w.fragment_pool(pool, order)
    assert not held
    st = kv.PagedKVStorage(pool, kvh, hd, w.DTYPES[dtype], 0)
    seqs = []
    for L in lens:
        s = kv.SequenceState(len(seqs) + 1, pool)
        s.append_tokens(L)
        seqs.append(s)
    view = np.int16 if dtype != "float32" else np.float32
    kv.write_paged_kv(st, torch.from_numpy(k.view(view)).cuda(), torch.from_numpy(v.view(view)).cuda(),
                      kv.build_slot_mapping([(s, t) for s in seqs for t in range(s.num_tokens())]))
    o = torch.empty(len(lens) * qh * hd, device="cuda")
    kv.paged_attention_batch(st, seqs, torch.from_numpy(q).cuda(), o, qh)
    got = o.cpu().numpy()

    assert np.isfinite(o_ref).all()
    assert float(np.abs(got - o_ref).max()) < TOL[dtype]
    kf, vf = w.decode(k, dtype), w.decode(v, dtype)
    off = 0
    for r, L in enumerate(lens):
        rows = slice(off * kvh * hd, (off + L) * kvh * hd)
        exp = oracle.reference_attention(q[r * qh * hd:(r + 1) * qh * hd], kf[rows], vf[rows], (1, L, qh, kvh, hd))
        assert float(np.abs(o_ref[r * qh * hd:(r + 1) * qh * hd] - exp).max()) < TOL[dtype]  # the reference itself
        off += L

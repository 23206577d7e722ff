"""kvfx_attention_batch: causal attention over several sequences of one cache
in one call. Every sequence's output is bit-identical to kvfx_attention on
that sequence alone (the tensor-core shapes share one persistent launch whose
units do the same arithmetic in the same order; the other shapes run the
single-sequence path), and within max_abs_err 2e-3 (BF16/FP16) / 1e-5 (FP32)
of the FP64 oracle on the last rows of each sequence. Ragged batches mix
lengths whose query tiles run out at different unit rounds, single-query
sequences (batch-decode kernel), empty ones (skipped) and FP32 caches
(generic kernel). The C++ API over it, paged_attention_prefill_batch, is
bit-identical to one paged_attention per sequence (also past one launch's
KVFX_MAX_PREFILL_SEQS sequences) and raises the reference's exception types
for bad shapes, foreign pools and overlapping buffers."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w
from test_gpu_capi import _decode_case, call, u64

pytestmark = pytest.mark.gpu

TOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 2e-3}


@pytest.fixture(autouse=True)
def clear_status(cuda):
    kv.device_status(0, clear=True)
    yield


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _u64s(xs):
    return (ctypes.c_uint64 * len(xs))(*[int(x) for x in xs])


def _run_batch(c, table, qs, outs, lq, lens, qh, ws=None):
    width = table.shape[1]
    td = u64(table)
    wsp, wsb = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    rc = kv.lib.kvfx_attention_batch(ctypes.byref(c.desc), len(qs), _ptrs(qs), _ptrs(outs), td.data_ptr(), width,
                                     _u64s(lq), _u64s(lens), qh, wsp, wsb, None)
    torch.cuda.synchronize()
    kv.check(rc, "kvfx_attention_batch")


@pytest.mark.parametrize("dtype,kvh,group,lq,lens", [
    # config-4-like ragged prefill: whole sequences, query tiles end at different rounds
    ("bfloat16", 8, 4, [700, 128, 1, 333, 64], [700, 128, 9, 333, 64]),
    # suffix-aligned chunks, an empty sequence, a 2-query one
    ("float16", 2, 3, [100, 0, 2, 257], [517, 40, 2, 300]),
    # one sequence (the single-call path through the batch entry point)
    ("bfloat16", 1, 8, [129], [129]),
    # FP32 cache: every sequence on the generic kernel
    ("float32", 2, 2, [33, 5, 64], [70, 5, 64]),
])
def test_batch_bit_identical_to_single_calls(dtype, kvh, group, lq, lens):
    hd = 128 if dtype != "float32" else 64
    c, table, _, _, qh = _decode_case(dtype, hd, 16, kvh, group, lens, seed=sum(lens) + group)
    qs, outs, singles = [], [], []
    for i, (a, L) in enumerate(zip(lq, lens)):
        q = w.normal(31 + i, max(a, 1) * qh * hd)
        qs.append(torch.from_numpy(q).cuda())
        outs.append(torch.full((max(a, 1) * qh * hd,), 777.0, device="cuda"))
        singles.append(torch.full_like(outs[-1], 555.0))
    need = max(kv.lib.kvfx_attention_workspace_bytes(ctypes.byref(c.desc), a, L, qh) for a, L in zip(lq, lens))
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    _run_batch(c, table, qs, outs, lq, lens, qh, ws)
    for i, (a, L) in enumerate(zip(lq, lens)):
        if a == 0:
            assert (outs[i].cpu().numpy() == 777.0).all(), "empty sequence written"
            continue
        call(kv.lib.kvfx_attention, ctypes.byref(c.desc), qs[i].data_ptr(), singles[i].data_ptr(),
             u64(table[i]), a, L, qh, ws.data_ptr(), ws.numel(), None)
        got = outs[i].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), singles[i].cpu().numpy().view(np.uint32)), f"sequence {i}"
        lo = max(0, a - 40)
        exp = oracle.attention_rows(c.host_k, c.host_v, w.DTYPE_CODE[dtype], c.nb, kvh, 16, hd, table[i], a, L, qh,
                                    qs[i].cpu().numpy(), row_begin=lo, row_end=a, threads=8).reshape(a, -1)
        err = float(np.abs(got.reshape(a, -1)[lo:a] - exp[lo:a]).max())
        assert err < TOL[dtype], (i, err)
    assert kv.device_status(0) == 0


def test_batch_of_max_sequences():
    """KVFX_MAX_PREFILL_SEQS short sequences in one launch (more sequences x
    heads than SMs): each bit-identical to its single call."""
    n = kv.KVFX_MAX_PREFILL_SEQS
    lens = [int(x) for x in w.uniform_ints(5, n, 2, 300)]
    c, table, _, _, qh = _decode_case("bfloat16", 128, 16, 2, 4, lens, seed=321)
    qs = [torch.from_numpy(w.normal(400 + i, L * qh * 128)).cuda() for i, L in enumerate(lens)]
    outs = [torch.empty(L * qh * 128, device="cuda") for L in lens]
    _run_batch(c, table, qs, outs, lens, lens, qh)
    for i, L in enumerate(lens):
        one = torch.empty_like(outs[i])
        call(kv.lib.kvfx_attention, ctypes.byref(c.desc), qs[i].data_ptr(), one.data_ptr(), u64(table[i]), L, L, qh,
             None, 0, None)
        assert torch.equal(outs[i].view(torch.int32), one.view(torch.int32)), f"sequence {i}"
    assert kv.device_status(0) == 0


def test_batch_argument_errors():
    c, table, _, _, qh = _decode_case("bfloat16", 128, 16, 2, 4, [40, 20], seed=9)
    q = torch.zeros(40 * qh * 128, device="cuda")
    o = torch.zeros_like(q)
    td = u64(table)
    f = kv.lib.kvfx_attention_batch
    d = ctypes.byref(c.desc)
    qq, oo = _ptrs([q, q]), _ptrs([o, o])
    n = kv.KVFX_MAX_PREFILL_SEQS + 1
    assert f(d, n, _ptrs([q] * n), _ptrs([o] * n), td.data_ptr(), 3, _u64s([2] * n), _u64s([2] * n), qh,
             None, 0, None) == kv.KVFX_EINVAL                                                  # too many sequences
    assert f(d, 2, qq, oo, td.data_ptr(), 3, _u64s([41, 2]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_EINVAL
    assert f(d, 2, qq, oo, td.data_ptr(), 2, _u64s([4, 2]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_EINVAL
    assert f(d, 2, qq, oo, None, 3, _u64s([4, 2]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_EINVAL
    assert f(d, 2, None, oo, td.data_ptr(), 3, _u64s([4, 2]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_EINVAL
    assert f(d, 2, qq, oo, td.data_ptr(), 3, _u64s([4, 2]), _u64s([40, 20]), 3, None, 0, None) == kv.KVFX_EINVAL
    # a single-query sequence needs the decode workspace
    assert f(d, 2, qq, oo, td.data_ptr(), 3, _u64s([4, 1]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_ENOSPACE
    assert f(d, 0, None, None, None, 0, None, None, qh, None, 0, None) == kv.KVFX_OK            # nothing to do
    assert f(d, 2, qq, oo, None, 0, _u64s([0, 0]), _u64s([40, 20]), qh, None, 0, None) == kv.KVFX_OK
    torch.cuda.synchronize()
    assert kv.device_status(0) == 0


# -------------------------------------------------------------- C++ API ---

def _storage_case(dtype, kvh, hd, lens, seed):
    bs = 16
    batch = w.decode_batch_on_pool(sum((l + bs - 1) // bs for l in lens) + 8, bs, lens, seed=seed)
    st = kv.PagedKVStorage(batch.pool, kvh, hd, w.DTYPES[dtype], 0)
    total = sum(lens)
    view = np.int16 if dtype != "float32" else np.float32
    k = w.encode(w.normal(seed + 1, total * kvh * hd), dtype).view(view)
    v = w.encode(w.normal(seed + 2, total * kvh * hd), dtype).view(view)
    writes = [(s, t) for s in batch.sequences for t in range(s.num_tokens())]
    kv.write_paged_kv(st, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), kv.build_slot_mapping(writes))
    return batch, st


@pytest.mark.parametrize("dtype,kvh,group,hd,lens,lq", [
    ("bfloat16", 2, 4, 128, [300, 77, 129, 40], [300, 0, 64, 1]),
    ("float32", 2, 2, 64, [50, 33], [50, 7]),
])
def test_api_prefill_batch_bit_identical_to_paged_attention(dtype, kvh, group, hd, lens, lq):
    batch, st = _storage_case(dtype, kvh, hd, lens, seed=sum(lens))
    qh = kvh * group
    qs = [torch.from_numpy(w.normal(60 + i, max(a, 1) * qh * hd)).cuda() for i, a in enumerate(lq)]
    outs = [torch.full((max(a, 1) * qh * hd,), 3.0, device="cuda") for a in lq]
    kv.paged_attention_prefill_batch(st, batch.sequences, qs, outs, lq, qh)
    for i, a in enumerate(lq):
        if a == 0:
            assert (outs[i].cpu().numpy() == 3.0).all(), "sequence without queries written"
            continue
        one = torch.empty_like(outs[i])
        kv.paged_attention(st, batch.sequences[i], qs[i], one, a, qh)
        assert torch.equal(outs[i].view(torch.int32), one.view(torch.int32)), f"sequence {i}"
    assert kv.device_status(0) == 0


def test_api_prefill_batch_more_sequences_than_one_launch():
    n = kv.KVFX_MAX_PREFILL_SEQS + 8
    lens = [int(x) for x in w.uniform_ints(17, n, 2, 200)]
    batch, st = _storage_case("float16", 1, 128, lens, seed=77)
    qh = 4
    qs = [torch.from_numpy(w.normal(500 + i, L * qh * 128)).cuda() for i, L in enumerate(lens)]
    outs = [torch.empty(L * qh * 128, device="cuda") for L in lens]
    kv.paged_attention_prefill_batch(st, batch.sequences, qs, outs, lens, qh)
    for i, L in enumerate(lens):
        one = torch.empty_like(outs[i])
        kv.paged_attention(st, batch.sequences[i], qs[i], one, L, qh)
        assert torch.equal(outs[i].view(torch.int32), one.view(torch.int32)), f"sequence {i}"


def test_api_prefill_batch_errors():
    batch, st = _storage_case("bfloat16", 2, 128, [40, 30], seed=3)
    other = kv.PhysicalBlockPool(8, 16)
    foreign = kv.SequenceState(9, other)
    foreign.append_tokens(5)
    qh = 8
    q = torch.zeros(40 * qh * 128, device="cuda")
    o = torch.zeros_like(q)
    o2 = torch.zeros_like(q)
    seqs = batch.sequences
    with pytest.raises(ValueError):   # array lengths differ
        kv.paged_attention_prefill_batch(st, seqs, [q], [o, o2], [4, 4], qh)
    with pytest.raises(ValueError):   # more queries than tokens
        kv.paged_attention_prefill_batch(st, seqs, [q, q], [o, o2], [41, 4], qh)
    with pytest.raises(ValueError):   # sequence of another pool
        kv.paged_attention_prefill_batch(st, [seqs[0], foreign], [q, q], [o, o2], [4, 4], qh)
    with pytest.raises(ValueError):   # two outputs overlap
        kv.paged_attention_prefill_batch(st, seqs, [q, q], [o, o], [4, 4], qh)
    with pytest.raises(ValueError):   # an output overlaps another sequence's Q
        kv.paged_attention_prefill_batch(st, seqs, [q, o2], [o2, o], [4, 4], qh)
    with pytest.raises(ValueError):   # head count not a multiple of the KV heads
        kv.paged_attention_prefill_batch(st, seqs, [q, q], [o, o2], [4, 4], 3)
    kv.paged_attention_prefill_batch(st, seqs, [None, None], [None, None], [0, 0], qh)  # nothing to do
    kv.paged_attention_prefill_batch(st, [], [], [], [], qh)
    torch.cuda.synchronize()
    assert kv.device_status(0) == 0

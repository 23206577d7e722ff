"""The fused decode step: kvfx_decode_append (C ABI) and BatchDecodeSession
(C++ API, device-resident block table).

Checked against the CPU oracle and against the unfused path on the same
inputs: the cache after the step is byte-exact with the oracle's write of the
new rows; the device table holds each new token's page at its column; the
attention output is within max_abs_err 1e-5 (FP32 caches) / 2e-3 (FP16/BF16)
of the FP64 reference and bit-identical to kvfx_decode run afterwards on the
updated cache and table. Cases: new pages (a row whose last page was full),
in-page appends, a copy-on-written last page (the slot names a page other
than the table's), fast-kernel and generic shapes, and slots at the wrong
offset (flagged, not written)."""
import ctypes

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from gpu_util import d2h, h2d
from kvflux_b200 import workloads as w
from test_gpu_capi import TOL, Cache, _page_order, call, u64

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def clear_status(cuda):
    kv.device_status(0, clear=True)
    yield


def _append_case(dtype, hd, bs, kvh, group, lens, seed, cow_rows=()):
    """A cache holding `lens` tokens per row, plus each row's new token: its
    slot (a fresh page when the last page is full, or for `cow_rows` a fresh
    copy of the partial last page), K/V rows and Q."""
    batch = len(lens)
    spare = batch + len(cow_rows) + 8
    c = Cache(int(sum((l + bs - 1) // bs for l in lens)) + spare, kvh, bs, hd, dtype, seed=seed)
    ids = [int(x) for x in _page_order("perm", c.nb, seed + 3)]
    width = max(l // bs + 1 for l in lens) + 2
    table = np.full((batch, width), 2**64 - 1, np.uint64)
    k = 0
    for r, l in enumerate(lens):
        p = (l + bs - 1) // bs
        table[r, :p] = ids[k:k + p]
        k += p
    free = ids[k:]
    slots = np.zeros(batch, np.uint64)
    for r, l in enumerate(lens):
        off = l % bs
        if off == 0:
            page = free.pop(0)
        elif r in cow_rows:
            # The step's page is a private copy of the shared last page.
            old, page = int(table[r, l // bs]), free.pop(0)
            for cache in (c.host_k, c.host_v):
                cache[page * c.page:(page + 1) * c.page] = cache[old * c.page:(old + 1) * c.page]
        else:
            page = int(table[r, l // bs])
        slots[r] = page * bs + off
    h2d(c.base, c.host_k)
    h2d(c.base + c.cache_bytes, c.host_v)
    n = batch * kvh * hd
    kn = w.encode(w.normal(seed + 5, n), dtype).view(np.uint8)
    vn = w.encode(w.normal(seed + 6, n), dtype).view(np.uint8)
    q = w.normal(seed + 9, batch * kvh * group * hd)
    return c, table, slots, kn, vn, q


def _expected(c, table, lens, slots, kn, vn):
    """Cache bytes and table after the step, by the oracle's write."""
    hk, hv = c.host_k.copy(), c.host_v.copy()
    oracle.write(hk, hv, c.nb, c.h, c.bs, c.row, kn, vn, slots)
    t = table.copy()
    for r, l in enumerate(lens):
        t[r, l // c.bs] = int(slots[r]) // c.bs
    return hk, hv, t


@pytest.mark.parametrize("dtype,hd,bs,kvh,group", [
    ("bfloat16", 128, 16, 8, 4),   # fast kernel, Llama-3-8B heads
    ("float16", 64, 16, 2, 8),     # fast kernel, group 8
    ("bfloat16", 128, 16, 1, 8),   # fast kernel, one KV head
    ("float32", 32, 16, 2, 2),     # generic path
    ("bfloat16", 64, 8, 2, 4),     # generic path (block 8)
])
def test_decode_append_matches_oracle_and_unfused(dtype, hd, bs, kvh, group):
    lens = [16, 1, 15, 17, 31, 32, 100, 511, 512, 2047, 2048, 3000]
    c, table, slots, kn, vn, q = _append_case(dtype, hd, bs, kvh, group, lens, seed=hd + 7 * group,
                                              cow_rows=(4, 7, 11))
    batch, qh = len(lens), kvh * group
    new_lens = np.array(lens, np.uint64) + 1
    max_len = int(new_lens.max())
    hk, hv, t_exp = _expected(c, table, lens, slots, kn, vn)

    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), batch, qh, max_len, 0)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    td = u64(table)
    qd = torch.from_numpy(q).cuda()
    out = torch.full((batch * qh * hd + 1,), 12345.0, device="cuda")
    dk, dv = torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda()
    call(kv.lib.kvfx_decode_append, ctypes.byref(c.desc), dk.data_ptr(), dv.data_ptr(), u64(slots), qd.data_ptr(),
         out.data_ptr(), td, u64(new_lens), batch, table.shape[1], qh, max_len, 0, ws.data_ptr(), ws.numel(), None)
    assert kv.device_status(0) == 0

    got_k, got_v = c.device_bytes()
    assert np.array_equal(got_k, hk) and np.array_equal(got_v, hv), "cache differs from the oracle's write"
    assert np.array_equal(td.cpu().numpy().view(np.uint64), t_exp), "device table not updated as expected"

    got = out.cpu().numpy()
    assert got[-1] == 12345.0
    exp = oracle.decode_batch(hk, hv, w.DTYPE_CODE[dtype], c.nb, kvh, bs, hd, t_exp, new_lens, qh, q, threads=8)
    assert np.isfinite(got[:-1]).all()
    err = float(np.abs(got[:-1] - exp).max())
    assert err < TOL[dtype], err

    # The unfused path over the updated cache and table gives the same bits.
    out2 = torch.empty_like(out)
    call(kv.lib.kvfx_decode, ctypes.byref(c.desc), qd.data_ptr(), out2.data_ptr(), td, u64(new_lens), batch,
         table.shape[1], qh, max_len, 0, ws.data_ptr(), ws.numel(), None)
    assert np.array_equal(out2.cpu().numpy()[:-1].view(np.uint32), got[:-1].view(np.uint32))


@pytest.mark.parametrize("dtype,hd,bs", [("bfloat16", 128, 16), ("float32", 32, 4)])
def test_decode_append_wrong_offset_is_flagged_not_written(dtype, hd, bs):
    lens = [40, 7]
    c, table, slots, kn, vn, q = _append_case(dtype, hd, bs, 2, 4, lens, seed=3)
    bad = slots.copy()
    bad[0] = (int(slots[0]) // bs) * bs + (int(slots[0]) + 1) % bs  # right page, wrong offset
    before_k, before_v = c.device_bytes()
    new_lens = np.array(lens, np.uint64) + 1
    ws_bytes = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), 2, 8, 41, 0)
    ws = torch.zeros(max(int(ws_bytes), 16), dtype=torch.uint8, device="cuda")
    td = u64(table)
    out = torch.empty(2 * 8 * hd, device="cuda")
    dk, dv = torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda()
    call(kv.lib.kvfx_decode_append, ctypes.byref(c.desc), dk.data_ptr(), dv.data_ptr(), u64(bad),
         torch.from_numpy(q).cuda().data_ptr(), out.data_ptr(), td, u64(new_lens), 2, table.shape[1], 8, 41, 0,
         ws.data_ptr(), ws.numel(), None)
    assert kv.device_status(0) & kv.KVFX_FLAG_BAD_INDEX
    after_k, after_v = c.device_bytes()
    # Row 0's bad slot wrote nothing; row 1's good slot was written.
    hk, hv = before_k.copy(), before_v.copy()
    oracle.write(hk, hv, c.nb, c.h, c.bs, c.row, kn[c.h * c.row:], vn[c.h * c.row:], slots[1:])
    assert np.array_equal(after_k, hk) and np.array_equal(after_v, hv)


def test_decode_append_argument_errors():
    c = Cache(8, 2, 16, 128, "bfloat16", seed=1)
    x = torch.zeros(64, dtype=torch.int64, device="cuda")
    p = x.data_ptr()
    f = kv.lib.kvfx_decode_append
    assert f(ctypes.byref(c.desc), p, p, p, p, p, p, p, 1, 4, 7, 16, 0, p, 512, None) == kv.KVFX_EINVAL  # 7 % 2
    assert f(ctypes.byref(c.desc), None, p, p, p, p, p, p, 1, 4, 8, 16, 0, p, 512, None) == kv.KVFX_EINVAL
    assert f(ctypes.byref(c.desc), p, p, p, p, p, p, p, 1, 1, 8, 17, 0, p, 512, None) == kv.KVFX_EINVAL  # table
    assert f(ctypes.byref(c.desc), p, p, p, p, p, p, p, 0, 1, 8, 17, 0, None, 0, None) == kv.KVFX_OK  # empty
    need = kv.lib.kvfx_decode_workspace_bytes(ctypes.byref(c.desc), 1, 8, 1000, 4)
    assert f(ctypes.byref(c.desc), p, p, p, p, p, p, p, 1, 63, 8, 1000, 4, p, need - 1, None) == kv.KVFX_ENOSPACE


# ------------------------------------------------------------ C++ session ---

class _Twin:
    """Sequences on a fragmented pool with a host record of every token's K/V
    rows, so any sequence's contents can be recomputed after forks and
    copy-on-write."""

    def __init__(self, dtype, kvh, hd, bs, capacity, seed):
        self.dtype, self.kvh, self.hd, self.bs = dtype, kvh, hd, bs
        self.pool = kv.PhysicalBlockPool(capacity, bs)
        held = [self.pool.allocate() for _ in range(capacity)]
        for i in w.permutation(seed, np.arange(capacity))[::-1]:
            self.pool.free(held[int(i)])
        self.storage = kv.PagedKVStorage(self.pool, kvh, hd, w.DTYPES[dtype], 0)
        self.rows = {}  # id(seq) -> list of (k_row, v_row) raw bytes per token
        self.seed = seed

    def rand_rows(self, n):
        self.seed += 2
        k = w.encode(w.normal(self.seed, n * self.kvh * self.hd), self.dtype).view(np.uint8)
        v = w.encode(w.normal(self.seed + 1, n * self.kvh * self.hd), self.dtype).view(np.uint8)
        return k, v

    def prefill(self, seq, n):
        pos = seq.num_tokens()
        seq.append_tokens(n)
        k, v = self.rand_rows(n)
        kv.write_paged_kv(self.storage, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                          kv.build_slot_mapping([(seq, pos + t) for t in range(n)]))
        rb = self.kvh * self.hd * w.ELEM_BYTES[self.dtype]
        self.rows.setdefault(id(seq), []).extend((k[t * rb:(t + 1) * rb], v[t * rb:(t + 1) * rb]) for t in range(n))

    def fork(self, seq, rid):
        child = seq.fork_shared(rid)
        self.rows[id(child)] = list(self.rows[id(seq)])
        return child

    def expected_out(self, seqs, q, qh):
        out = []
        for r, s in enumerate(seqs):
            rows = self.rows[id(s)]
            kf = w.decode(np.concatenate([a for a, _ in rows]).view(np.uint16 if self.dtype != "float32"
                                                                     else np.uint32), self.dtype)
            vf = w.decode(np.concatenate([b for _, b in rows]).view(np.uint16 if self.dtype != "float32"
                                                                    else np.uint32), self.dtype)
            L = len(rows)
            out.append(oracle.reference_attention(q[r * qh * self.hd:(r + 1) * qh * self.hd], kf, vf,
                                                  (1, L, qh, self.kvh, self.hd)))
        return np.concatenate(out)


@pytest.mark.parametrize("dtype,hd,bs,kvh,group", [("bfloat16", 128, 16, 2, 4), ("float32", 16, 4, 2, 2)])
def test_batch_decode_session_steps_with_forks(dtype, hd, bs, kvh, group):
    t = _Twin(dtype, kvh, hd, bs, capacity=2048, seed=17)
    qh = kvh * group
    a = kv.SequenceState(1, t.pool)
    t.prefill(a, 3 * bs + bs // 2)          # partial last page, shared after the forks below
    b = t.fork(a, 2)
    c = t.fork(a, 3)
    d = kv.SequenceState(4, t.pool)
    t.prefill(d, 5 * bs)                     # full last page: the first step opens a new page
    e = kv.SequenceState(5, t.pool)
    t.prefill(e, 1)
    seqs = [a, b, c, d, e]
    sess = kv.BatchDecodeSession(t.storage, seqs, qh)
    batch = len(seqs)
    steps = bs + 3                           # crosses a page boundary in every row
    for step in range(steps):
        k, v = t.rand_rows(batch)
        q = w.normal(1000 + step, batch * qh * hd)
        o = torch.full((batch * qh * hd,), 7.0, device="cuda")
        locs = sess.step(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(q).cuda(), o)
        rb = kvh * hd * w.ELEM_BYTES[dtype]
        for r, s in enumerate(seqs):
            t.rows[id(s)].append((k[r * rb:(r + 1) * rb], v[r * rb:(r + 1) * rb]))
            loc = s.token_location(s.num_tokens() - 1)
            assert (locs[r].physical_block, locs[r].offset_in_block) == (loc.physical_block, loc.offset_in_block)
        got = o.cpu().numpy()
        exp = t.expected_out(seqs, q, qh)
        err = float(np.abs(got - exp).max())
        assert err < TOL[dtype], (step, err)
    # The shared prefix pages stayed shared; the copied tails are private.
    assert a.physical_block_id(0) == b.physical_block_id(0) == c.physical_block_id(0)
    assert len({a.physical_block_id(3), b.physical_block_id(3), c.physical_block_id(3)}) == 3
    # Device table rows equal the sequences' tables.
    tab = d2h(sess.device_table(), batch * sess.table_width() * 8).view(np.uint64).reshape(batch, -1)
    for r, s in enumerate(seqs):
        n = s.num_allocated_blocks()
        assert [int(x) for x in tab[r, :n]] == [s.physical_block_id(j) for j in range(n)]


def test_batch_decode_session_refresh_after_outside_growth():
    t = _Twin("bfloat16", 2, 128, 16, capacity=4096, seed=29)
    a, b = kv.SequenceState(1, t.pool), kv.SequenceState(2, t.pool)
    t.prefill(a, 20)
    t.prefill(b, 33)
    sess = kv.BatchDecodeSession(t.storage, [a, b], 8)
    width = sess.table_width()
    t.prefill(b, 16 * (width + 3))           # grows past the device table outside the session
    sess.refresh(1)
    assert sess.table_width() > width
    k, v = t.rand_rows(2)
    q = w.normal(5, 2 * 8 * 128)
    o = torch.empty(2 * 8 * 128, device="cuda")
    sess.step(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(q).cuda(), o)
    rb = 2 * 128 * 2
    for r, s in enumerate([a, b]):
        t.rows[id(s)].append((k[r * rb:(r + 1) * rb], v[r * rb:(r + 1) * rb]))
    err = float(np.abs(o.cpu().numpy() - t.expected_out([a, b], q, 8)).max())
    assert err < 2e-3, err


def test_batch_decode_session_argument_errors():
    t = _Twin("bfloat16", 2, 128, 16, capacity=64, seed=3)
    a = kv.SequenceState(1, t.pool)
    with pytest.raises(ValueError):
        kv.BatchDecodeSession(t.storage, [a], 8)       # empty sequence
    t.prefill(a, 5)
    with pytest.raises(ValueError):
        kv.BatchDecodeSession(t.storage, [a, a], 8)    # twice
    with pytest.raises(ValueError):
        kv.BatchDecodeSession(t.storage, [a], 3)       # head ratio
    sess = kv.BatchDecodeSession(t.storage, [a], 8)
    x = torch.zeros(4096, device="cuda")
    with pytest.raises(ValueError):
        sess.step(np.zeros(512, np.uint8), x, x, x)    # host K
    assert a.num_tokens() == 5                        # nothing appended on a rejected call


def test_batch_decode_session_step_host_matches_step():
    """step_host (pinned host K/V/Q/O, two row chunks) gives the bits of
    step() on device copies, on twin sessions built from the same seeds."""
    kvh, hd, bs, group = 2, 128, 16, 4
    qh = kvh * group
    twins = [_Twin("bfloat16", kvh, hd, bs, capacity=4096, seed=41) for _ in range(2)]
    batches = []
    for t in twins:
        seqs = []
        for i in range(20):                      # >= 16 rows: the two-chunk path
            s = kv.SequenceState(i + 1, t.pool)
            t.prefill(s, 1 + 37 * i)
            seqs.append(s)
        seqs.append(t.fork(seqs[3], 99))         # a shared partial page: copy-on-write on the first step
        batches.append(seqs)
    sess = [kv.BatchDecodeSession(t.storage, b, qh) for t, b in zip(twins, batches)]
    batch = len(batches[0])
    for step in range(5):
        k, v = twins[0].rand_rows(batch)
        twins[1].rand_rows(batch)
        q = w.normal(500 + step, batch * qh * hd)
        o_dev = torch.empty(batch * qh * hd, device="cuda")
        locs_d = sess[0].step(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(q).cuda(),
                              o_dev)
        kp, vp = torch.from_numpy(k).pin_memory(), torch.from_numpy(v).pin_memory()
        qp, op = torch.from_numpy(q).pin_memory(), torch.full((batch * qh * hd,), 3.0).pin_memory()
        locs_h = sess[1].step_host(kp, vp, qp, op)
        assert [(a.physical_block, a.offset_in_block) for a in locs_d] == \
            [(a.physical_block, a.offset_in_block) for a in locs_h]
        assert np.array_equal(o_dev.cpu().numpy().view(np.uint32), op.numpy().view(np.uint32)), step
        rb = kvh * hd * 2
        for t in twins:
            for r, s in enumerate(batches[twins.index(t)]):
                t.rows[id(s)].append((k[r * rb:(r + 1) * rb], v[r * rb:(r + 1) * rb]))
        err = float(np.abs(op.numpy() - twins[1].expected_out(batches[1], q, qh)).max())
        assert err < 2e-3, (step, err)
    with pytest.raises(ValueError):
        sess[1].step_host(np.zeros(8, np.uint8), vp, qp, op)   # pageable K

"""Parity at the benchmark configurations' full sizes (the same setup code the
benchmark times): config 1 exactly as stated (the reference's [27, 3, 91]
request, written, gathered and decoded through the drop-in API against the
oracle); config 2's step write against the oracle's write on host mirrors of
every touched page, its batched gather byte for byte against the oracle's
gather for 8 whole sequences, and every byte of every sequence against the
rows that were written; every row of config 3's batch decode against the
FP64 oracle, sampled requests of config 5, and config 4's prefix-sharing flow
(copy-on-write page copies byte-exact, prefill rows against the oracle)."""
import ctypes

import numpy as np
import pytest
import torch

import bench
import kvflux_b200 as kv
import oracle
from gpu_util import d2h
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu


def test_config1_verbatim_through_the_api(cuda):
    """Config 1: one request of 40 tokens on pages [27, 3, 91] of a 128-page
    pool (the recipe of the reference's tests/paged_kv_read_test.cpp:42-49),
    8 Q / 2 KV heads, head_size 64, FP32 Q/K/V ~ N(0, 1) from a seed. K/V go
    in through write_paged_kv over build_slot_mapping, come back through
    read_paged_kv, and the last token's query is decoded by
    paged_attention_batch and by paged_attention (query_tokens = 1); the
    write and gather are compared with the oracle's byte for byte and the
    attention with the oracle's reference_attention within 1e-5."""
    heads, qh, hd, bs, tokens = 2, 8, 64, 16, 40
    pool = kv.PhysicalBlockPool(128, bs)
    st = kv.PagedKVStorage(pool, heads, hd, kv.DType.Float32, 0)
    held = [pool.allocate() for _ in range(27)]
    req = kv.SequenceState(1001, pool)
    req.append_tokens(16)
    held += [pool.allocate() for _ in range(28, 91)]
    pool.free(held[3])
    req.append_tokens(16)
    req.append_tokens(8)
    assert kv.build_read_block_table(req) == [27, 3, 91]
    slots = kv.build_slot_mapping([(req, t) for t in range(tokens)])
    assert slots == list(range(432, 448)) + list(range(48, 64)) + list(range(1456, 1464))

    n = tokens * heads * hd
    k = w.normal(0xC0F1, n)
    v = w.normal(0xC0F1 + 1, n)
    q = w.normal(0xC0F1 + 2, qh * hd)
    kv.write_paged_kv(st, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), slots)

    # The whole cache against the oracle's write into a zeroed host cache.
    lay = st.layout()
    row_bytes = hd * 4
    hk = np.zeros(lay.cache_bytes(), np.uint8)
    hv = np.zeros_like(hk)
    dk, dv = d2h(st.key_base(), lay.cache_bytes()), d2h(st.value_base(), lay.cache_bytes())
    oracle.write(hk, hv, 128, heads, bs, row_bytes, k.view(np.uint8), v.view(np.uint8), np.array(slots, np.uint64))
    touched = np.zeros(128, bool)
    touched[[27, 3, 91]] = True
    page = lay.page_bytes()
    for pid in np.nonzero(touched)[0]:
        lo = pid * page
        # tokens past 40 in page 91 were never written: compare written rows only
        rows = bs if pid != 91 else 8
        for h in range(heads):
            a = lo + (h * bs) * row_bytes
            assert np.array_equal(dk[a:a + rows * row_bytes], hk[a:a + rows * row_bytes]), (pid, h)
            assert np.array_equal(dv[a:a + rows * row_bytes], hv[a:a + rows * row_bytes]), (pid, h)

    ko = torch.empty(n, device="cuda")
    vo = torch.empty(n, device="cuda")
    kv.read_paged_kv(st, req, ko, vo)
    ek, ev = oracle.gather(hk, hv, 128, heads, bs, row_bytes, np.array([27, 3, 91], np.uint64), tokens)
    assert np.array_equal(ko.cpu().numpy().view(np.uint8), ek)
    assert np.array_equal(vo.cpu().numpy().view(np.uint8), ev)
    assert np.array_equal(ek.view(np.float32), k) and np.array_equal(ev.view(np.float32), v)

    exp = oracle.reference_attention(q, k, v, (1, tokens, qh, heads, hd))
    qd = torch.from_numpy(q).cuda()
    ob = torch.full((qh * hd,), float("nan"), device="cuda")
    kv.paged_attention_batch(st, [req], qd, ob, qh)
    err_b = float(np.abs(ob.cpu().numpy() - exp).max())
    op = torch.full((qh * hd,), float("nan"), device="cuda")
    kv.paged_attention(st, req, qd, op, 1, qh)
    err_p = float(np.abs(op.cpu().numpy() - exp).max())
    assert err_b < 1e-5 and err_p < 1e-5, (err_b, err_p)
    assert kv.device_status(0) == 0


def _pages_to_host(storage, pids):
    """K and V bytes of pages `pids` (in that order) as [len][page_bytes]."""
    page = storage.layout().page_bytes()
    hk = np.empty((len(pids), page), np.uint8)
    hv = np.empty_like(hk)
    for i, p in enumerate(pids):
        bench.d2h(storage.key_base() + int(p) * page, hk[i])
        bench.d2h(storage.value_base() + int(p) * page, hv[i])
    return hk, hv


def test_config2_full_size_against_oracle(cuda):
    """Config 2 at full size (64 sequences x 8192 tokens on the odd/even
    65,536-page pool). (1) The step's 256-row write: every touched page is
    mirrored on the host before the write, the oracle's write is applied to
    the mirror, and the device pages after the write equal it byte for byte.
    (2) The batched gather of 8 whole sequences (0 and 63 among them) equals
    the oracle's gather over host copies of all their pages. (3) Every byte of
    every sequence's gather equals the rows written into it: the fill's rows
    (regenerated from their seed) and the step's rows."""
    cfg = w.CONFIG2
    wg = bench.WriteGather(kv, w, cfg, 0, 1)
    heads, hd, bs = wg.heads, wg.hd, wg.bs
    row_bytes = hd * 2
    pre, new, nseq, L = cfg["prefill"], cfg["new_tokens"], wg.nseq, wg.total_len

    # (1) the step write against the oracle's on host mirrors of its pages
    touched = np.unique(wg.slots_np // np.uint64(bs))
    remap = {int(p): i for i, p in enumerate(touched)}
    mk, mv = _pages_to_host(wg.storage, touched)
    wg.write(None)
    torch.cuda.synchronize()
    compact = np.array([remap[int(s) // bs] * bs + int(s) % bs for s in wg.slots_np], np.uint64)
    k_rows = wg.k_new.cpu().view(torch.int16).numpy().view(np.uint8)
    v_rows = wg.v_new.cpu().view(torch.int16).numpy().view(np.uint8)
    oracle.write(mk.reshape(-1), mv.reshape(-1), len(touched), heads, bs, row_bytes, k_rows, v_rows, compact)
    dk, dv = _pages_to_host(wg.storage, touched)
    assert np.array_equal(dk, mk) and np.array_equal(dv, mv)

    # (2) the batched gather against the oracle's, 8 whole sequences
    wg.gather(None)
    torch.cuda.synchronize()
    table, _ = wg.b.table()
    per = L * heads * hd
    for r in (0, 9, 18, 27, 36, 45, 54, 63):
        pids = table[r, :L // bs]
        hk, hv = _pages_to_host(wg.storage, pids)
        ek, ev = oracle.gather(hk.reshape(-1), hv.reshape(-1), len(pids), heads, bs, row_bytes,
                               np.arange(len(pids), dtype=np.uint64), L)
        gk = wg.k_out[r * per:(r + 1) * per].cpu().view(torch.int16).numpy().view(np.uint8)
        gv = wg.v_out[r * per:(r + 1) * per].cpu().view(torch.int16).numpy().view(np.uint8)
        assert np.array_equal(gk, ek), r
        assert np.array_equal(gv, ev), r

    # (3) every sequence: its fill rows (bench.fill_cache's seeded stream,
    # regenerated chunk by chunk in the same order) then the step's rows
    gen = torch.Generator(device="cuda")
    gen.manual_seed(cfg["seed"] * 5)
    chunk = 1 << 16
    k_exp = torch.empty(nseq * per, dtype=torch.bfloat16, device="cuda")
    v_exp = torch.empty_like(k_exp)
    rows = heads * hd
    for start in range(0, nseq * L, chunk):
        cnt = min(chunk, nseq * L - start)
        kb = torch.empty(chunk * rows, dtype=torch.bfloat16, device="cuda")
        vb = torch.empty_like(kb)
        kb[:cnt * rows].normal_(generator=gen)
        vb[:cnt * rows].normal_(generator=gen)
        k_exp[start * rows:(start + cnt) * rows] = kb[:cnt * rows]
        v_exp[start * rows:(start + cnt) * rows] = vb[:cnt * rows]
    k_exp = k_exp.view(nseq, L, heads, hd)
    v_exp = v_exp.view(nseq, L, heads, hd)
    k_exp[:, pre:] = wg.k_new.view(nseq, new, heads, hd)
    v_exp[:, pre:] = wg.v_new.view(nseq, new, heads, hd)
    assert torch.equal(wg.k_out.view(torch.int16), k_exp.reshape(-1).view(torch.int16))
    assert torch.equal(wg.v_out.view(torch.int16), v_exp.reshape(-1).view(torch.int16))
    assert kv.device_status(0) == 0


def test_config2_write_gather_roundtrip(cuda):
    wg = bench.WriteGather(kv, w, w.CONFIG2, 0, 1)
    wg.write(None)
    wg.gather(None)
    torch.cuda.synchronize()
    per = wg.total_len * wg.heads * wg.hd
    # The step's 4 new tokens of every sequence come back at positions 8188..8191.
    pre = w.CONFIG2["prefill"]
    new = w.CONFIG2["new_tokens"]
    k_out = wg.k_out.view(wg.nseq, wg.total_len, wg.heads, wg.hd)
    v_out = wg.v_out.view(wg.nseq, wg.total_len, wg.heads, wg.hd)
    k_new = wg.k_new.view(wg.nseq, new, wg.heads, wg.hd)
    v_new = wg.v_new.view(wg.nseq, new, wg.heads, wg.hd)
    assert torch.equal(k_out[:, pre:].view(torch.int16), k_new.view(torch.int16))
    assert torch.equal(v_out[:, pre:].view(torch.int16), v_new.view(torch.int16))
    # Every other token: the gather of every sequence equals a gather through
    # the single-sequence entry point (independent kernel path) for 3 sequences.
    for r in (0, 31, 63):
        ko = torch.empty(per, dtype=torch.bfloat16, device="cuda")
        vo = torch.empty_like(ko)
        kv.read_paged_kv(wg.storage, wg.b.sequences[r], ko, vo)
        assert torch.equal(ko.view(torch.int16), wg.k_out[r * per:(r + 1) * per].view(torch.int16))
        assert torch.equal(vo.view(torch.int16), wg.v_out[r * per:(r + 1) * per].view(torch.int16))
    assert kv.device_status(0) == 0


def _decode_vs_oracle(wl, requests, tol):
    wl.launch(None)
    torch.cuda.synchronize()
    hk, hv, nb, table, lens, q, o_gpu = wl.host_sample(requests)
    exp = oracle.decode_batch(hk, hv, 1, nb, wl.kvh, wl.bs, wl.hd, table, lens, wl.qh, q, threads=16)
    err = float(np.abs(o_gpu - exp).max())
    assert np.isfinite(o_gpu).all()
    assert err < tol, err
    return err


def test_config3_decode_all_rows(cuda):
    wl = bench.Decode(kv, w, w.CONFIG3, 0, 1)
    _decode_vs_oracle(wl, list(range(wl.batch)), 2e-3)


def test_config3_api_matches_capi(cuda):
    """paged_attention_batch (host table written in parallel into pinned
    staging) against the C-ABI launch on the same table: bit-identical."""
    wl = bench.Decode(kv, w, w.CONFIG3, 0, 1)
    wl.launch(None)
    torch.cuda.synchronize()
    ref = wl.o.clone()
    wl.o.fill_(12345.0)
    kv.paged_attention_batch(wl.storage, wl.b.sequences, wl.q, wl.o, wl.qh)
    assert torch.equal(wl.o, ref)
    assert kv.device_status(0) == 0


def test_config3_api_waits_for_callers_upload(cuda):
    """The API's second chunk runs on its own stream; it must still see the Q
    that the caller uploaded on the default stream just before the call, even
    when that upload is held back (a ~1 ms spin queued ahead of it)."""
    wl = bench.Decode(kv, w, w.CONFIG3, 0, 1)
    wl.launch(None)
    torch.cuda.synchronize()
    ref = wl.o.clone()
    q_host = wl.q.cpu().pin_memory()
    wl.q.zero_()
    wl.o.fill_(12345.0)
    torch.cuda.synchronize()
    torch.cuda._sleep(2_000_000)
    wl.q.copy_(q_host, non_blocking=True)
    kv.paged_attention_batch(wl.storage, wl.b.sequences, wl.q, wl.o, wl.qh)
    torch.cuda.synchronize()
    assert torch.equal(wl.o, ref)
    assert kv.device_status(0) == 0


def test_api_workspace_reused_across_shapes(cuda):
    """Two paged_attention_batch calls on one storage: 16 rows of 4096 tokens
    (every (request, head, split) partial written), then 3 of those rows, on
    the storage's one workspace: right only if the first launch left every
    split counter at zero for the second."""
    cfg = dict(batch=16, q_heads=32, kv_heads=8, head_size=128, block_size=16, min_len=4096, max_len=4096,
               dtype="bfloat16", seed=0xC0F6)
    wl = bench.Decode(kv, w, cfg, 0, 1)
    seqs = wl.b.sequences
    kv.paged_attention_batch(wl.storage, seqs, wl.q, wl.o, wl.qh)
    torch.cuda.synchronize()
    pick = [2, 9, 15]
    q2 = wl.q.view(wl.batch, -1)[pick].contiguous().view(-1)
    o2 = torch.full_like(q2, float("nan"))
    kv.paged_attention_batch(wl.storage, [seqs[i] for i in pick], q2, o2, wl.qh)
    torch.cuda.synchronize()
    hk, hv, nb, table, lens, q, o_first = wl.host_sample(pick)
    exp = oracle.decode_batch(hk, hv, 1, nb, wl.kvh, wl.bs, wl.hd, table, lens, wl.qh, q, threads=16)
    got = o2.cpu().numpy()
    assert np.isfinite(got).all()
    assert float(np.abs(got - exp).max()) < 2e-3
    assert float(np.abs(o_first - exp).max()) < 2e-3
    assert kv.device_status(0) == 0


def test_config5_decode_sampled_rows(cuda):
    wl = bench.Decode(kv, w, w.CONFIG5, 0, 1)
    lens = wl.lens
    pick = [int(np.argmin(lens)), int(np.argmax(lens)), 0, 100, 255]
    _decode_vs_oracle(wl, pick, 2e-3)


def test_config4_prefix_sharing_cow_and_prefill(cuda):
    cfg = dict(w.CONFIG4)
    pf = bench.Prefill(kv, w, cfg)
    assert pf.cow_copies == cfg["shared_group"] - 1
    # Shared full pages are the same physical pages; the copied tail pages are
    # distinct and hold byte-identical first 8 tokens.
    bs, shared = 16, cfg["shared_prefix"]
    full = shared // bs
    ids = [kv.build_read_block_table(s) for s in pf.seqs[:cfg["shared_group"]]]
    for t in ids[1:]:
        assert t[:full] == ids[0][:full]
    tails = [t[full] for t in ids]
    assert len(set(tails)) == len(tails)
    lay = pf.storage.layout()
    page = lay.page_bytes()

    def page_bytes(kind, pid):
        out = np.empty(page, np.uint8)
        bench.d2h((pf.storage.key_base() if kind == 0 else pf.storage.value_base()) + pid * page, out)
        return out.reshape(cfg["kv_heads"], 16, 128 * 2)

    for kind in (0, 1):
        ref_page = page_bytes(kind, tails[0])
        for tail in tails[1:]:
            # tokens 0..7 were copied, token 8 is each sequence's own new token
            assert np.array_equal(page_bytes(kind, tail)[:, :8], ref_page[:, :8])

    # Prefill of sequence 1 (shares 2056 tokens with sequence 0) and 5: sampled rows.
    L, qh = pf.L, pf.qh
    for si in (1, 5):
        t = pf.tables[si]
        rc = kv.lib.kvfx_attention(ctypes.byref(pf.desc), pf.q.data_ptr(), pf.o.data_ptr(), t.data_ptr(), L, L, qh,
                                   None, 0, None)
        kv.check(rc, "kvfx_attention")
        torch.cuda.synchronize()
        blocks = np.array(kv.build_read_block_table(pf.seqs[si]), np.uint64)
        uniq = np.unique(blocks)
        remap = {int(p): i for i, p in enumerate(uniq)}
        hk = np.empty((len(uniq), page), np.uint8)
        hv = np.empty_like(hk)
        for i, p in enumerate(uniq):
            bench.d2h(pf.storage.key_base() + int(p) * page, hk[i])
            bench.d2h(pf.storage.value_base() + int(p) * page, hv[i])
        ctab = np.array([remap[int(p)] for p in blocks], np.uint64)
        q = pf.q.cpu().numpy()
        got = pf.o.cpu().numpy().reshape(L, -1)
        for lo, hi in [(0, 64), (2048, 2072), (L - 32, L)]:
            exp = oracle.attention_rows(hk.reshape(-1), hv.reshape(-1), 1, len(uniq), cfg["kv_heads"], 16, 128, ctab,
                                        L, L, qh, q, row_begin=lo, row_end=hi, threads=16).reshape(L, -1)
            err = float(np.abs(got[lo:hi] - exp[lo:hi]).max())
            assert err < 2e-3, (si, lo, err)

"""Parity at the benchmark configurations' full sizes (the same setup code the
benchmark times): byte-exact write -> gather round trips on config 2, every
row of config 3's batch decode against the FP64 oracle, sampled requests of
config 5, and config 4's prefix-sharing flow (copy-on-write page copies
byte-exact, prefill rows against the oracle)."""
import ctypes

import numpy as np
import pytest
import torch

import bench
import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu


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
    (every (request, head, split) partial written), then 3 of those rows. The
    second call's split counters lie where the first call's partials are: it
    is right only if each launch starts from cleared counters."""
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

"""paged_attention_batch keeps the batch page table on the GPU between calls
and uploads only what changed. Every call here is checked against the
oracle's decode over the whole table (build_batch_block_table of the same
sequences), while the batch changes between calls in every way a serving loop
changes it: rows growing by tokens and pages, a forked row whose shared
partial page is copied on write, rows reordered, dropped, added and repeated.
The bytes each call uploads show that unchanged rows are not re-sent, and a
handle that went stale under a row kept from an earlier call still raises
std::invalid_argument (ValueError here), as build_batch_block_table does."""
import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from gpu_util import h2d
from kvflux_b200 import workloads as w

pytestmark = pytest.mark.gpu

KVH, QH, HD, BS, PAGES = 2, 8, 128, 16, 2048


class Setup:
    def __init__(self):
        self.pool = kv.PhysicalBlockPool(PAGES, BS)
        self.st = kv.PagedKVStorage(self.pool, KVH, HD, kv.DType.BFloat16, 0)
        lay = self.st.layout()
        n = lay.cache_bytes() // 2
        # Every page holds seeded data, so rows may read any page (the test
        # checks addressing, not the write kernel).
        self.hk = w.encode(w.normal(0xA1, n), "bfloat16")
        self.hv = w.encode(w.normal(0xA2, n), "bfloat16")
        h2d(self.st.key_base(), self.hk.view(np.uint8))
        h2d(self.st.value_base(), self.hv.view(np.uint8))
        self.calls = 0

    def mirror_copy(self, src, dst):
        """The host mirror of a whole-page copy (what append_token_cow did)."""
        per = KVH * BS * HD
        self.hk[dst * per:(dst + 1) * per] = self.hk[src * per:(src + 1) * per]
        self.hv[dst * per:(dst + 1) * per] = self.hv[src * per:(src + 1) * per]

    def run(self, seqs, tol=2e-3):
        """paged_attention_batch and paged_attention_batch_host on `seqs`;
        both against the oracle. Returns the first call's upload bytes."""
        self.calls += 1
        b = len(seqs)
        q = w.normal(0xB0 + self.calls, b * QH * HD)
        qd = torch.from_numpy(q).cuda()
        o = torch.full((b * QH * HD,), float("nan"), device="cuda")
        kv.paged_attention_batch(self.st, seqs, qd, o, QH)
        up = kv.paged_attention_batch_table_upload_bytes(self.st)
        qh_ = torch.from_numpy(q).pin_memory()
        oh = torch.full_like(qh_, float("nan")).pin_memory()
        kv.paged_attention_batch_host(self.st, seqs, qh_, oh, QH)
        t = kv.build_batch_block_table(seqs)
        table = np.array(t.block_table(), np.uint64).reshape(b, t.max_blocks_per_sequence())
        lens = np.array(t.sequence_lengths(), np.uint64)
        exp = oracle.decode_batch(self.hk.view(np.uint8), self.hv.view(np.uint8), 1, PAGES, KVH, BS, HD, table, lens,
                                  QH, q, threads=8)
        got = o.cpu().numpy()
        assert np.isfinite(got).all()
        assert float(np.abs(got - exp).max()) < tol
        assert np.array_equal(oh.numpy().view(np.uint32), got.view(np.uint32))  # host form: bit-identical
        assert kv.device_status(0) == 0
        return up


def _pages(seqs):
    return sum(s.num_allocated_blocks() for s in seqs)


def test_resident_table_follows_every_change(cuda):
    S = Setup()
    lens = [1, 15, 16, 17, 33, 300, 512, 700, 65, 130, 2, 47]
    seqs = []
    for i, L in enumerate(lens):
        s = kv.SequenceState(i + 1, S.pool)
        s.append_tokens(L)
        seqs.append(s)
    full = S.run(seqs)
    assert full >= 8 * _pages(seqs)
    # Unchanged batch: only the lengths go up.
    assert S.run(seqs) <= 512

    # Rows grow: new tokens in old pages and new pages.
    seqs[0].append_tokens(40)
    seqs[3].append_token()
    seqs[7].append_tokens(16)
    grown = S.run(seqs)
    # lengths + 2 runs + 3 new ids, each array at a 256-byte aligned offset
    assert grown <= 3 * 256 < full

    # A forked row whose shared partial last page is copied on write.
    child = seqs[5].fork_shared(100)
    kv.append_token_cow(S.st, child)
    src = seqs[5].physical_block_id(seqs[5].num_allocated_blocks() - 1)
    dst = child.physical_block_id(child.num_allocated_blocks() - 1)
    assert src != dst
    S.mirror_copy(src, dst)
    seqs.append(child)
    S.run(seqs)
    kv.append_token_cow(S.st, seqs[5])  # the parent's page is private again: no copy
    S.run(seqs)

    # Reordered, dropped, repeated and new rows.
    seqs = seqs[::-1]
    S.run(seqs)
    seqs = seqs[:7]
    S.run(seqs)
    extra = kv.SequenceState(200, S.pool)
    extra.append_tokens(999)
    seqs = seqs + [extra, seqs[0]]
    S.run(seqs)
    # Longer rows than the resident table's row stride: it is re-laid out.
    extra.append_tokens(4000)
    S.run(seqs)
    assert S.run(seqs) <= 512


def test_stale_handle_under_a_kept_row_raises(cuda):
    S = Setup()
    seqs = []
    for i, L in enumerate([40, 64, 20]):
        s = kv.SequenceState(i + 1, S.pool)
        s.append_tokens(L)
        seqs.append(s)
    S.run(seqs)
    S.run(seqs)  # row 1 is now kept on the device
    cache = kv.PrefixCache(S.pool)
    cache.publish_computed_block(seqs[1], 0, list(range(16)))
    h = seqs[1].block_table().handle(0)
    S.pool.free(h)  # misuse: drops the table's own reference (page goes idle)
    qd = torch.zeros(3 * QH * HD, device="cuda")
    o = torch.empty_like(qd)
    with pytest.raises(ValueError):
        kv.paged_attention_batch(S.st, seqs, qd, o, QH)
    S.pool.retain(h)  # the reference is back: the same handle is live again
    S.run(seqs)

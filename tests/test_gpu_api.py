"""The reference's GPU tests, ported to the Python binding of the drop-in C++
API (KVFlux tests/paged_kv_write_test.cpp, paged_kv_read_test.cpp,
paged_kv_gather_test.cpp, paged_kv_storage_test.cpp, paged_attention_test.cu,
paged_attention_batch_test.cu, copy_on_write_gpu_test.cpp,
sequence_lifecycle_test.cpp). Same recipes, payloads, sentinels and
tolerances (max_abs_err < 1e-5 for all three dtypes against
reference_attention, here the oracle's bit-exact restatement of it)."""
import math

import numpy as np
import pytest
import torch

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w
from gpu_util import memset, read_elem

pytestmark = pytest.mark.gpu

INT = {2: torch.int16, 4: torch.int32}
NPU = {2: np.uint16, 4: np.uint32}
DT = [(kv.DType.Float16, 2), (kv.DType.BFloat16, 2), (kv.DType.Float32, 4)]
DNAME = {kv.DType.Float16: "float16", kv.DType.BFloat16: "bfloat16", kv.DType.Float32: "float32"}


def dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def host(t: torch.Tensor, np_dtype) -> np.ndarray:
    return t.cpu().numpy().view(np_dtype)


@pytest.mark.parametrize("dtype,elem", DT)
def test_write_three_slots_and_untouched_neighbours(cuda, dtype, elem):
    heads, dims, bs = 2, 4, 16
    pool = kv.PhysicalBlockPool(64, bs)
    st = kv.PagedKVStorage(pool, heads, dims, dtype)
    held = []

    def occupy(n):
        while pool.capacity() - pool.available() < n:
            held.append(pool.allocate())

    occupy(10)
    a = kv.SequenceState(1001, pool)
    a.append_tokens(14)
    occupy(32)
    b = kv.SequenceState(1002, pool)
    b.append_tokens(11)
    occupy(59)
    c = kv.SequenceState(1003, pool)
    c.append_tokens(1)
    slots = kv.build_slot_mapping([(a, 13), (b, 10), (c, 0)])
    assert slots == [173, 522, 944]
    lay = st.layout()
    memset(st.key_base(), 0xA5, lay.total_bytes())
    n = len(slots) * heads * dims
    keys = (0x1200 + np.arange(n)).astype(NPU[elem])
    vals = (0x3400 + np.arange(n)).astype(NPU[elem])
    kd, vd = dev(keys), dev(vals)
    kv.write_paged_kv(st, kd, vd, slots)
    for bi, s in enumerate(slots):
        for h in range(heads):
            for d in range(dims):
                i = (bi * heads + h) * dims + d
                assert read_elem(st.slot_address(kv.KVKind.Key, s, h, d), elem) == keys[i]
                assert read_elem(st.slot_address(kv.KVKind.Value, s, h, d), elem) == vals[i]
    untouched = 0xA5A5 if elem == 2 else 0xA5A5A5A5
    for s in slots:
        assert read_elem(st.slot_address(kv.KVKind.Key, s + 1, 1, 3), elem) == untouched
        assert read_elem(st.slot_address(kv.KVKind.Value, s + 1, 1, 3), elem) == untouched
    kv.write_paged_kv(st, None, None, [])
    with pytest.raises(ValueError):
        kv.write_paged_kv(st, None, vd, slots)
    with pytest.raises(IndexError):
        kv.write_paged_kv(st, kd, vd, [lay.slot_count()])
    with pytest.raises(ValueError):
        kv.write_paged_kv(st, kd, vd, [173, 173])
    with pytest.raises(ValueError):
        kv.write_paged_kv(st, keys, vd, slots)  # host pointer
    del a, b, c
    for h in held:
        pool.free(h)
    assert pool.available() == pool.capacity()


@pytest.mark.parametrize("dtype,elem", DT)
def test_read_27_3_91_sentinel_and_prefix_shared(cuda, dtype, elem):
    heads, dims, tokens = 2, 3, 40
    n = tokens * heads * dims
    pool = kv.PhysicalBlockPool(96, 16)
    st = kv.PagedKVStorage(pool, heads, dims, dtype)
    held = [pool.allocate() for _ in range(27)]
    r = kv.SequenceState(1001, pool)
    r.append_tokens(16)
    held += [pool.allocate() for _ in range(28, 91)]
    pool.free(held[3])
    r.append_tokens(16)
    r.append_tokens(8)
    assert kv.build_read_block_table(r) == [27, 3, 91]
    slots = kv.build_slot_mapping([(r, t) for t in range(tokens)])
    keys = (0x1000 + np.arange(n)).astype(NPU[elem])
    vals = (0x3000 + np.arange(n)).astype(NPU[elem])
    kv.write_paged_kv(st, dev(keys), dev(vals), slots)
    ko = torch.full((n + 1,), -23131 if elem == 2 else -1515870811, dtype=INT[elem], device="cuda")  # 0xA5A5...
    vo = ko.clone()
    kv.read_paged_kv(st, r, ko, vo)
    ak, av = host(ko, NPU[elem]), host(vo, NPU[elem])
    assert np.array_equal(ak[:n], keys) and np.array_equal(av[:n], vals)
    sentinel = 0xA5A5 if elem == 2 else 0xA5A5A5A5
    assert ak[n] == sentinel and av[n] == sentinel

    cache = kv.PrefixCache(pool)
    prompt = list(range(tokens))
    cache.publish_computed_block(r, 0, prompt[:16])
    cache.publish_computed_block(r, 1, prompt[:32])
    shared = kv.SequenceState(1004, pool)
    prompt[32] = 999
    assert cache.attach_cached_prefix(shared, prompt) == 32
    kv.read_paged_kv(st, shared, ko, vo)
    m = 32 * heads * dims
    assert np.array_equal(host(ko, NPU[elem])[:m], keys[:m])
    assert np.array_equal(host(vo, NPU[elem])[:m], vals[:m])

    with pytest.raises(ValueError):
        kv.read_paged_kv(st, r, None, vo)
    with pytest.raises(ValueError):
        kv.read_paged_kv(st, r, ko, ko)
    with pytest.raises(ValueError):
        kv.read_paged_kv(st, r, keys, vo)
    with pytest.raises(ValueError):
        kv.read_paged_kv(st, r, st.key_base(), vo)
    other_pool = kv.PhysicalBlockPool(96, 16)
    other = kv.SequenceState(1002, other_pool)
    other.append_tokens(1)
    with pytest.raises(ValueError):
        kv.read_paged_kv(st, other, ko, vo)
    empty = kv.SequenceState(1003, pool)
    kv.read_paged_kv(st, empty, None, None)


@pytest.mark.parametrize("dtype,elem", DT)
def test_interleaved_requests_gather_independently(cuda, dtype, elem):
    heads, dims = 2, 3
    ept = heads * dims
    pool = kv.PhysicalBlockPool(5, 2)
    st = kv.PagedKVStorage(pool, heads, dims, dtype)
    a, b = kv.SequenceState(101, pool), kv.SequenceState(202, pool)
    a.append_tokens(2)
    b.append_tokens(2)
    a.append_tokens(2)
    b.append_tokens(2)
    a.append_token()
    assert kv.build_read_block_table(a) == [0, 2, 4] and kv.build_read_block_table(b) == [1, 3]
    writes = [(b, 0), (a, 0), (b, 1), (a, 1), (b, 2), (a, 2), (b, 3), (a, 3), (a, 4)]
    ik, iv = [], []
    exp = {id(a): (np.zeros(5 * ept, NPU[elem]), np.zeros(5 * ept, NPU[elem])),
           id(b): (np.zeros(4 * ept, NPU[elem]), np.zeros(4 * ept, NPU[elem]))}
    for s, pos in writes:
        for e in range(ept):
            ident = (100 if s is a else 200) + pos * ept + e
            ik.append(0x1000 + ident)
            iv.append(0x3000 + ident)
            exp[id(s)][0][pos * ept + e] = 0x1000 + ident
            exp[id(s)][1][pos * ept + e] = 0x3000 + ident
    kv.write_paged_kv(st, dev(np.array(ik, NPU[elem])), dev(np.array(iv, NPU[elem])), kv.build_slot_mapping(writes))
    for s in (a, b):
        ek, ev = exp[id(s)]
        ko = torch.full((ek.size + 1,), -23131 if elem == 2 else -1515870811, dtype=INT[elem], device="cuda")
        vo = ko.clone()
        kv.read_paged_kv(st, s, ko, vo)
        assert np.array_equal(host(ko, NPU[elem])[:-1], ek) and np.array_equal(host(vo, NPU[elem])[:-1], ev)
        assert host(ko, NPU[elem])[-1] == (0xA5A5 if elem == 2 else 0xA5A5A5A5)
    assert pool.available() == 0


def test_storage_addresses_and_slot_roundtrip(cuda):
    pool = kv.PhysicalBlockPool(4, 2)
    st = kv.PagedKVStorage(pool, 2, 3, kv.DType.Float32)
    lay = st.layout()
    assert (lay.page_bytes(), lay.cache_bytes(), lay.total_bytes(), lay.slot_count()) == (48, 192, 384, 8)
    assert st.value_base() == st.key_base() + lay.cache_bytes()
    r = kv.SequenceState(1001, pool)
    r.append_tokens(5)
    holder = pool.allocate()
    assert pool.id(holder) == 3
    assert st.page_address(kv.KVKind.Key, holder) == st.key_base() + 3 * 48
    assert st.element_address(kv.KVKind.Value, holder, 1, 1, 2) == st.value_base() + 3 * 48 + (6 + 3 + 2) * 4
    assert st.slot_address(kv.KVKind.Key, 6, 1, 1) == st.element_address(kv.KVKind.Key, holder, 1, 0, 1)
    with pytest.raises(IndexError):
        st.slot_address(kv.KVKind.Key, 8, 0, 0)
    with pytest.raises(IndexError):
        st.slot_address(kv.KVKind.Key, 0, 2, 0)
    pool.free(holder)
    with pytest.raises(ValueError):
        st.page_address(kv.KVKind.Key, holder)
    reused = pool.allocate()
    assert reused.id == holder.id and reused.generation != holder.generation


def _attention_compare(dtype, elem, query_tokens_list):
    tokens, kvh, qh, hd = 10, 2, 4, 4
    n = tokens * kvh * hd
    name = DNAME[dtype]
    pool = kv.PhysicalBlockPool(8, 4)
    st = kv.PagedKVStorage(pool, kvh, hd, dtype)
    held = [pool.allocate() for _ in range(5)]
    s = kv.SequenceState(1001, pool)
    s.append_tokens(4)
    held.append(pool.allocate())
    pool.free(held[1])
    s.append_tokens(4)
    s.append_tokens(2)
    assert kv.build_read_block_table(s) == [5, 1, 7]
    kf = np.array([0.125 * ((i * 7 % 17) - 8) for i in range(n)], np.float32)
    vf = np.array([0.125 * ((i * 11 % 23) - 11) for i in range(n)], np.float32)
    lay = st.layout()
    memset(st.key_base(), 0xFF, lay.total_bytes())
    kv.write_paged_kv(st, dev(w.encode(kf, name)), dev(w.encode(vf, name)),
                      kv.build_slot_mapping([(s, t) for t in range(tokens)]))
    kc = torch.empty(n, dtype=INT[elem], device="cuda")
    vc = torch.empty(n, dtype=INT[elem], device="cuda")
    kv.read_paged_kv(st, s, kc, vc)
    ck = w.decode(host(kc, NPU[elem]), name)
    cv = w.decode(host(vc, NPU[elem]), name)
    assert np.array_equal(ck, w.decode(w.encode(kf, name), name))
    worst = 0.0
    for lq in query_tokens_list:
        q = np.array([0.125 * ((i * 5 % 19) - 9) for i in range(lq * qh * hd)], np.float32)
        expected = oracle.reference_attention(q, ck, cv, (lq, tokens, qh, kvh, hd))
        out = torch.full((lq * qh * hd + 1,), 12345.0, device="cuda")
        qd = dev(q)
        kv.paged_attention(st, s, qd, out, lq, qh)
        got = out.cpu().numpy()
        assert np.isfinite(got[:-1]).all()
        err = float(np.abs(got[:-1] - expected).max())
        assert err < 1e-5, (lq, err)
        worst = max(worst, err)
        assert got[-1] == 12345.0
        if lq == 1:
            with pytest.raises(ValueError):
                kv.paged_attention(st, s, None, out, 1, qh)
            with pytest.raises(ValueError):
                kv.paged_attention(st, s, qd, qd, 1, qh)
            with pytest.raises(ValueError):
                kv.paged_attention(st, s, q, out, 1, qh)
            with pytest.raises(ValueError):
                kv.paged_attention(st, s, qd, out, 1, 3)
            with pytest.raises(ValueError):
                kv.paged_attention(st, s, qd, out, tokens + 1, qh)
    kv.paged_attention(st, s, None, None, 0, qh)
    other_pool = kv.PhysicalBlockPool(8, 4)
    other = kv.SequenceState(1002, other_pool)
    other.append_tokens(1)
    with pytest.raises(ValueError):
        kv.paged_attention(st, other, None, None, 0, qh)
    return worst


@pytest.mark.parametrize("dtype,elem", DT)
def test_paged_attention_matches_reference(cuda, dtype, elem):
    _attention_compare(dtype, elem, [10, 3, 1])


@pytest.mark.parametrize("dtype,elem", DT)
def test_batch_attention_variable_lengths(cuda, dtype, elem):
    kvh, qh, hd = 2, 4, 3
    name = DNAME[dtype]
    tokens = 16
    n = tokens * kvh * hd
    pool = kv.PhysicalBlockPool(16, 4)
    st = kv.PagedKVStorage(pool, kvh, hd, dtype)
    a, b, c = (kv.SequenceState(i, pool) for i in (1, 2, 3))
    a.append_tokens(4)
    b.append_tokens(4)
    c.append_tokens(2)
    a.append_token()
    b.append_tokens(5)
    seqs = [a, b, c]
    t = kv.build_batch_block_table(seqs)
    assert t.sequence_lengths() == [5, 9, 2]
    pad = 2**64 - 1
    assert t.block_table() == [0, 3, pad, 1, 4, 5, 2, pad, pad]
    writes = [(s, p) for s in seqs for p in range(s.num_tokens())]
    kf = np.array([0.125 * ((i * 7 % 19) - 9) for i in range(n)], np.float32)
    vf = np.array([0.125 * ((i * 11 % 23) - 11) for i in range(n)], np.float32)
    lay = st.layout()
    memset(st.key_base(), 0xFF, lay.total_bytes())
    kv.write_paged_kv(st, dev(w.encode(kf, name)), dev(w.encode(vf, name)), kv.build_slot_mapping(writes))
    q = np.array([0.125 * ((i * 5 % 17) - 8) for i in range(3 * qh * hd)], np.float32)
    qd = dev(q)
    out = torch.full((3 * qh * hd + 1,), 12345.0, device="cuda")
    kv.paged_attention_batch(st, seqs, qd, out, qh)
    got = out.cpu().numpy()
    kd = w.decode(w.encode(kf, name), name)
    vd = w.decode(w.encode(vf, name), name)
    off = 0
    for r, s in enumerate(seqs):
        L = s.num_tokens()
        e = oracle.reference_attention(q[r * qh * hd:(r + 1) * qh * hd], kd[off * kvh * hd:(off + L) * kvh * hd],
                                       vd[off * kvh * hd:(off + L) * kvh * hd], (1, L, qh, kvh, hd))
        g = got[r * qh * hd:(r + 1) * qh * hd]
        assert np.isfinite(g).all() and float(np.abs(g - e).max()) < 1e-5
        off += L
    assert got[-1] == 12345.0
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, seqs, None, out, qh)
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, seqs, qd, qd, qh)
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, seqs, q, out, qh)
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, seqs, qd, out, 3)
    empty = kv.SequenceState(4, pool)
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, [a, empty], qd, out, qh)
    op = kv.PhysicalBlockPool(2, 4)
    other = kv.SequenceState(5, op)
    other.append_token()
    with pytest.raises(ValueError):
        kv.paged_attention_batch(st, [a, other], qd, out, qh)
    kv.paged_attention_batch(st, [], None, None, qh)


@pytest.mark.parametrize("dtype,elem", DT)
def test_copy_on_write_gpu_isolation(cuda, dtype, elem):
    heads, dims = 2, 3
    ept = heads * dims
    pool = kv.PhysicalBlockPool(3, 4)
    st = kv.PagedKVStorage(pool, heads, dims, dtype)
    a = kv.SequenceState(1, pool)
    a.append_tokens(3)
    old = a.physical_block_id(0)
    ik = (0x1100 + np.arange(3 * ept)).astype(NPU[elem])
    iv = (0x2200 + np.arange(3 * ept)).astype(NPU[elem])
    kv.write_paged_kv(st, dev(ik), dev(iv), kv.build_slot_mapping([(a, 0), (a, 1), (a, 2)]))
    b = a.fork_shared(2)
    assert pool.ref_count(a.block_table().handle(0)) == 2
    loc = kv.append_token_cow(st, a)
    assert loc.physical_block != old and loc.offset_in_block == 3
    assert a.num_tokens() == 4 and b.num_tokens() == 3 and b.physical_block_id(0) == old
    ak = (0x3300 + np.arange(ept)).astype(NPU[elem])
    av = (0x4400 + np.arange(ept)).astype(NPU[elem])
    bk = (0x5500 + np.arange(ept)).astype(NPU[elem])
    bv = (0x6600 + np.arange(ept)).astype(NPU[elem])
    kv.write_paged_kv(st, dev(ak), dev(av), kv.build_slot_mapping([(a, 3)]))
    outs = [torch.empty(4 * ept, dtype=INT[elem], device="cuda") for _ in range(4)]
    kv.read_paged_kv(st, a, outs[0], outs[1])
    kv.read_paged_kv(st, b, outs[2], outs[3])
    h = [host(o, NPU[elem]) for o in outs]
    assert np.array_equal(h[0][:3 * ept], ik) and np.array_equal(h[2][:3 * ept], ik)
    assert np.array_equal(h[1][:3 * ept], iv) and np.array_equal(h[3][:3 * ept], iv)
    assert np.array_equal(h[0][3 * ept:], ak) and np.array_equal(h[1][3 * ept:], av)
    bl = b.append_token()
    assert bl.physical_block == old and bl.offset_in_block == 3
    kv.write_paged_kv(st, dev(bk), dev(bv), kv.build_slot_mapping([(b, 3)]))
    kv.read_paged_kv(st, b, outs[2], outs[3])
    kv.read_paged_kv(st, a, outs[0], outs[1])
    h = [host(o, NPU[elem]) for o in outs]
    assert np.array_equal(h[2][3 * ept:], bk) and np.array_equal(h[3][3 * ept:], bv)
    assert np.array_equal(h[0][3 * ept:], ak) and np.array_equal(h[0][:3 * ept], ik)
    assert a.physical_block_id(0) != b.physical_block_id(0)


def test_sequence_lifecycle_prefill_decode_release(cuda):
    qh = 2
    pool = kv.PhysicalBlockPool(4, 2)
    st = kv.PagedKVStorage(pool, 1, 2, kv.DType.Float32)
    lay = st.layout()
    memset(st.key_base(), 0xFF, lay.total_bytes())
    keys = [0.2, -0.1, 0.3, 0.4, -0.2, 0.5]
    vals = [1.0, 2.0, 3.0, -1.0, 0.5, 4.0]
    pq = [0.1, 0.2, -0.3, 0.4, 0.5, -0.2, 0.1, 0.3, -0.4, 0.6, 0.2, -0.1]
    f = lambda x: torch.tensor(x, dtype=torch.float32, device="cuda")  # noqa: E731

    def compare(out, q, k, v, lq):
        e = oracle.reference_attention(q, k, v, (lq, len(k) // 2, qh, 1, 2))
        got = out.cpu().numpy()
        assert np.isfinite(got[:e.size]).all() and float(np.abs(got[:e.size] - e).max()) < 1e-5
        assert got[e.size] == 12345.0

    pk, pv, pqd = f(keys), f(vals), f(pq)
    pout = f([12345.0] * 13)
    one_out = f([12345.0] * 5)
    req = kv.SequenceLifecycle(1001, pool, st, qh)
    assert req.sequence().num_tokens() == 0 and pool.available() == 4
    with pytest.raises(ValueError):
        req.prefill(0, pk, pv, pqd, pout)
    assert not req.finished()
    req.prefill(3, pk, pv, pqd, pout)
    assert req.sequence().num_tokens() == 3 and pool.available() == 2
    compare(pout, pq, keys, vals, 3)
    with pytest.raises(kv.LogicError):
        req.prefill(3, pk, pv, pqd, pout)
    with pytest.raises(ValueError):
        req.decode(None, pv, pqd, one_out)
    fk, fv, fq = [0.6, -0.3], [2.0, 1.5], [0.2, 0.7, -0.1, 0.4]
    one_out.copy_(f([12345.0] * 5))
    loc = req.decode(f(fk), f(fv), f(fq), one_out)
    assert loc.offset_in_block == 1 and loc.physical_block == req.sequence().physical_block_id(1)
    keys += fk
    vals += fv
    compare(one_out, fq, keys, vals, 1)
    sk, sv, sq = [-0.5, 0.2], [-2.0, 3.0], [0.8, -0.2, 0.3, 0.1]
    one_out.copy_(f([12345.0] * 5))
    loc2 = req.decode(f(sk), f(sv), f(sq), one_out)
    assert loc2.offset_in_block == 0 and loc2.physical_block == req.sequence().physical_block_id(2)
    keys += sk
    vals += sv
    compare(one_out, sq, keys, vals, 1)
    req.finish()
    assert req.finished() and pool.available() == pool.capacity()
    with pytest.raises(kv.LogicError):
        req.sequence()
    failed = kv.SequenceLifecycle(1002, pool, st, qh)
    with pytest.raises(ValueError):
        failed.prefill(1, pk, pv, np.array(pq, np.float32), one_out)
    assert failed.finished() and pool.available() == pool.capacity()

    pool1 = kv.PhysicalBlockPool(1, 2)
    st1 = kv.PagedKVStorage(pool1, 1, 2, kv.DType.Float32)
    kvd = f([0.1, 0.2, 0.3, 0.4])
    qd = f([0.2, 0.1, 0.4, 0.3, 0.6, 0.5, 0.8, 0.7])
    out = torch.empty(9, device="cuda")
    r = kv.SequenceLifecycle(2001, pool1, st1, 2)
    r.prefill(2, kvd, kvd, qd, out)
    assert pool1.available() == 0
    with pytest.raises(kv.CapacityError):
        r.decode(kvd, kvd, qd, out)
    assert r.finished() and pool1.available() == 1

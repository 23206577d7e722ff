"""Pins the CPU oracle (oracle/kvoracle.c) before it is trusted.

1. The reference's own known answers for reference_attention
   (tests/reference_attention_test.cpp:29-77 in KVFlux): causal, decode with
   scale, suffix alignment, GQA grouping, stable softmax, error cases.
2. Committed golden fixtures made by running the reference's compiled CPU
   code (tests/golden/make_golden.py).
3. Bit-exact agreement with the compiled reference on fresh seeded inputs,
   when oracle/_ref was built in this checkout.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from kvflux_b200 import workloads as w

GOLDEN = Path(__file__).resolve().parent / "golden"


def close(actual, expected, tol=1e-6):
    assert abs(float(actual) - expected) < tol, (actual, expected)


def test_known_answers_causal_and_decode():
    causal = oracle.reference_attention([0, 0, 0], [0, 0, 0], [2, 4, 8], (3, 3, 1, 1, 1))
    close(causal[0], 2.0)
    close(causal[1], 3.0)
    close(causal[2], 14.0 / 3.0)
    dec = oracle.reference_attention([2, 0, 0, 0], [0, 0, 0, 0, 1, 0, 0, 0], [0, 0, 0, 0, 10, 0, 0, 0],
                                     (1, 2, 1, 1, 4))
    close(dec[0], 10.0 * math.e / (1.0 + math.e))
    close(dec[1], 0.0)


def test_known_answers_suffix_gqa_stable():
    suffix = oracle.reference_attention([0, 0], [0, 0, 0, 0], [1, 2, 3, 4], (2, 4, 1, 1, 1))
    close(suffix[0], 2.0)
    close(suffix[1], 2.5)
    grouped = oracle.reference_attention([0, 0, 0, 0], [0, 0, 0, 0], [1, 10, 3, 30], (1, 2, 4, 2, 1))
    assert grouped.tolist() == [2, 2, 20, 20]
    stable = oracle.reference_attention([1e20], [1e20, 1e20], [2, 4], (1, 2, 1, 1, 1))
    close(stable[0], 3.0)
    assert oracle.reference_attention([], [], [], (0, 0, 1, 1, 1)).size == 0


@pytest.mark.parametrize("shape", [(2, 1, 1, 1, 1), (1, 1, 1, 0, 1), (1, 1, 3, 2, 1)])
def test_invalid_shapes_rejected(shape):
    lq, lkv, hq, hkv, hd = shape
    with pytest.raises(oracle.OracleError):
        oracle.reference_attention(np.ones(max(lq * hq * hd, 1)), np.ones(max(lkv * max(hkv, 1) * hd, 1)),
                                   np.ones(max(lkv * max(hkv, 1) * hd, 1)), shape)


def test_non_finite_rejected():
    with pytest.raises(oracle.OracleError):
        oracle.reference_attention([float("nan")], [1], [1], (1, 1, 1, 1, 1))


def _case(seed, lq, lkv, hq, hkv, hd):
    q = w.normal(seed, lq * hq * hd)
    k = w.normal(seed + 1, lkv * hkv * hd)
    v = w.normal(seed + 2, lkv * hkv * hd)
    return q, k, v


def test_golden_fixtures_match():
    data = json.loads((GOLDEN / "reference_attention.json").read_text())
    assert len(data["cases"]) >= 4
    for case in data["cases"]:
        q, k, v = _case(case["seed"], *case["shape"])
        got = oracle.reference_attention(q, k, v, tuple(case["shape"]))
        expect = np.array(case["output_f32_bits"], np.uint32).view(np.float32)
        assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), case["shape"]


def test_golden_input_generator_is_stable():
    data = json.loads((GOLDEN / "reference_attention.json").read_text())
    for case in data["cases"]:
        q, _, _ = _case(case["seed"], *case["shape"])
        assert np.array_equal(q[:4].view(np.uint32), np.array(case["q_head_f32_bits"], np.uint32))


@pytest.mark.skipif(oracle.ref() is None, reason="reference CPU library not built in this checkout")
@pytest.mark.parametrize("shape", [(1, 40, 8, 2, 64), (10, 10, 4, 2, 4), (3, 10, 4, 2, 4), (7, 33, 6, 3, 5),
                                   (1, 300, 32, 8, 128)])
def test_bit_exact_against_compiled_reference(shape):
    q, k, v = _case(0xABC + sum(shape), *shape)
    mine = oracle.reference_attention(q, k, v, shape)
    theirs = oracle.ref_reference_attention(q, k, v, shape)
    assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))


def test_write_gather_roundtrip_and_layout():
    # [27, 3, 91] recipe of tests/paged_kv_read_test.cpp:37-51 on a byte cache.
    heads, hd, bs, nb, elem = 2, 3, 16, 96, 2
    row = hd * elem
    k_cache = np.full(nb * heads * bs * row, 0xA5, np.uint8)
    v_cache = k_cache.copy()
    blocks = np.array([27, 3, 91], np.uint64)
    tokens = 40
    slots = np.array([blocks[t // bs] * bs + t % bs for t in range(tokens)], np.uint64)
    k_new = (0x1000 + np.arange(tokens * heads * hd)).astype(np.uint16).view(np.uint8)
    v_new = (0x3000 + np.arange(tokens * heads * hd)).astype(np.uint16).view(np.uint8)
    oracle.write(k_cache, v_cache, nb, heads, bs, row, k_new, v_new, slots)
    k_out, v_out = oracle.gather(k_cache, v_cache, nb, heads, bs, row, blocks, tokens)
    assert np.array_equal(k_out, k_new) and np.array_equal(v_out, v_new)
    # element (block 3, head 1, token 2, dim 1) sits at ((3*H+1)*bs+2)*hd+1
    idx = ((3 * heads + 1) * bs + 2) * hd + 1
    t = 16 + 2
    assert k_cache.view(np.uint16)[idx] == 0x1000 + (t * heads + 1) * hd + 1
    with pytest.raises(oracle.OracleError):
        oracle.write(k_cache, v_cache, nb, heads, bs, row, k_new[:row * heads], v_new[:row * heads],
                     np.array([nb * bs], np.uint64))


def test_decode_batch_composition_matches_reference_attention():
    # decode_batch == gather + reference_attention with one query per request.
    heads, hq, hd, bs, nb = 2, 4, 8, 4, 32
    bt_lens = [5, 9, 2]
    table = np.array([[0, 3, 2**64 - 1], [1, 4, 5], [2, 2**64 - 1, 2**64 - 1]], np.uint64)
    kc = w.encode(w.normal(7, nb * heads * bs * hd), "bfloat16")
    vc = w.encode(w.normal(8, nb * heads * bs * hd), "bfloat16")
    q = w.normal(9, 3 * hq * hd)
    out = oracle.decode_batch(kc, vc, 1, nb, heads, bs, hd, table, bt_lens, hq, q, threads=2)
    for r, L in enumerate(bt_lens):
        ko, vo = oracle.gather(kc.view(np.uint8), vc.view(np.uint8), nb, heads, bs, hd * 2, table[r], L)
        exp = oracle.reference_attention(q[r * hq * hd:(r + 1) * hq * hd], oracle.to_f32(ko, 1),
                                         oracle.to_f32(vo, 1), (1, L, hq, heads, hd))
        assert np.array_equal(out[r * hq * hd:(r + 1) * hq * hd], exp)

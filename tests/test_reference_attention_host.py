"""kvflux::v2::reference_attention as libkvflux_b200 exports it (a host
function, as in KVFlux's own library: src/v2/reference_attention.cpp:28-91).

Pinned three ways: the known answers of the reference's
tests/reference_attention_test.cpp:29-77 (causal, decode scale, suffix, GQA,
stable softmax, error types), bit-identical outputs to the oracle's
restatement on seeded shapes, and bit-identical outputs to the reference's
own compiled function when oracle/_ref was built."""
import math

import numpy as np
import pytest

import kvflux_b200 as kv
import oracle
from kvflux_b200 import workloads as w


def ra(q, k, v, shape):
    return np.array(kv.reference_attention(list(map(float, q)), list(map(float, k)), list(map(float, v)), *shape),
                    np.float32)


def close(a, b, tol=1e-6):
    assert abs(float(a) - b) < tol, (a, b)


def test_known_answers():
    causal = ra([0, 0, 0], [0, 0, 0], [2, 4, 8], (3, 3, 1, 1, 1))
    close(causal[0], 2.0)
    close(causal[1], 3.0)
    close(causal[2], 14.0 / 3.0)
    dec = ra([2, 0, 0, 0], [0, 0, 0, 0, 1, 0, 0, 0], [0, 0, 0, 0, 10, 0, 0, 0], (1, 2, 1, 1, 4))
    close(dec[0], 10.0 * math.e / (1.0 + math.e))
    close(dec[1], 0.0)
    suffix = ra([0, 0], [0, 0, 0, 0], [1, 2, 3, 4], (2, 4, 1, 1, 1))
    close(suffix[0], 2.0)
    close(suffix[1], 2.5)
    assert ra([0, 0, 0, 0], [0, 0, 0, 0], [1, 10, 3, 30], (1, 2, 4, 2, 1)).tolist() == [2, 2, 20, 20]
    close(ra([1e20], [1e20, 1e20], [2, 4], (1, 2, 1, 1, 1))[0], 3.0)
    assert ra([], [], [], (0, 0, 1, 1, 1)).size == 0


def test_error_types():
    with pytest.raises(ValueError):  # std::invalid_argument
        ra([1], [1], [1], (2, 1, 1, 1, 1))
    with pytest.raises(ValueError):
        ra([1], [1], [1], (1, 1, 1, 0, 1))
    with pytest.raises(ValueError):
        ra([1, 2, 3], [1], [1], (1, 1, 3, 2, 1))
    with pytest.raises(ValueError):
        ra([1], [1], [], (1, 1, 1, 1, 1))
    with pytest.raises(ValueError):
        ra([float("nan")], [1], [1], (1, 1, 1, 1, 1))
    with pytest.raises(OverflowError):  # std::overflow_error
        ra([], [], [], (1, 1, 2**64 - 1, 1, 2))


@pytest.mark.parametrize("shape", [(1, 40, 8, 2, 64), (7, 23, 4, 4, 16), (16, 16, 6, 2, 5), (3, 300, 32, 8, 128)])
def test_bit_identical_to_oracle_and_reference(shape):
    lq, lkv, hq, hkv, hd = shape
    seed = sum(shape)
    q = w.normal(seed, lq * hq * hd)
    k = w.normal(seed + 1, lkv * hkv * hd)
    v = w.normal(seed + 2, lkv * hkv * hd)
    got = np.array(kv.reference_attention(q.tolist(), k.tolist(), v.tolist(), *shape), np.float32)
    exp = oracle.reference_attention(q, k, v, shape)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    if oracle.ref() is not None:
        ref = oracle.ref_reference_attention(q, k, v, shape)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))

"""Seeded synthetic inputs of the paged-KV benchmark configurations: a
splitmix64 stream, Box-Muller N(0, 1) values, seeded permutations, and the
host's round-to-nearest-even float32 -> bfloat16 conversion; plus the
configurations' shapes. Plain numpy: importing this module loads no native
code, so a process that must not load the library (the benchmark's
reference arm) can use the same inputs.
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """n outputs of the splitmix64 generator started at `seed`."""
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int) -> np.ndarray:
    """Doubles in (0, 1) from the top 53 bits."""
    return ((splitmix64(seed, n) >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed: int, n: int) -> np.ndarray:
    """N(0, 1) float32 by Box-Muller on pairs of uniforms."""
    m = (n + 1) // 2
    u = uniform(seed, 2 * m)
    r = np.sqrt(-2.0 * np.log(u[0::2]))
    t = 2.0 * np.pi * u[1::2]
    out = np.empty(2 * m, np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return out[:n].astype(np.float32)


def uniform_ints(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi] (inclusive)."""
    return lo + (splitmix64(seed, n) % np.uint64(hi - lo + 1)).astype(np.int64)


def permutation(seed: int, items) -> np.ndarray:
    """Seeded shuffle of `items`: ordered by a splitmix64 key per position."""
    a = np.array(items, dtype=np.int64)
    return a[np.argsort(splitmix64(seed, len(a)), kind="stable")]


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (NaN kept quiet)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    nan = (b & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    rounded = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    out = rounded.astype(np.uint16)
    out[nan] = ((b[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return out


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def encode(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> raw cache elements (uint16 bits for 16-bit types, float32 otherwise)."""
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x)
    if dtype == "float16":
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
    return np.ascontiguousarray(x, np.float32)


def decode(raw: np.ndarray, dtype: str) -> np.ndarray:
    """Raw cache elements (bit patterns or floats) -> float32 values."""
    raw = np.asarray(raw)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(raw)
    if dtype == "float16":
        return raw.astype(np.uint16).view(np.float16).astype(np.float32)
    if raw.dtype in (np.uint32, np.int32):
        return raw.view(np.float32)
    return raw.astype(np.float32)


ELEM_BYTES = {"float16": 2, "bfloat16": 2, "float32": 4}
DTYPE_CODE = {"float16": 0, "bfloat16": 1, "float32": 2}


# Benchmark configurations (shapes from the reference's headline configs).
CONFIG3 = dict(batch=64, q_heads=32, kv_heads=8, head_size=128, block_size=16, min_len=512, max_len=8192,
               pool_pages=65536, dtype="bfloat16", seed=0xC0F3)
CONFIG5 = dict(batch=256, q_heads=64, kv_heads=8, head_size=128, block_size=16, min_len=4096, max_len=32768,
               dtype="bfloat16", seed=0xC0F5)
CONFIG2 = dict(sequences=64, new_tokens=4, prefill=8188, kv_heads=8, head_size=128, block_size=16,
               pool_pages=65536, dtype="bfloat16", seed=0xC0F2)
CONFIG4 = dict(sequences=8, tokens=4096, shared_prefix=2056, shared_group=4, q_heads=32, kv_heads=8, head_size=128,
               block_size=16, dtype="bfloat16", seed=0xC0F4)


def config_lengths(cfg: dict) -> np.ndarray:
    return uniform_ints(cfg["seed"], cfg["batch"], cfg["min_len"], cfg["max_len"])

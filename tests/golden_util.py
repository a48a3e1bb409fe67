"""Helpers shared by the tests: golden-vector loading and the reference's
seeded operand generators (crates/tiler-reference/tests/
contraction_profile_cells.rs:238-259), vectorised with numpy."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name="reference_vectors.json"):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def h(s) -> int:
    return int(s, 16)


def f(bits_hex) -> np.float32:
    return np.array([h(bits_hex)], dtype=np.uint32).view(np.float32)[0]


def fbits(values) -> np.ndarray:
    return np.array([h(v) for v in values], dtype=np.uint32).view(np.float32)


def fvals(values) -> np.ndarray:
    return np.array([np.nan if v == "nan" else v for v in values], dtype=np.float32)


def bits_of(a) -> list:
    return [int(b) for b in np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).ravel()]


_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """splitmix64 of contraction_profile_cells.rs:238-244 (wrapping u64)."""
    with np.errstate(over="ignore"):
        x = x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)
        z = x
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def prng_values(seed: int, count: int) -> np.ndarray:
    """prng_value of contraction_profile_cells.rs:247-259 for indices 0..count."""
    idx = np.arange(count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        b = splitmix64(np.uint64(seed) + idx * np.uint64(0x2545F4914F6CDD1D))
    field = ((b >> np.uint64(40)) & np.uint64(0xFFFFFF)).astype(np.int64)
    return ((field - 8388608).astype(np.float32) * np.float32(1.0 / 16777216.0)).astype(np.float32)


def seeded_uniform(seed: int, count: int, lo=-1.0, hi=1.0) -> np.ndarray:
    """U[lo,hi) from the same counter-based splitmix64 stream (24-bit grid)."""
    idx = np.arange(count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        b = splitmix64(np.uint64(seed) + idx * np.uint64(0x9E3779B97F4A7C15))
    u = ((b >> np.uint64(40)).astype(np.float64) / 16777216.0)
    return (lo + (hi - lo) * u).astype(np.float32)


def seeded_normal(seed: int, count: int, std=1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(count) * std).astype(np.float32)

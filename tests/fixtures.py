"""Deterministic input generators shared by the tests (numpy, vectorized).

splitmix64 is counter-based: draw t of a stream seeded with s is
mix(s + (t+1)*gamma), so whole streams vectorize (lib.rs:259-270).
"""
from __future__ import annotations

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)


def splitmix64_stream(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        t = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed) + t * GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def next_f64_stream(seed: int, n: int) -> np.ndarray:
    return (splitmix64_stream(seed, n) >> np.uint64(11)).astype(np.float64) / float(1 << 53)


def rand_rows(n: int, dim: int, seed: int, scale: float = 1.0) -> np.ndarray:
    """Gaussian-ish rows for GPU-vs-oracle parity (inputs only; both sides
    consume the same array, so no libm agreement is needed)."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, dim)) * scale).astype(np.float32)

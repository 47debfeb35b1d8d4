"""phyz-gpu's per-world random stream, vectorised over worlds.

world_seed is SplitMix64 of (seed, world) with xorshift's zero guard and
the stream is xorshift64 with uniforms from the top 53 bits and
Box-Muller normals — crates/phyz-gpu/src/policy_pipeline.rs:417-457
(`world_seed`, `KernelRng`). Each element of the arrays below is one
world's independent stream.
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def world_seed(seed: int, worlds) -> np.ndarray:
    w = np.asarray(worlds, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + np.uint64(0x9E3779B97F4A7C15) * (w + np.uint64(1))
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return np.where(z == 0, np.uint64(1), z)


class KernelRng:
    """Vector of xorshift64 streams (one per world)."""

    def __init__(self, seed: int, worlds):
        self.s = world_seed(seed, worlds).copy()

    def next_u64(self) -> np.ndarray:
        x = self.s
        with np.errstate(over="ignore"):
            x = x ^ ((x << np.uint64(13)) & _M64)
            x = x ^ (x >> np.uint64(7))
            x = x ^ ((x << np.uint64(17)) & _M64)
        self.s = x
        return x

    def uniform(self) -> np.ndarray:
        return (self.next_u64() >> np.uint64(11)).astype(np.float64) / float(1 << 53)

    def normal(self) -> np.ndarray:
        u1 = self.uniform()
        u2 = self.uniform()
        return np.sqrt(-2.0 * np.log(np.maximum(u1, 1e-300))) * np.cos(2.0 * np.pi * u2)

    def uniform_range(self, lo: float, hi: float) -> np.ndarray:
        return lo + (hi - lo) * self.uniform()

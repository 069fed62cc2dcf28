"""Seeded synthetic inputs shared by tests, bench and the oracle (no dataset is involved).

SplitMix64 with one seed per tensor: draw i of seed s is mix(s + (i+1) * 0x9E3779B97F4A7C15).
uniform[-1, 1) = ((u >> 40) * 2^-24) * 2 - 1 (exact in f32); normal(0, 1) is Box-Muller in
double on two draws, rounded once to f32.  The bytes are generated once and fed to both the
GPU and the CPU oracle, so only their statistics matter, not libm bit patterns.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, start: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, shape, chunk: int = 1 << 24) -> np.ndarray:
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        u = splitmix64(seed, e - s, s)
        out[s:e] = ((u >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)) * np.float32(2) - np.float32(1)
    return out.reshape(shape)


def normal(seed: int, shape, scale: float = 1.0, chunk: int = 1 << 23) -> np.ndarray:
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        u = splitmix64(seed, 2 * (e - s), 2 * s)
        u1 = ((u[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53  # (0, 1]
        u2 = (u[1::2] >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
        z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
        out[s:e] = (z * scale).astype(np.float32)
    return out.reshape(shape)

"""Seeded synthetic tensors (no datasets): splitmix64 streams, Box-Muller normals.

Shared by the tests, the bench and the CPU baseline so every arm sees the same
bytes. Value distributions follow the benchmark configurations: U[lo,hi) and
N(mean, std).
"""
import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix(seed, n):
    with np.errstate(over="ignore"):
        s = np.uint64(seed) + _GOLDEN * np.arange(1, n + 1, dtype=np.uint64)
        z = s
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def unit(seed, n):
    """n doubles in [0, 1) from the top 53 bits of a splitmix64 stream."""
    return (_splitmix(seed, n) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def uniform(seed, shape, lo=0.0, hi=1.0):
    n = int(np.prod(shape))
    return (lo + (hi - lo) * unit(seed, n)).reshape(shape)


def normal(seed, shape, mean=0.0, std=1.0):
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u = unit(seed, 2 * m)
    u1 = np.maximum(u[0::2], 1e-300)
    u2 = u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    z = np.empty(2 * m)
    z[0::2] = r * np.cos(t)
    z[1::2] = r * np.sin(t)
    return (mean + std * z[:n]).reshape(shape)


def sub_seed(seed, index):
    """Independent stream number `index` derived from a config seed."""
    return (int(seed) * 1_000_003 + int(index) * 7_919 + 1) & 0xFFFFFFFFFFFFFFFF

"""Seeded synthetic inputs for the benchmark workloads and the tests.

The reference publishes no datasets for this path; the workloads are
synthetic with the shapes and value distributions of the benchmark configs:
uniform bytes from a splitmix64 stream, and N(mu, sigma) from Box-Muller over
the same stream, rounded to the storage dtype with round-to-nearest-even.
Everything is deterministic in (seed, size), so the GPU and the CPU oracle
see identical bytes.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

CONFIG_SEED = 0x5EED0000


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n outputs of splitmix64 starting at stream position `offset`."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (np.arange(offset + 1, offset + n + 1, dtype=np.uint64) * _GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform_bytes(seed: int, n: int) -> np.ndarray:
    """n bytes, each uniform over 0..255."""
    words = splitmix64(seed, (n + 7) // 8)
    return words.view(np.uint8)[:n].copy()


def normal_f32(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
    """N(mu, sigma) float32 values by Box-Muller in float64: elements offset .. offset+n-1 of the
    stream (offset even; value 2j and 2j+1 come from stream words 2j and 2j+1)."""
    if offset % 2:
        raise ValueError("normal_f32: offset must be even")
    m = (n + 1) // 2
    w = splitmix64(seed, 2 * m, offset)
    u1 = ((w[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)  # (0, 1]
    u2 = (w[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m, dtype=np.float64)
    z[0::2] = r * np.cos(2.0 * np.pi * u2)
    z[1::2] = r * np.sin(2.0 * np.pi * u2)
    return (mu + sigma * z[:n]).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> BF16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def normal_bf16(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    return f32_to_bf16_bits(normal_f32(seed, n, mu, sigma))


def abs_normal_bf16(seed: int, n: int, sigma: float) -> np.ndarray:
    return f32_to_bf16_bits(np.abs(normal_f32(seed, n, 0.0, sigma)))


def normal_bf16_large(seed: int, n: int, mu: float = 0.0, sigma: float = 1.0, piece: int = 1 << 24,
                      threads: int = 8) -> np.ndarray:
    """normal_bf16(seed, n, mu, sigma), generated in pieces on a thread pool (the float64
    temporaries of one 500M-element call would need ~15 GB)."""
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty(n, dtype=np.uint16)

    def fill(a: int) -> None:
        b = min(n, a + piece)
        out[a:b] = f32_to_bf16_bits(normal_f32(seed, b - a, mu, sigma, offset=a))

    with ThreadPoolExecutor(max(1, threads)) as ex:
        list(ex.map(fill, range(0, n, piece)))
    return out

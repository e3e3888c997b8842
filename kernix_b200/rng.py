"""Seeded synthetic inputs: Kernix's SplitMix64 ``SeededRng`` (crates/kernix/src/
training.rs:132-171), vectorised with numpy.

``uniform`` matches ``SeededRng::uniform`` bit for bit: draw i uses the state
``seed + (i + 1) * 0x9e3779b97f4a7c15 (mod 2^64)``, the fraction
``(u >> 11) * 2^-53`` and ``low + (high - low) * fraction`` in f64, then rounds
to the element type.  ``normal`` is Box-Muller over consecutive uniform pairs
(u1, u2): ``sqrt(-2 ln(1 - u1)) * (cos 2 pi u2, sin 2 pi u2)``, scaled by ``std``.
"""
from __future__ import annotations

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
_CHUNK = 1 << 24


def _mix(x: np.ndarray) -> np.ndarray:
    x = (x ^ (x >> np.uint64(30))) * M1
    x = (x ^ (x >> np.uint64(27))) * M2
    return x ^ (x >> np.uint64(31))


def splitmix_block(seed: int, start: int, count: int) -> np.ndarray:
    """Outputs ``start .. start+count`` of the stream seeded with ``seed``."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 1, start + count + 1, dtype=np.uint64)
        return _mix(np.uint64(seed) + i * GAMMA)


def fractions(seed: int, start: int, count: int) -> np.ndarray:
    return (splitmix_block(seed, start, count) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def uniform(seed: int, n: int, low: float, high: float, dtype=np.float32, out: np.ndarray | None = None,
            start: int = 0) -> np.ndarray:
    """``SeededRng::new(seed).uniform([start + n], low, high)[start:]`` as a
    flat array (the stream is counter-based, so any window is direct)."""
    if out is None:
        out = np.empty(n, dtype=dtype)
    width = float(high) - float(low)
    for s in range(0, n, _CHUNK):
        c = min(_CHUNK, n - s)
        out[s:s + c] = float(low) + width * fractions(seed, start + s, c)
    return out


def normal(seed: int, n: int, std: float = 1.0, dtype=np.float32, out: np.ndarray | None = None,
           start: int = 0) -> np.ndarray:
    """Standard normals (times ``std``) by Box-Muller over the seeded stream;
    ``start`` (even: values come in pairs) skips that many values, so a
    window of the stream is generated directly."""
    if start % 2:
        raise ValueError("normal(): start must be even")
    if out is None:
        out = np.empty(n, dtype=dtype)
    pairs = (n + 1) // 2
    step = _CHUNK // 2
    for s in range(0, pairs, step):
        c = min(step, pairs - s)
        f = fractions(seed, start + 2 * s, 2 * c)
        u1, u2 = f[0::2], f[1::2]
        r = np.sqrt(-2.0 * np.log1p(-u1)) * float(std)
        z = np.empty(2 * c, dtype=np.float64)
        z[0::2] = r * np.cos(2.0 * np.pi * u2)
        z[1::2] = r * np.sin(2.0 * np.pi * u2)
        lo, hi = 2 * s, min(2 * s + 2 * c, n)
        out[lo:hi] = z[: hi - lo]
    return out

"""Vectorised mirror of lightx2v-core's `Rng` (crates/lightx2v-core/src/rng.rs:8-53):
SplitMix64 plus Box-Muller in f32, used to make BASELINE's seeded synthetic
inputs. The u64 stream is bit-identical to the reference; the f32 transcendental
calls are evaluated in f64 and rounded to f32; that equals glibc (which the C
oracle and the Rust reference call) for ~98.5% of samples and is within one
ulp of it for the rest. Parity tests feed the same arrays to both sides.
"""
from __future__ import annotations

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_PI = np.float32(np.pi)


def _u64_stream(seed: int, start: int, n: int) -> np.ndarray:
    """next_u64() outputs number start+1 .. start+n of Rng::new(seed) (rng.rs:20-26)."""
    with np.errstate(over="ignore"):
        i = np.arange(start + 2, start + n + 2, dtype=np.uint64)  # state = seed + G*(i)
        z = np.uint64(seed) + _GAMMA * i
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def next_f32(seed: int, n: int, start: int = 0) -> np.ndarray:
    """next_f32() (rng.rs:29-31): (u64 >> 40) / 2^24 in f32."""
    return ((_u64_stream(seed, start, n) >> np.uint64(40)).astype(np.float32) /
            np.float32(1 << 24)).astype(np.float32)


def uniform(seed: int, n: int, a: float) -> np.ndarray:
    """Rng::new(seed).uniform(n, a) (rng.rs:34-36)."""
    u = next_f32(seed, n)
    return ((u * np.float32(2.0) - np.float32(1.0)) * np.float32(a)).astype(np.float32)


def normal(seed: int, n: int, std: float = 1.0) -> np.ndarray:
    """std * Rng::new(seed).normal(n) (rng.rs:39-52)."""
    pairs = (n + 1) // 2
    u = next_f32(seed, 2 * pairs)
    u1 = np.maximum(u[0::2], np.float32(1e-7))
    u2 = u[1::2]
    # logf / cosf / sinf evaluated in f64 and rounded once to f32.
    ln = np.log(u1.astype(np.float64)).astype(np.float32)
    r = np.sqrt((np.float32(-2.0) * ln).astype(np.float32)).astype(np.float32)
    t = (np.float32(2.0) * _PI * u2).astype(np.float32)
    t64 = t.astype(np.float64)
    out = np.empty(2 * pairs, np.float32)
    out[0::2] = r * np.cos(t64).astype(np.float32)
    out[1::2] = r * np.sin(t64).astype(np.float32)
    out = out[:n]
    if std != 1.0:
        out = (out * np.float32(std)).astype(np.float32)
    return out

"""Seeded synthetic tensors for the benchmark workloads.

The reference has no normal sampler; its tests draw inputs from the LCG of
crates/tpt-infer-ops/src/dispatch.rs:274-282 (s = s*1664525 + 1013904223 mod
2^32, value = (s >> 8) / 2^24). ``uniform`` produces that stream; ``normal``
applies Box–Muller to consecutive pairs (u1 = 1 - (s1>>8)/2^24 in (0, 1],
u2 = (s2>>8)/2^24), evaluated in float64 and rounded once to float32.

The stream is generated with jump-ahead (s_{i+h} = A_h s_i + C_h) so that
hundreds of millions of values take well under a second in numpy.
"""
from __future__ import annotations

import numpy as np

_A, _C, _M = 1664525, 1013904223, 1 << 32


def _states(n: int, seed: int) -> np.ndarray:
    """s_1 .. s_n of the LCG started at `seed` (uint64 array holding u32 values)."""
    if n <= 0:
        return np.zeros(0, np.uint64)
    s = np.array([(seed * _A + _C) % _M], np.uint64)
    a_h, c_h = _A, _C  # jump of h = len(s) steps
    while s.size < n:
        nxt = (s * np.uint64(a_h) + np.uint64(c_h)) & np.uint64(_M - 1)
        s = np.concatenate([s, nxt])
        # compose the jump with itself: h -> 2h
        c_h = (a_h * c_h + c_h) % _M
        a_h = (a_h * a_h) % _M
    return s[:n]


def uniform(n: int, seed: int) -> np.ndarray:
    """U[0,1) from the reference's test LCG, float32."""
    s = _states(n, seed)
    return ((s >> np.uint64(8)).astype(np.float64) / 16777216.0).astype(np.float32)


def normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """N(mean, std), Box–Muller on consecutive LCG pairs, float32."""
    m = (n + 1) // 2
    s = _states(2 * m, seed) >> np.uint64(8)
    u1 = 1.0 - s[0::2].astype(np.float64) / 16777216.0
    u2 = s[1::2].astype(np.float64) / 16777216.0
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    out = np.empty(2 * m, np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return (float(mean) + float(std) * out[:n]).astype(np.float32)

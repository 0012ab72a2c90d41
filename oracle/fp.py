"""Floating-point helpers of the oracle: exact fused multiply-add, bf16 rounding, flush-to-zero.

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this.

``fma_f32`` computes round_to_f32(a*b + c) exactly: a*b of two f32 values is exact in f64 (48
significant bits), and the f64 sum s = a*b + c is off the exact sum by at most half an f64 ulp.
Rounding s to f32 can then only go wrong when s lands exactly on a midpoint between two f32
values while the exact sum is not there (double rounding); the TwoSum error term ``e`` tells which
side the exact sum lies on, and the tie is broken toward it.
"""

from __future__ import annotations

import numpy as np


def two_sum(a: np.ndarray, b: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """s, e with s = fl(a + b) and a + b = s + e exactly (Knuth's TwoSum)."""
    s = a + b
    bb = s - a
    e = (a - (s - bb)) + (b - bb)
    return s, e


def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """round_f32(a*b + c) exactly, elementwise, for f32 inputs."""
    a64 = np.asarray(a, np.float32).astype(np.float64)
    b64 = np.asarray(b, np.float32).astype(np.float64)
    c64 = np.asarray(c, np.float32).astype(np.float64)
    p = a64 * b64  # exact
    with np.errstate(invalid="ignore", over="ignore"):
        s, e = two_sum(p, c64)
        r = s.astype(np.float32)
        back = r.astype(np.float64)
        # the f32 neighbour of r on s's side, and the midpoint between them
        toward = np.where(s > back, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
        other = np.nextafter(r, toward)
        mid = (back + other.astype(np.float64)) * 0.5
        tie = (s == mid) & (e != 0) & np.isfinite(s) & (s != back)
        if np.any(tie):
            # the exact sum lies beyond the midpoint on e's side: pick that neighbour
            lo = np.minimum(r, other)
            hi = np.maximum(r, other)
            r = np.where(tie, np.where(e > 0, hi, lo), r)
    return r.astype(np.float32)


def fma_f64(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """round_f64(a*b + c) exactly (through Python fractions; for small test arrays only)."""
    from fractions import Fraction

    a, b, c = (np.asarray(x, np.float64) for x in np.broadcast_arrays(a, b, c))
    out = np.empty(a.shape, np.float64)
    for i in np.ndindex(a.shape):
        x, y, z = float(a[i]), float(b[i]), float(c[i])
        if not all(np.isfinite(v) for v in (x, y, z)):
            out[i] = x * y + z
            continue
        out[i] = float(Fraction(x) * Fraction(y) + Fraction(z))
    return out


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to the nearest bf16 (ties to even), returned as f32 values."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, np.float32))
    r = (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), r).astype(np.float32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def ftz32(x: np.ndarray) -> np.ndarray:
    """Flush f32 subnormals to signed zero (the .ftz behaviour)."""
    x = np.asarray(x, np.float32)
    tiny = np.abs(x) < np.float32(2.0**-126)
    return np.where(tiny, np.copysign(np.float32(0.0), x), x).astype(np.float32)


def rn32(x: np.ndarray) -> np.ndarray:
    """An f64 value rounded to f32 (nearest even)."""
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(x, np.float64).astype(np.float32)

"""The oracle pinned against the reference's known answers, and its exact arithmetic."""

from __future__ import annotations

import math
from fractions import Fraction

import numpy as np
import pytest
from conftest import oracle_run, reference_inputs, shipped

from oracle.fp import bf16_round, fma_f32
from ptxgen import problems


def _softmax(x: np.ndarray) -> np.ndarray:
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(-1, keepdims=True)


# The reference's problem semantics and tolerances (tools/expressions_open.py:39-85,
# tools/expressions_closed.py:137-142, 367-369), restated.
KNOWN = {
    "p02_scale_shift": (lambda x: x * np.float32(2.0) + np.float32(1.0), 1e-6, 1e-6),
    "r02_big_sum": (lambda x: x.astype(np.float64).sum(), 1e-3, 1e-3),
    "m01_matmul_512": (lambda a, b: a.astype(np.float64) @ b.astype(np.float64), 1e-3, 1e-3),
    "a01_attention": (lambda q, kt, v: _softmax(q.astype(np.float64) @ kt / 8.0) @ v, 1e-3,
                      1e-4),
    "a03_noscale": (lambda q, kt, v: _softmax(q.astype(np.float64) @ kt) @ v, 1e-3, 1e-4),
}


@pytest.mark.parametrize("name", sorted(KNOWN))
def test_oracle_matches_reference_semantics(name: str) -> None:
    graph, meta = shipped(name)
    ins = reference_inputs(meta)
    out = next(iter(oracle_run(graph, meta, ins).values()))
    fn, rtol, atol = KNOWN[name]
    ref = fn(*[ins[n].astype(np.float64) for n in meta["graph_inputs"]])
    np.testing.assert_allclose(out.astype(np.float64).reshape(np.shape(ref)), ref, rtol=rtol,
                               atol=atol)


def test_oracle_p02_is_one_fma_per_element() -> None:
    """p02's x*2+1 is one fused multiply-add in the lowering, so the oracle rounds once."""
    graph, meta = shipped("p02_scale_shift")
    ins = reference_inputs(meta)
    out = next(iter(oracle_run(graph, meta, ins).values()))
    want = fma_f32(ins["x"], np.float32(2.0), np.float32(1.0))
    assert np.array_equal(out.reshape(-1), want)


def _exact_fma(a: float, b: float, c: float) -> np.float32:
    """round_f32(a*b + c) through exact rationals and a round-to-nearest-even search."""
    x = Fraction(a) * Fraction(b) + Fraction(c)
    f = np.float32(float(x))
    lo, hi = (np.nextafter(f, np.float32(-np.inf)), f) if Fraction(float(f)) > x else \
        (f, np.nextafter(f, np.float32(np.inf)))
    dl, dh = abs(Fraction(float(lo)) - x), abs(Fraction(float(hi)) - x)
    if dl != dh:
        return lo if dl < dh else hi
    return lo if int(np.float32(lo).view(np.uint32)) % 2 == 0 else hi


def test_fma_f32_exact() -> None:
    rng = np.random.default_rng(3)
    a = rng.standard_normal(4000).astype(np.float32)
    b = rng.standard_normal(4000).astype(np.float32)
    c = rng.standard_normal(4000).astype(np.float32)
    # adversarial: products whose low bits meet c at an f32 midpoint
    a[:1000] = np.float32(1.0) + np.float32(2.0**-12) * rng.integers(0, 4096, 1000)
    b[:1000] = np.float32(1.0) + np.float32(2.0**-12) * rng.integers(0, 4096, 1000)
    c[:1000] = -(a[:1000].astype(np.float64) * b[:1000]).astype(np.float32)
    got = fma_f32(a, b, c)
    for i in range(0, 4000, 7):
        want = _exact_fma(float(a[i]), float(b[i]), float(c[i]))
        assert got[i] == want or (np.isnan(got[i]) and np.isnan(want)), i


def test_fma_f32_double_rounding_case() -> None:
    """A sum that lands on an f32 midpoint in f64 but lies just above it exactly."""
    a = np.float32(1.0 + 2.0**-23)
    b = np.float32(1.0 + 2.0**-23)
    c = np.float32(2.0**-24)  # a*b = 1 + 2^-22 + 2^-46; + 2^-24 sits near a midpoint
    assert fma_f32(np.array([a]), np.array([b]), np.array([c]))[0] == _exact_fma(
        float(a), float(b), float(c))


def test_generated_configs_match_formulas() -> None:
    from oracle.fp import bf16_bits_to_f32

    s = problems.pointwise_add(3000)
    ins = reference_inputs(s.meta)
    out = oracle_run(s.graph, s.meta, ins)["add"]
    assert np.array_equal(out, ins["x"] + ins["y"])

    s = problems.gelu_chain(32, 256)
    ins = reference_inputs(s.meta)
    out = bf16_bits_to_f32(oracle_run(s.graph, s.meta, ins)["mul_1"])
    a, b = s.kernel["args"][0]["data"][0], s.kernel["args"][1]["data"][0]
    u = a * bf16_bits_to_f32(ins["x"]).astype(np.float64) + b
    ref = 0.5 * u * (1 + np.tanh(math.sqrt(2 / math.pi) * (u + 0.044715 * u**3))) * ins["s"][:, None]
    np.testing.assert_allclose(out, bf16_round(ref.astype(np.float32)), rtol=2**-7, atol=2**-12)

    s = problems.row_softmax(32, 512)
    ins = reference_inputs(s.meta)
    out = oracle_run(s.graph, s.meta, ins)["softmax"]
    np.testing.assert_allclose(out, _softmax(ins["x"].astype(np.float64)), rtol=1e-3, atol=1e-5)

    s = problems.full_sum(1 << 18, 128, 8)
    ins = reference_inputs(s.meta)
    out = oracle_run(s.graph, s.meta, ins)["sum_1"]
    np.testing.assert_allclose(out[0], ins["x"].astype(np.float64).sum(), rtol=1e-5)

    s = problems.matmul(128, 256, 128)
    ins = reference_inputs(s.meta)
    out = oracle_run(s.graph, s.meta, ins)["matmul"]
    ref = bf16_bits_to_f32(ins["x0"]).astype(np.float64) @ bf16_bits_to_f32(ins["x1"])
    np.testing.assert_allclose(out, ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())

"""Fast f32 math functions, as a fast-math build computes them (reference ``ptxgen/fastmath.py``).

Each is a short sequence over the hardware approximations ``ex2.approx``, ``lg2.approx``,
``rcp.approx``, ``sin.approx`` and ``cos.approx`` (each good to about 2 ulp), built from the
mathematical identity named in its docstring:

* ``exp(x) = 2^(x * log2 e)``, ``log(x) = log2(x) * ln 2``;
* ``tanh(x) = 1 - 2 / (e^(2x) + 1)``: it saturates exactly to +-1 at both ends, unlike the
  ``tanh.approx`` instruction, which is only good to about 2^-11;
* ``sigmoid(x) = 1 / (1 + e^-x)``;
* ``erf`` by Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26
  (|error| < 1.5e-7);
* ``pow(x, y) = 2^(y * log2|x|)`` with C ``powf``'s sign rules.

The products feeding ``ex2``/``lg2`` round to nearest like every other multiply here, so the
NumPy oracle can bound each function's error from those roundings plus the instruction's.
"""

from __future__ import annotations

import math
from collections.abc import Callable

from .dtypes import literal
from .ptx import Kernel

ONE, ZERO = literal(1.0, "f32"), literal(0.0, "f32")
LOG2E = math.log2(math.e)
LN2 = math.log(2.0)
# Abramowitz & Stegun 7.1.26: erf(x) ~ 1 - (a1 t + ... + a5 t^5) e^(-x^2), t = 1 / (1 + p x)
AS_P = 0.3275911
AS_A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def _f(k: Kernel, op: str, *srcs: str) -> str:
    return k.pure(op, "f32", *srcs)


def _p(k: Kernel, op: str, *srcs: str) -> str:
    return k.pure(op, "pred", *srcs)


def exp2(k: Kernel, x: str) -> str:
    return _f(k, "ex2.approx.ftz.f32", x)


def exp(k: Kernel, x: str) -> str:
    return exp2(k, _f(k, "mul.rn.f32", x, literal(LOG2E, "f32")))


def log2(k: Kernel, x: str) -> str:
    return _f(k, "lg2.approx.ftz.f32", x)


def log(k: Kernel, x: str) -> str:
    return _f(k, "mul.rn.f32", log2(k, x), literal(LN2, "f32"))


def tanh(k: Kernel, x: str) -> str:
    """1 - 2 / (e^(2x) + 1)."""
    e = exp2(k, _f(k, "mul.rn.f32", x, literal(2.0 * LOG2E, "f32")))
    r = _f(k, "rcp.approx.ftz.f32", _f(k, "add.rn.f32", e, ONE))
    return _f(k, "fma.rn.f32", r, literal(-2.0, "f32"), ONE)


def sigmoid(k: Kernel, x: str) -> str:
    """1 / (1 + e^-x)."""
    e = exp2(k, _f(k, "mul.rn.f32", x, literal(-LOG2E, "f32")))
    return _f(k, "rcp.approx.ftz.f32", _f(k, "add.rn.f32", e, ONE))


def erf(k: Kernel, x: str) -> str:
    """Abramowitz & Stegun 7.1.26, evaluated by Horner's rule, signed like x."""
    ax = _f(k, "abs.f32", x)
    t = _f(k, "rcp.approx.ftz.f32", _f(k, "fma.rn.f32", ax, literal(AS_P, "f32"), ONE))
    poly = literal(AS_A[4], "f32")
    for c in (*reversed(AS_A[:4]), 0.0):
        poly = _f(k, "fma.rn.f32", t, poly, literal(c, "f32"))
    e = exp(k, _f(k, "neg.f32", _f(k, "mul.rn.f32", ax, ax)))
    return _f(k, "copysign.f32", x, _f(k, "fma.rn.f32", _f(k, "neg.f32", poly), e, ONE))


def sin(k: Kernel, x: str) -> str:
    return _f(k, "sin.approx.ftz.f32", x)


def cos(k: Kernel, x: str) -> str:
    return _f(k, "cos.approx.ftz.f32", x)


def pow_(k: Kernel, x: str, y: str) -> str:
    """2^(y log2|x|); x < 0 gives -r for an odd integer y, r for an even one, nan for a
    fraction; y == 0 gives 1."""
    r = exp2(k, _f(k, "mul.rn.f32", log2(k, _f(k, "abs.f32", x)), y))
    whole = _p(k, "setp.eq.f32", _f(k, "cvt.rni.f32.f32", y), y)
    half = _f(k, "mul.rn.f32", y, literal(0.5, "f32"))
    odd = _p(k, "and.pred", whole, _p(k, "setp.neu.f32", _f(k, "cvt.rni.f32.f32", half), half))
    neg = _p(k, "setp.lt.f32", x, ZERO)
    r = _f(k, "selp.f32", _f(k, "neg.f32", r), r, _p(k, "and.pred", neg, odd))
    r = _f(k, "selp.f32", r, literal(math.nan, "f32"),
           _p(k, "or.pred", whole, _p(k, "not.pred", neg)))
    return _f(k, "selp.f32", ONE, r, _p(k, "setp.eq.f32", y, ZERO))


F32_FUNCS: dict[str, Callable[..., str]] = {
    "exp": exp, "exp2": exp2, "log": log, "log2": log2, "tanh": tanh, "sigmoid": sigmoid,
    "erf": erf, "sin": sin, "cos": cos, "pow": pow_,
}

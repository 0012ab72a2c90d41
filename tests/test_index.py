"""The index algebra (``ptxgen.index``) against integer arithmetic, on the CPU.

Random affine indices over registers whose values lie in known ranges and are known multiples of
known divisors are divided and reduced by constants through ``div``/``mod`` and compared through
``compare``. The instructions the algebra emitted are then evaluated as unsigned 32-bit PTX on
random register values that respect those facts, and every folded quotient, remainder and decided
comparison must equal what Python's integers give. This pins the folds that make an index free:
terms a divisor absorbs, remainders that provably never carry, constants that never carry past a
divisibility, and compares decided from ranges.
"""

from __future__ import annotations

import operator

import numpy as np
import pytest

from ptxgen import index
from ptxgen.index import Aff
from ptxgen.ptx import Kernel

M32 = 0xFFFFFFFF
CMP = {"lt": operator.lt, "le": operator.le, "gt": operator.gt, "ge": operator.ge,
       "eq": operator.eq, "ne": operator.ne}
PY_CMP = {"<": operator.lt, "<=": operator.le, ">": operator.gt, ">=": operator.ge,
          "==": operator.eq, "!=": operator.ne}


def _s32(v: int) -> int:
    v &= M32
    return v - (1 << 32) if v >> 31 else v


def run(k: Kernel, env: dict[str, int]) -> dict[str, int]:
    """Evaluate the kernel's emitted index instructions as u32 PTX."""
    val = dict(env)

    def get(s: str) -> int:
        return val[s] if s.startswith("%") else int(s)

    for ins in k.body:
        op, src = ins.op, [get(s) for s in ins.src]
        base = op.split(".")[0]
        if base == "mov":
            out = src[0]
        elif base == "add":
            out = src[0] + src[1]
        elif base == "sub":
            out = src[0] - src[1]
        elif op == "mad.lo.u32":
            out = src[0] * src[1] + src[2]
        elif op in ("mul.lo.u32",):
            out = src[0] * src[1]
        elif base == "shl":
            out = src[0] << src[1]
        elif base == "shr":
            out = (src[0] & M32) >> src[1]
        elif base == "and":
            out = src[0] & src[1]
        elif base == "div":
            out = (src[0] & M32) // (src[1] & M32)
        elif base == "rem":
            out = (src[0] & M32) % (src[1] & M32)
        elif base == "min":
            out = min(src[0] & M32, src[1] & M32)
        elif base == "setp":
            out = int(CMP[op.split(".")[1]](_s32(src[0]), _s32(src[1])))
        elif base == "selp":
            out = src[0] if src[2] else src[1]
        else:
            raise AssertionError(f"unexpected index instruction {op}")
        val[ins.dst[0]] = out & M32 if base != "setp" else out
    return val


def value(x: Aff, val: dict[str, int]) -> int:
    return sum(c * val[r] for r, c in x.terms.items()) + x.const


@pytest.mark.parametrize("seed", range(40))
def test_divmod_and_compare_match_integers(seed: int) -> None:
    rng = np.random.default_rng(seed)
    k = Kernel("t", [], 256)
    regs = {}
    for i in range(int(rng.integers(1, 4))):
        mult = int(rng.choice([1, 2, 4, 8, 16]))
        hi = int(rng.integers(1, 5000)) * mult
        regs[k.reg("u32", rng=(0, hi), mult=mult)] = (hi, mult)
    coeffs = [1, 2, 3, 4, 7, 8, 16, 64, 100, 1024]
    x = Aff({r: int(rng.choice(coeffs)) for r in regs}, int(rng.integers(0, 100)))
    y = Aff({r: int(rng.choice(coeffs)) for r in regs if rng.random() < 0.7},
            int(rng.integers(0, 20000)))
    checks = []
    for m in (1, 2, 3, 4, 7, 8, 16, 64, 100, 1024, 8192):
        q, r = index.div(k, x, m), index.mod(k, x, m)
        checks.append(("div", m, q))
        checks.append(("mod", m, r))
        # a split index re-joined, and a division of a remainder, as flattened indices do
        checks.append(("join", m, q * m + r))
        checks.append(("modmod", m, index.mod(k, r, max(1, m // 2))))
    decided = {}
    for op in PY_CMP:
        c = index.compare(k, op, x, y)
        decided[op] = c
    for _ in range(200):
        env = {r: int(rng.integers(0, hi // mult + 1)) * mult for r, (hi, mult) in regs.items()}
        val = run(k, env)
        xv, yv = value(x, env), value(y, env)
        for kind, m, form in checks:
            got = value(form, val)
            want = {"div": xv // m, "mod": xv % m, "join": xv,
                    "modmod": (xv % m) % max(1, m // 2)}[kind]
            assert got == want, (kind, m, form, env)
        for op, c in decided.items():
            truth = PY_CMP[op](xv, yv)
            assert (c if isinstance(c, bool) else bool(val[c])) == truth, (op, x, y, env)


def test_divmod_exhaustive_small_ranges() -> None:
    """Every boundary: one register over [0, hi] (a multiple of ``mult``) for every small hi,
    coefficient, constant and divisor, each value of the range checked."""
    for mult in (1, 2, 3, 4):
        for hi in range(0, 21):
            if hi % mult:
                continue
            for c in range(1, 6):
                for const in range(0, 5):
                    for m in (*range(1, 10), 16):
                        k = Kernel("t", [], 32)
                        r = k.reg("u32", rng=(0, hi), mult=mult)
                        x = Aff({r: c}, const)
                        q, rem = index.div(k, x, m), index.mod(k, x, m)
                        for v in range(0, hi + 1, mult):
                            val = run(k, {r: v})
                            xv = c * v + const
                            assert value(q, val) == xv // m, (mult, hi, c, const, m, v)
                            assert value(rem, val) == xv % m, (mult, hi, c, const, m, v)

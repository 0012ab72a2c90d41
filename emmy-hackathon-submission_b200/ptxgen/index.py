"""Unsigned 32-bit index arithmetic as affine forms over registers.

An index value is an ``Aff``: ``sum(coeff * reg) + const``. Adding, subtracting and scaling by a
constant stay affine and emit nothing, so the constant part of an index only ever reaches the
immediate offset of a load (``[%rd4+12]``), and the unrolled copies of a loop share one address
register. Each index register carries two facts in the kernel: its value range
(``Kernel.ranges``) and a number its value is known to be a multiple of (``Kernel.mult``).

They drive the folding of ``/`` and ``%`` by a constant ``m``:

* terms whose coefficient ``m`` divides go straight into the quotient;
* if the remaining part ``r`` provably stays in ``[0, m)``, the division is free (``r`` is the
  remainder, the quotient gets nothing from it);
* if ``r = g*X + c`` with ``g`` dividing ``m`` and ``0 <= c < g``, the constant can never carry
  (``g*X mod m`` is a multiple of ``g``, at most ``m - g``), so ``r / m == g*X / m`` and the ``c``
  copies of an unrolled group share one division; this is what keeps ``(a0*8 + j) / 8192`` a
  single shift for all eight ``j``;
* otherwise a power of two becomes ``shr``/``and`` and anything else ``div``/``rem``, and the pair is
  recorded so a later ``m*(X/m) + X%m`` re-joins into ``X``.

The divisibility facts also give every address its alignment, which the vectorizer needs.
Indices are never negative (Emmy's guarantee), so unsigned shifts are exact.
"""

from __future__ import annotations

import math

from .ptx import Kernel, Range

_CMP = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}


class Aff:
    """An affine integer form ``sum(coeff * register) + const``; immutable."""

    __slots__ = ("const", "terms")

    def __init__(self, terms: dict[str, int] | None = None, const: int = 0):
        self.terms = {r: c for r, c in sorted((terms or {}).items()) if c}
        self.const = int(const)

    @classmethod
    def of(cls, reg: str) -> Aff:
        return cls({reg: 1})

    @classmethod
    def k(cls, value: int) -> Aff:
        return cls(const=value)

    @property
    def is_const(self) -> bool:
        return not self.terms

    def var_part(self) -> Aff:
        return Aff(self.terms)

    def __add__(self, other: Aff | int) -> Aff:
        other = other if isinstance(other, Aff) else Aff(const=other)
        terms = dict(self.terms)
        for r, c in other.terms.items():
            terms[r] = terms.get(r, 0) + c
        return Aff(terms, self.const + other.const)

    def __sub__(self, other: Aff | int) -> Aff:
        return self + (other * -1 if isinstance(other, Aff) else -other)

    def __mul__(self, k: int) -> Aff:
        return Aff({r: c * k for r, c in self.terms.items()}, self.const * k)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, Aff) and self.terms == other.terms and self.const == other.const

    def __hash__(self) -> int:
        return hash((tuple(self.terms.items()), self.const))

    def __repr__(self) -> str:
        parts = [f"{c}*{r}" for r, c in self.terms.items()] + [str(self.const)]
        return "Aff(" + " + ".join(parts) + ")"

    def range(self, ranges: dict[str, Range]) -> Range | None:
        lo = hi = self.const
        for r, c in self.terms.items():
            if r not in ranges:
                return None
            a, b = ranges[r][0] * c, ranges[r][1] * c
            lo, hi = lo + min(a, b), hi + max(a, b)
        return lo, hi

    def var_mult(self, mult: dict[str, int]) -> int:
        """A number the variable part is always a multiple of (0 when there is none)."""
        g = 0
        for r, c in self.terms.items():
            g = math.gcd(g, abs(c) * mult.get(r, 1))
        return g


def operand(k: Kernel, x: Aff) -> str:
    """An immediate or a register holding x."""
    return str(x.const & 0xFFFFFFFF) if x.is_const else reg_of(k, x)


def _note(k: Kernel, x: Aff) -> tuple[Range | None, int | None]:
    rng = x.range(k.ranges)
    g = math.gcd(x.var_mult(k.mult), x.const) if x.terms else x.const
    return rng, (g or None)


def reg_of(k: Kernel, x: Aff) -> str:
    """A register holding x (u32)."""
    x = _rejoin(k, x)
    if x.is_const:
        return k.pure("mov.u32", "u32", str(x.const & 0xFFFFFFFF), rng=(x.const, x.const),
                      mult=x.const or None)
    if x.const:
        rng, mult = _note(k, x)
        return k.pure("add.u32", "u32", reg_of(k, x.var_part()), str(x.const & 0xFFFFFFFF),
                      rng=rng, mult=mult)
    (first, c), *rest = x.terms.items()
    acc = first if c == 1 else _mul_imm(k, first, c)
    acc_form = Aff({first: c})
    for reg, c in rest:
        acc_form = acc_form + Aff({reg: c})
        rng, mult = _note(k, acc_form)
        if c == 1:
            acc = k.pure("add.u32", "u32", acc, reg, rng=rng, mult=mult)
        elif c == -1:
            acc = k.pure("sub.u32", "u32", acc, reg, rng=rng, mult=mult)
        else:
            acc = k.pure("mad.lo.u32", "u32", reg, str(c & 0xFFFFFFFF), acc, rng=rng, mult=mult)
    return acc


def _mul_imm(k: Kernel, reg: str, c: int) -> str:
    rng, mult = _note(k, Aff({reg: c}))
    if c > 0 and not c & (c - 1):
        return k.pure("shl.b32", "u32", reg, str(c.bit_length() - 1), rng=rng, mult=mult)
    return k.pure("mul.lo.u32", "u32", reg, str(c & 0xFFFFFFFF), rng=rng, mult=mult)


def _rejoin(k: Kernel, x: Aff) -> Aff:
    """Fold ``c*m*(X / m) + c*(X % m)`` back into ``c*X``, as a split flat index re-joins."""
    for q, cq in x.terms.items():
        fact = k.divmods.get(q)
        if fact is None or fact[0] != "div":
            continue
        _, src, m = fact
        for r, cr in x.terms.items():
            if k.divmods.get(r) == ("mod", src, m) and cq == cr * m:
                return _rejoin(k, x - Aff({q: cq, r: cr}) + Aff.of(src) * cr)
    return x


def mul(k: Kernel, a: Aff, b: Aff) -> Aff:
    if a.is_const or b.is_const:
        return b * a.const if a.is_const else a * b.const
    ra, rb = a.range(k.ranges), b.range(k.ranges)
    rng = None
    if ra and rb:
        ends = [x * y for x in ra for y in rb]
        rng = (min(ends), max(ends))
    return Aff.of(k.pure("mul.lo.u32", "u32", reg_of(k, a), reg_of(k, b), rng=rng))


def div(k: Kernel, a: Aff, m: Aff | int) -> Aff:
    """a / m (floor) for m > 0."""
    return _divmod(k, a, m, "div")


def mod(k: Kernel, a: Aff, m: Aff | int) -> Aff:
    """a % m for m > 0."""
    return _divmod(k, a, m, "mod")


def _divmod(k: Kernel, a: Aff, m: Aff | int, kind: str) -> Aff:
    is_div = kind == "div"
    if isinstance(m, Aff) and not m.is_const:  # a divisor known only at run time
        op = "div.u32" if is_div else "rem.u32"
        return Aff.of(k.pure(op, "u32", operand(k, a), reg_of(k, m)))
    m = m.const if isinstance(m, Aff) else m
    if m <= 0:
        raise ValueError(f"index {kind} by {m}")
    if a.is_const:
        return Aff(const=a.const // m if is_div else a.const % m)
    if m == 1:
        return a if is_div else Aff()

    # a = m*q + rest, q collecting the terms m divides: only rest needs a division
    q = Aff({r: c // m for r, c in a.terms.items() if c % m == 0}, a.const // m)
    rest = Aff({r: c for r, c in a.terms.items() if c % m}, a.const % m)
    rng = rest.range(k.ranges)
    if rng is None or rng[0] < 0:  # the ops are unsigned: divide all of a
        q, rest, rng = Aff(), a, a.range(k.ranges)
    if rest.is_const:
        return q + rest.const // m if is_div else Aff(const=rest.const % m)
    if rng is not None and 0 <= rng[0] and rng[1] < m:  # rest never carries into q
        return q if is_div else rest

    # rest = g*X + c with g | m and 0 <= c < g: c never carries, divide g*X alone
    g = rest.var_mult(k.mult)
    if g > 1 and m % g == 0 and 0 < rest.const < g:
        c = rest.const
        base = rest - c
        if is_div:
            return q + _divmod(k, base, m, "div")
        return _divmod(k, base, m, "mod") + c
    # g*X / m == X / (m/g) when every term is a multiple of g through its coefficient
    if g > 1 and m % g == 0 and rest.const == 0 and all(c % g == 0 for c in rest.terms.values()):
        inner = Aff({r: c // g for r, c in rest.terms.items()})
        sub = _divmod(k, inner, m // g, kind)
        return q + sub if is_div else sub * g

    x = reg_of(k, rest)
    pow2 = not m & (m - 1)
    if is_div:
        op, imm = ("shr.u32", m.bit_length() - 1) if pow2 else ("div.u32", m)
        out_rng = (rng[0] // m, rng[1] // m) if rng else None
        out_mult = None
    else:
        op, imm = ("and.b32", m - 1) if pow2 else ("rem.u32", m)
        out_rng = (0, min(m - 1, rng[1])) if rng else (0, m - 1)
        out_mult = math.gcd(rest.var_mult(k.mult), m) or None
    r = k.pure(op, "u32", x, str(imm), rng=out_rng, mult=out_mult)
    k.divmods[r] = (kind, x, m)
    return q + Aff.of(r) if is_div else Aff.of(r)


def minimum(k: Kernel, a: Aff, b: Aff) -> Aff:
    if a.is_const and b.is_const:
        return Aff(const=min(a.const, b.const))
    ra, rb = a.range(k.ranges), b.range(k.ranges)
    if ra and rb:
        if ra[1] <= rb[0]:
            return a
        if rb[1] <= ra[0]:
            return b
    rng = (min(ra[0], rb[0]), min(ra[1], rb[1])) if ra and rb else None
    return Aff.of(k.pure("min.u32", "u32", reg_of(k, a), operand(k, b), rng=rng))


def decide(k: Kernel, op: str, a: Aff, b: Aff) -> bool | None:
    """``a op b`` when the ranges decide it, else None."""
    rng = (a - b).range(k.ranges)
    if rng is None:
        return None
    lo, hi = rng
    holds = {"<": hi < 0, "<=": hi <= 0, ">": lo > 0, ">=": lo >= 0, "==": lo == hi == 0,
             "!=": lo > 0 or hi < 0}
    fails = {"<": lo >= 0, "<=": lo > 0, ">": hi <= 0, ">=": hi < 0, "==": lo > 0 or hi < 0,
             "!=": lo == hi == 0}
    if holds[op]:
        return True
    if fails[op]:
        return False
    return None


def compare(k: Kernel, op: str, a: Aff, b: Aff) -> str | bool:
    """A predicate register for ``a op b``, or a bool when the ranges decide it. The compare is
    ``var(a - b) op -const(a - b)`` in signed 32-bit arithmetic, which stays exact while every
    index value is below 2^31 (the Tile limit), even when one side dips below zero."""
    known = decide(k, op, a, b)
    if known is not None:
        return known
    d = a - b
    return k.pure(f"setp.{_CMP[op]}.s32", "pred", reg_of(k, d.var_part()), str(-d.const))


def select(k: Kernel, pred: str, a: Aff, b: Aff) -> Aff:
    ra, rb = a.range(k.ranges), b.range(k.ranges)
    rng = (min(ra[0], rb[0]), max(ra[1], rb[1])) if ra and rb else None
    return Aff.of(k.pure("selp.b32", "u32", operand(k, a), operand(k, b), pred, rng=rng))

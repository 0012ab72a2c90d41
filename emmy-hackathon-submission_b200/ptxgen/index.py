"""Unsigned 32-bit index arithmetic: affine forms over registers, and what the kernel knows about
each register.

An index value is an ``Aff``: a constant plus integer multiples of u32 registers. ``Aff`` is pure
algebra: every sum, difference and scaling is one linear combination (``Aff.combine``), which
emits nothing. So the constant part of an index only ever reaches the immediate offset of an
access (``[%rd4+12]``), and the unrolled copies of a loop share one address register.

What an index can be is the kernel's knowledge of its registers (``Facts``): for each register a
value range (``Kernel.ranges``) and a number it is a multiple of (``Kernel.mult``). ``Facts``
answers the questions the folding asks of a whole form: its interval, and the largest number its
variable part is always a multiple of.

Division and remainder by a constant ``m`` first split the dividend into ``m * quot + rest``, where
``quot`` takes every term (and the part of the constant) that ``m`` divides exactly. Only ``rest``
can need an instruction, and an ordered list of rewrite rules (``_RULES``) tries to avoid that:

* ``rest`` a constant: the answer is a constant;
* ``rest`` confined to ``[0, m)``: it never carries, so the quotient is ``quot`` and the
  remainder ``rest``;
* ``rest = X + c`` where every value of ``X`` is a multiple of some ``g`` that divides ``m`` and
  ``0 < c < g``: ``X mod m`` is at most ``m - g``, so ``c`` can never carry and ``X`` is divided
  alone (the eight copies ``(a0*8 + j) / 8192`` of an unrolled group share one shift);
* ``rest = g * Y`` term by term with ``g`` dividing ``m``: divide ``Y`` by ``m / g`` instead.

What no rule folds becomes ``shr``/``and`` for a power of two and ``div``/``rem`` otherwise, and
the kernel records the (quotient, remainder) origin of that register, so a later
``c*m*(X / m) + c*(X % m)`` is recognised and re-joined into ``c*X`` before it is materialised.

Compares are decided, where the facts allow, by the signs the difference of the two sides can
take. Indices are never negative (Emmy's guarantee), so unsigned shifts are exact; a compare is
made in signed 32-bit arithmetic, exact while every index is below 2^31 (the Tile limit).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable, Mapping
from dataclasses import dataclass

from .ptx import Kernel, Range

U32 = 0xFFFFFFFF


class Aff:
    """``const + sum(coeff * register)``; immutable and hashable. ``terms`` maps each register
    to its nonzero coefficient, in register-name order."""

    __slots__ = ("const", "terms")

    def __init__(self, terms: Mapping[str, int] | None = None, const: int = 0):
        pairs = sorted((terms or {}).items())
        self.terms = {reg: c for reg, c in pairs if c}
        self.const = int(const)

    @staticmethod
    def combine(*parts: tuple[Aff | int, int]) -> Aff:
        """``sum(weight * part)`` over (part, weight) pairs; a part may be a plain integer."""
        acc: dict[str, int] = {}
        c0 = 0
        for part, w in parts:
            if isinstance(part, int):
                c0 += w * part
                continue
            c0 += w * part.const
            for reg, c in part.terms.items():
                acc[reg] = acc.get(reg, 0) + w * c
        return Aff(acc, c0)

    @classmethod
    def of(cls, reg: str) -> Aff:
        """The register itself."""
        return cls({reg: 1})

    @classmethod
    def k(cls, value: int) -> Aff:
        """A constant."""
        return cls(None, value)

    @property
    def is_const(self) -> bool:
        return len(self.terms) == 0

    def var_part(self) -> Aff:
        """The form without its constant."""
        return Aff(self.terms)

    def __add__(self, other: Aff | int) -> Aff:
        return Aff.combine((self, 1), (other, 1))

    def __sub__(self, other: Aff | int) -> Aff:
        return Aff.combine((self, 1), (other, -1))

    def __mul__(self, factor: int) -> Aff:
        return Aff.combine((self, factor))

    def __eq__(self, other: object) -> bool:
        if not isinstance(other, Aff):
            return False
        return (self.const, self.terms) == (other.const, other.terms)

    def __hash__(self) -> int:
        return hash((self.const, *self.terms.items()))

    def __repr__(self) -> str:
        body = " + ".join([*(f"{c}*{reg}" for reg, c in self.terms.items()), str(self.const)])
        return f"Aff({body})"

    # Questions about the form's values, given per-register facts (see ``Facts``).
    def range(self, ranges: Mapping[str, Range]) -> Range | None:
        """The interval the form's value lies in, or None when a register's range is unknown."""
        return Facts(ranges, {}).interval(self)

    def var_mult(self, mult: Mapping[str, int]) -> int:
        """A number the variable part is always a multiple of (0 for a constant form)."""
        return Facts({}, mult).stride(self)


@dataclass(frozen=True)
class Facts:
    """What is known of each u32 index register: its value range and a divisor of its value."""

    ranges: Mapping[str, Range]
    mult: Mapping[str, int]

    @classmethod
    def of(cls, k: Kernel) -> Facts:
        return cls(k.ranges, k.mult)

    def interval(self, x: Aff) -> Range | None:
        lo = hi = x.const
        for reg, c in x.terms.items():
            known = self.ranges.get(reg)
            if known is None:
                return None
            ends = (known[0] * c, known[1] * c)
            lo += min(ends)
            hi += max(ends)
        return lo, hi

    def stride(self, x: Aff) -> int:
        """The gcd over terms of |coefficient| times the register's own known divisor."""
        return math.gcd(*(abs(c) * self.mult.get(reg, 1) for reg, c in x.terms.items())) \
            if x.terms else 0

    def divisor(self, x: Aff) -> int | None:
        """A number every value of the whole form (constant included) is a multiple of."""
        g = math.gcd(self.stride(x), x.const) if x.terms else x.const
        return g or None

    def note(self, x: Aff) -> dict:
        """The facts a register holding ``x`` is created with."""
        return {"rng": self.interval(x), "mult": self.divisor(x)}


# --- materialising a form into a register --------------------------------------------------


def operand(k: Kernel, x: Aff) -> str:
    """An instruction operand for x: an immediate when it is constant, else a register."""
    if x.is_const:
        return str(x.const & U32)
    return reg_of(k, x)


def reg_of(k: Kernel, x: Aff) -> str:
    """A register holding x (u32). Split quotient/remainder pairs are re-joined first; then the
    variable part is built term by term (the first term scaled, each further one added,
    subtracted, or multiply-added), and the constant is added last."""
    x = _rejoin(k, x)
    facts = Facts.of(k)
    if x.is_const:
        return k.pure("mov.u32", "u32", str(x.const & U32), rng=(x.const, x.const),
                      mult=x.const or None)
    if x.const:
        base = reg_of(k, x.var_part())
        return k.pure("add.u32", "u32", base, str(x.const & U32), **facts.note(x))
    pairs = list(x.terms.items())
    first, c0 = pairs[0]
    acc = first if c0 == 1 else _scaled(k, first, c0)
    built = Aff({first: c0})
    for reg, c in pairs[1:]:
        built = Aff.combine((built, 1), (Aff({reg: c}), 1))
        acc = _accumulate(k, acc, reg, c, Facts.of(k).note(built))
    return acc


def _scaled(k: Kernel, reg: str, c: int) -> str:
    """``c * reg``: a shift for a positive power of two, else a multiply."""
    facts = Facts.of(k).note(Aff({reg: c}))
    if c > 0 and c & (c - 1) == 0:
        return k.pure("shl.b32", "u32", reg, str(c.bit_length() - 1), **facts)
    return k.pure("mul.lo.u32", "u32", reg, str(c & U32), **facts)


def _accumulate(k: Kernel, acc: str, reg: str, c: int, facts: dict) -> str:
    """``acc + c * reg`` in one instruction."""
    if c == 1:
        return k.pure("add.u32", "u32", acc, reg, **facts)
    if c == -1:
        return k.pure("sub.u32", "u32", acc, reg, **facts)
    return k.pure("mad.lo.u32", "u32", reg, str(c & U32), acc, **facts)


def _rejoin(k: Kernel, x: Aff) -> Aff:
    """Replace each ``c*m*(X / m) + c*(X % m)`` in x, both halves from one recorded split of
    register X, by ``c*X`` (until no such pair is left)."""
    while True:
        pair = _split_pair(k, x)
        if pair is None:
            return x
        q, r, src, weight = pair
        x = Aff.combine((x, 1), (Aff({q: x.terms[q], r: x.terms[r]}), -1),
                        (Aff.of(src), weight))


def _split_pair(k: Kernel, x: Aff) -> tuple[str, str, str, int] | None:
    """A quotient register and a remainder register of x from the same split of one source,
    with coefficients in the ratio m : 1; returned with the source and the remainder's
    coefficient."""
    quotients = {reg: k.divmods[reg] for reg in x.terms
                 if k.divmods.get(reg, ("",))[0] == "div"}
    for q, (_, src, m) in quotients.items():
        for r, cr in x.terms.items():
            if k.divmods.get(r) == ("mod", src, m) and x.terms[q] == cr * m:
                return q, r, src, cr
    return None


# --- multiply, divide, remainder, minimum -------------------------------------------------


def mul(k: Kernel, a: Aff, b: Aff) -> Aff:
    """a * b: a scaling when either side is constant, else one ``mul.lo``."""
    if b.is_const:
        return a * b.const
    if a.is_const:
        return b * a.const
    facts = Facts.of(k)
    ra, rb = facts.interval(a), facts.interval(b)
    rng = None
    if ra is not None and rb is not None:
        products = [p * q for p in ra for q in rb]
        rng = (min(products), max(products))
    return Aff.of(k.pure("mul.lo.u32", "u32", reg_of(k, a), reg_of(k, b), rng=rng))


def div(k: Kernel, a: Aff, m: Aff | int) -> Aff:
    """a / m (floor) for m > 0."""
    return _divmod(k, a, m, "div")


def mod(k: Kernel, a: Aff, m: Aff | int) -> Aff:
    """a % m for m > 0."""
    return _divmod(k, a, m, "mod")


@dataclass(frozen=True)
class _Split:
    """A dividend as ``m * quot + rest``: only ``rest`` can need a division. ``rng`` is the
    interval of ``rest``."""

    m: int
    quot: Aff
    rest: Aff
    rng: Range | None
    want_div: bool

    def answer(self, q_part: Aff, r_part: Aff) -> Aff:
        """The result, given rest's own quotient and remainder by m."""
        return self.quot + q_part if self.want_div else r_part


def _split(k: Kernel, a: Aff, m: int, want_div: bool) -> _Split:
    exact = {reg: c // m for reg, c in a.terms.items() if c % m == 0}
    left = {reg: c for reg, c in a.terms.items() if c % m}
    quot, rest = Aff(exact, a.const // m), Aff(left, a.const % m)
    rng = Facts.of(k).interval(rest)
    if rng is None or rng[0] < 0:
        # the instructions are unsigned: a possibly negative rest cannot be divided on its own
        quot, rest, rng = Aff(), a, Facts.of(k).interval(a)
    return _Split(m, quot, rest, rng, want_div)


def _rule_constant(k: Kernel, s: _Split) -> Aff | None:
    if not s.rest.is_const:
        return None
    return s.answer(Aff.k(s.rest.const // s.m), Aff.k(s.rest.const % s.m))


def _rule_no_carry(k: Kernel, s: _Split) -> Aff | None:
    if s.rng is None or not 0 <= s.rng[0] <= s.rng[1] < s.m:
        return None
    return s.answer(Aff(), s.rest)


def _rule_small_offset(k: Kernel, s: _Split) -> Aff | None:
    g = Facts.of(k).stride(s.rest)
    c = s.rest.const
    if g <= 1 or s.m % g or not 0 < c < g:
        return None
    base = s.rest - c
    if s.want_div:
        return s.quot + _divmod(k, base, s.m, "div")
    return _divmod(k, base, s.m, "mod") + c


def _rule_common_factor(k: Kernel, s: _Split) -> Aff | None:
    g = Facts.of(k).stride(s.rest)
    if g <= 1 or s.m % g or s.rest.const or any(c % g for c in s.rest.terms.values()):
        return None
    inner = Aff({reg: c // g for reg, c in s.rest.terms.items()})
    part = _divmod(k, inner, s.m // g, "div" if s.want_div else "mod")
    return s.quot + part if s.want_div else part * g


_RULES: tuple[Callable[[Kernel, _Split], Aff | None], ...] = (
    _rule_constant, _rule_no_carry, _rule_small_offset, _rule_common_factor)


def _divmod(k: Kernel, a: Aff, m: Aff | int, kind: str) -> Aff:
    want_div = kind == "div"
    if isinstance(m, Aff):
        if not m.is_const:  # a divisor known only at run time
            opcode = "div.u32" if want_div else "rem.u32"
            return Aff.of(k.pure(opcode, "u32", operand(k, a), reg_of(k, m)))
        m = m.const
    if m <= 0:
        raise ValueError(f"index {kind} by {m}")
    if a.is_const:
        return Aff.k(a.const // m if want_div else a.const % m)
    if m == 1:
        return a if want_div else Aff()
    s = _split(k, a, m, want_div)
    for rule in _RULES:
        folded = rule(k, s)
        if folded is not None:
            return folded
    return _emit_divmod(k, s)


def _emit_divmod(k: Kernel, s: _Split) -> Aff:
    """One instruction dividing ``rest``: shr/and for a power of two, div/rem otherwise; the
    result register remembers its origin for ``_rejoin``."""
    src = reg_of(k, s.rest)
    m, rng = s.m, s.rng
    shift = m.bit_length() - 1 if m & (m - 1) == 0 else None
    if s.want_div:
        opcode, imm = ("shr.u32", shift) if shift is not None else ("div.u32", m)
        facts = {"rng": (rng[0] // m, rng[1] // m) if rng else None, "mult": None}
    else:
        opcode, imm = ("and.b32", m - 1) if shift is not None else ("rem.u32", m)
        hi = min(m - 1, rng[1]) if rng else m - 1
        facts = {"rng": (0, hi), "mult": math.gcd(Facts.of(k).stride(s.rest), m) or None}
    out = k.pure(opcode, "u32", src, str(imm), **facts)
    kind = "div" if s.want_div else "mod"
    k.divmods[out] = (kind, src, m)
    return s.answer(Aff.of(out), Aff.of(out))


def minimum(k: Kernel, a: Aff, b: Aff) -> Aff:
    """min(a, b): one side when the facts order them, else ``min.u32``."""
    if a.is_const and b.is_const:
        return Aff.k(min(a.const, b.const))
    facts = Facts.of(k)
    ra, rb = facts.interval(a), facts.interval(b)
    if ra is not None and rb is not None:
        if ra[1] <= rb[0]:
            return a
        if rb[1] <= ra[0]:
            return b
        rng: Range | None = (min(ra[0], rb[0]), min(ra[1], rb[1]))
    else:
        rng = None
    return Aff.of(k.pure("min.u32", "u32", reg_of(k, a), operand(k, b), rng=rng))


# --- compares and selects ------------------------------------------------------------------

_SETP = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}
# for each compare, its truth when a - b is negative, zero, positive
_TRUTH = {"<": (True, False, False), "<=": (True, True, False), ">": (False, False, True),
          ">=": (False, True, True), "==": (False, True, False), "!=": (True, False, True)}


def _signs(rng: Range) -> Iterable[int]:
    """Which of negative (0), zero (1), positive (2) a value in ``rng`` can be."""
    lo, hi = rng
    return [i for i, possible in enumerate((lo < 0, lo <= 0 <= hi, hi > 0)) if possible]


def decide(k: Kernel, op: str, a: Aff, b: Aff) -> bool | None:
    """``a op b`` when every value the facts allow gives the same answer, else None."""
    rng = Facts.of(k).interval(a - b)
    if rng is None:
        return None
    outcomes = {_TRUTH[op][sign] for sign in _signs(rng)}
    return outcomes.pop() if len(outcomes) == 1 else None


def compare(k: Kernel, op: str, a: Aff, b: Aff) -> str | bool:
    """A predicate register for ``a op b``, or a bool when the facts decide it. The register
    compares ``var(a - b) op -const(a - b)`` as signed 32-bit values, which stays exact while
    every index is below 2^31, even when one side dips below zero."""
    known = decide(k, op, a, b)
    if known is not None:
        return known
    d = a - b
    return k.pure(f"setp.{_SETP[op]}.s32", "pred", reg_of(k, d.var_part()), str(-d.const))


def select(k: Kernel, pred: str, a: Aff, b: Aff) -> Aff:
    """``pred ? a : b`` as a register, its range the hull of both sides'."""
    facts = Facts.of(k)
    ra, rb = facts.interval(a), facts.interval(b)
    rng = (min(ra[0], rb[0]), max(ra[1], rb[1])) if ra and rb else None
    return Aff.of(k.pure("selp.b32", "u32", operand(k, a), operand(k, b), pred, rng=rng))

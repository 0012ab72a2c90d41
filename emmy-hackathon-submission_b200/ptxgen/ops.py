"""Data values and the instruction sequences of Emmy's elementwise ops.

A data value is a ``Val``: a register and its Emmy dtype (a bool is a predicate register).

Every elementwise op is one row of ``SPECS``: its arity, its mnemonic on float registers, its
mnemonic on integer registers, how its operands are formed (``x, x`` for a square, ``x, 0`` for a
relu, the ``cvt.rXi`` form of a rounding), and on which float types it computes natively. Where an
op computes is Emmy's dtype rule (reference ``ptxgen/ops.py:173-192``), stated by itself in
``compute_type``: natively for f16's simple ops, for integer ops over integers and for f64; every
other op converts its inputs to f32, computes, and converts the result back once. One emitter,
``_emit``, turns a row into instructions for the chosen type; the f32 fast-math functions come
from ``fastmath``.

Float arithmetic rounds to nearest and says so: ``add.rn``, ``sub.rn`` and ``mul.rn`` carry the
modifier explicitly, which stops ptxas from contracting a multiply and an add on its own. The
only contraction is the one this backend makes, ``fma_operands``: an f32/f64 add whose operand is
a still-reusable multiply of the same type becomes one ``fma.rn``. So every rounding in the
emitted kernel is decided here, and the NumPy oracle can reproduce results bit for bit.

``--no_fusion`` keeps the reference's meaning (``compile.py:8``, ``ptxgen/ops.py:56-71``): this
backend fuses nothing, and writes ``add``, ``sub`` and ``mul`` without a rounding modifier, so
ptxas may still contract a multiply and an add by itself. The flag then measures this backend's
fusion against ptxas's, as the reference's op-fusion tables do, and each product rounds once or
not at all, as ptxas chooses.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass

from . import fastmath
from .dtypes import FLOAT_TYPES, is_float, is_int, literal, move_type, reg_type, size
from .ptx import Kernel

# Other spellings of Emmy's op names.
ALIASES = {"sub": "subtract", "mul": "multiply", "div": "divide", "max": "maximum",
           "min": "minimum", "sum": "add", "prod": "multiply", "amax": "maximum",
           "amin": "minimum", "true_divide": "divide", "neg": "negative", "pow_": "pow",
           "power": "pow", "rsqrt_": "rsqrt"}
# Ops an accumulator folds with -> (float mnemonic, integer mnemonic).
ACCUM = {"add": ("add.rn", "add"), "subtract": ("sub.rn", "sub"), "multiply": ("mul.rn", "mul.lo"),
         "divide": ("div.rn", "div"), "maximum": ("max", "max"), "minimum": ("min", "min")}
COMPARE = {"equal": "eq", "not_equal": "ne", "greater": "gt", "less": "lt",
           "greater_equal": "ge", "less_equal": "le"}
CMP_SYMBOL = {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}


def canonical(name: str) -> str:
    return ALIASES.get(name, name)


@dataclass(frozen=True)
class Val:
    """A data value: the register holding it and its Emmy dtype."""

    reg: str
    dtype: str


@dataclass(frozen=True)
class Spec:
    """How one elementwise op lowers.

    ``fop`` is its mnemonic on float registers (None: no float instruction; f32 may still have
    a fast-math function), ``iop`` its integer mnemonic and whether that takes a ``.b<bits>``
    type. ``operands`` forms the instruction's sources: ``"args"`` as given, ``"self"`` the one
    argument twice, ``"zero"`` the argument and 0. ``rounding`` ops are ``cvt.<mode>.t.t``.
    ``natives`` lists the float types that compute the op natively besides f32."""

    arity: int
    fop: str | None = None
    iop: tuple[str, bool] | None = None
    operands: str = "args"
    rounding: bool = False
    natives: frozenset[str] = frozenset({"f16", "f64"})


_F64_ONLY = frozenset({"f64"})
SPECS: dict[str, Spec] = {
    "add": Spec(2, "add.rn", ("add", False)),
    "subtract": Spec(2, "sub.rn", ("sub", False)),
    "multiply": Spec(2, "mul.rn", ("mul.lo", False)),
    "divide": Spec(2, "div.rn", natives=_F64_ONLY),
    "maximum": Spec(2, "max", ("max", False)),
    "minimum": Spec(2, "min", ("min", False)),
    "pow": Spec(2),
    "relu": Spec(1, "max", operands="zero"),
    "negative": Spec(1, "neg"),
    "abs": Spec(1, "abs"),
    "square": Spec(1, "mul.rn", operands="self", natives=_F64_ONLY),
    "reciprocal": Spec(1, "rcp.rn", natives=_F64_ONLY),
    "sqrt": Spec(1, "sqrt.rn", natives=_F64_ONLY),
    "rsqrt": Spec(1, "rsqrt.approx", natives=frozenset()),
    "floor": Spec(1, "cvt.rmi", rounding=True, natives=_F64_ONLY),
    "ceil": Spec(1, "cvt.rpi", rounding=True, natives=_F64_ONLY),
    "trunc": Spec(1, "cvt.rzi", rounding=True, natives=_F64_ONLY),
    "round": Spec(1, "cvt.rni", rounding=True, natives=_F64_ONLY),
    "floor_divide": Spec(2, iop=("div", False)),
    "remainder": Spec(2, iop=("rem", False)),
    "mod": Spec(2, iop=("rem", False)),
    "left_shift": Spec(2, iop=("shl", True)),
    "right_shift": Spec(2, iop=("shr", False)),
    "bitwise_and": Spec(2, iop=("and", True)),
    "bitwise_or": Spec(2, iop=("or", True)),
    "bitwise_xor": Spec(2, iop=("xor", True)),
}
for _name in fastmath.F32_FUNCS:
    SPECS.setdefault(_name, Spec(1))


def const(k: Kernel, value: float, typ: str) -> str:
    """A register holding ``value`` (16-bit float arithmetic takes no immediates)."""
    return k.pure(f"mov.{move_type(typ)}", typ, literal(value, typ))


# The forms ``--no_fusion`` writes: no rounding modifier, so ptxas may contract them.
UNFUSED = {"add.rn": "add", "sub.rn": "sub", "mul.rn": "mul"}


def arith(k: Kernel, m: str) -> str:
    """Mnemonic ``m`` as this kernel writes it: ``add.rn``/``sub.rn``/``mul.rn`` lose their
    rounding modifier with fusion off; everything else is unchanged."""
    return UNFUSED.get(m, m) if k.no_fusion else m


def fma_operands(k: Kernel, t: str, a: str, b: str) -> tuple[str, str, str] | None:
    """``(x, y, c)`` when ``a + b`` is ``x * y + c`` for a multiply of type ``t`` that is still
    reusable here, trying ``a`` as the product first; never with fusion off, and only for
    f32/f64."""
    if k.no_fusion or t not in ("f32", "f64"):
        return None
    wanted = f"mul.rn.{t}"
    for prod, addend in ((a, b), (b, a)):
        key = k.definition(prod)  # (mnemonic, x, y), plus a uniquifier with CSE off
        if key is not None and key[0] == wanted:
            return key[1], key[2], addend
    return None


# --- where an op computes, and the instructions ---------------------------------------------


def compute_type(name: str, arg_dtypes: Sequence[str], dtype: str) -> str:
    """The Emmy dtype op ``name`` computes in for result ``dtype``: f16's simple ops over f16
    arguments, integer ops over integer arguments and f64 ops compute natively; everything else
    in f32."""
    spec = SPECS.get(name)
    if spec is not None:
        typ = reg_type(dtype)
        if typ == "f16":
            same = all(d == dtype for d in arg_dtypes)
            if same and spec.fop is not None and "f16" in spec.natives:
                return dtype
        elif is_int(dtype):
            if spec.iop is not None and all(is_int(d) for d in arg_dtypes):
                return dtype
        elif dtype == "f64" and spec.fop is not None and "f64" in spec.natives:
            return dtype
    return "f32"


def _emit(k: Kernel, name: str, spec: Spec, typ: str, srcs: list[str]) -> str:
    """The instructions of op ``name`` on registers of PTX type ``typ``."""
    if spec.iop is not None and typ not in FLOAT_TYPES:
        mnemonic, bit_typed = spec.iop
        if mnemonic in ("shl", "shr") and size(typ) != 4:
            raise NotImplementedError(f"{typ} op {name}: shift of a non-32-bit integer")
        suffix = f"b{size(typ) * 8}" if bit_typed else typ
        return k.pure(f"{mnemonic}.{suffix}", typ, *srcs)
    if spec.rounding:
        return k.pure(f"{spec.fop}.{typ}.{typ}", typ, *srcs)
    if name == "add" and (fused := fma_operands(k, typ, *srcs)) is not None:
        return k.pure(f"fma.rn.{typ}", typ, *fused)
    if spec.operands == "self":
        srcs = [srcs[0], srcs[0]]
    elif spec.operands == "zero":
        zero = const(k, 0.0, typ) if typ == "f16" else literal(0.0, typ)
        srcs = [srcs[0], zero]
    return k.pure(f"{arith(k, spec.fop)}.{typ}", typ, *srcs)


def _operation(name: str, at: str) -> Callable[[Kernel, list[str]], str] | None:
    """How op ``name`` runs on registers of Emmy dtype ``at``, or None if it cannot."""
    spec = SPECS.get(name)
    typ = reg_type(at)
    if at == "f32" and spec is not None and spec.fop is None and name in fastmath.F32_FUNCS:
        return lambda k, srcs: fastmath.F32_FUNCS[name](k, *srcs)
    if spec is None:
        return None
    if typ in FLOAT_TYPES and spec.fop is None:
        return None
    if typ not in FLOAT_TYPES and spec.iop is None:
        return None
    return lambda k, srcs: _emit(k, name, spec, typ, srcs)


def apply(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    """name(args) at result ``dtype`` under Emmy's rule: native where Emmy computes there,
    otherwise in f32, converted once."""
    name = canonical(name)
    at = compute_type(name, [a.dtype for a in args], dtype)
    run = _operation(name, at)
    if run is None:
        raise NotImplementedError(f"{at} op {name}")
    want = SPECS[name].arity
    if len(args) != want:
        raise ValueError(f"{at} op {name} takes {want} argument(s), got {len(args)}")
    srcs = [convert(k, a, at).reg for a in args]
    return convert(k, Val(run(k, srcs), at), dtype)


# --- conversions -----------------------------------------------------------------------------


def _cvt_modifier(src: str, dst: str) -> str:
    """C's rules: a float result rounds to nearest (widening a float is exact and takes none),
    a float to integer truncates, integer to integer needs none."""
    if src in FLOAT_TYPES and dst in FLOAT_TYPES:
        return "" if size(dst) > size(src) else ".rn"
    if dst in FLOAT_TYPES:
        return ".rn"
    return ".rzi" if src in FLOAT_TYPES else ""


def cvt(k: Kernel, x: str, src: str, dst: str) -> str:
    """Register ``x`` from PTX type ``src`` to ``dst``: two floats neither of which is f32 meet
    in f32 (exact for the 16-bit ones); bf16 -> f32 is a register pack."""
    if src == dst:
        return x
    both_float = src in FLOAT_TYPES and dst in FLOAT_TYPES
    if both_float and src != "f32" and dst != "f32":
        return cvt(k, cvt(k, x, src, "f32"), "f32", dst)
    if (src, dst) == ("bf16", "f32"):
        # exact: the bf16 bits are the upper half of the f32 bits. A register pack runs on the
        # integer pipe, where cvt.f32.bf16 would take a slot of the XU pipe that ex2/rcp need.
        low = k.pure("mov.b16", "b16", "0")
        return k.pure("mov.b32", "f32", f"{{{low}, {x}}}")
    return k.pure(f"cvt{_cvt_modifier(src, dst)}.{dst}.{src}", dst, x)


def _bool_to(k: Kernel, p: str, dtype: str) -> Val:
    """A predicate as 1 / 0 of ``dtype`` (16-bit floats take registers, not immediates)."""
    typ = reg_type(dtype)
    if typ in ("f16", "bf16"):
        one = const(k, 1.0, typ)
        zero = const(k, 0.0, typ)
    else:
        one, zero = literal(1.0, typ), literal(0.0, typ)
    return select(k, p, one, zero, dtype)


def _to_bool(k: Kernel, v: Val) -> Val:
    """Nonzero as true: compared in f32 for floats, in i32 for integers."""
    wide = convert(k, v, "f32" if is_float(v.dtype) else "i32")
    typ = reg_type(wide.dtype)
    return Val(k.pure(f"setp.ne.{typ}", "pred", wide.reg, literal(0.0, typ)), "bool")


def convert(k: Kernel, v: Val, dtype: str) -> Val:
    """``v`` as Emmy dtype ``dtype``: rounding conversions, bool as 1/0, nonzero as true."""
    if v.dtype == dtype:
        return v
    if v.dtype == "bool":
        return _bool_to(k, v.reg, dtype)
    if dtype == "bool":
        return _to_bool(k, v)
    return Val(cvt(k, v.reg, reg_type(v.dtype), reg_type(dtype)), dtype)


def select(k: Kernel, cond: str, a: str, b: str, dtype: str) -> Val:
    """``cond ? a : b``; bools by predicate logic (a selp has no predicate form)."""
    typ = reg_type(dtype)
    if typ != "pred":
        return Val(k.pure(f"selp.{move_type(typ)}", typ, a, b, cond), dtype)
    take_a = k.pure("and.pred", "pred", cond, a)
    take_b = k.pure("and.pred", "pred", k.pure("not.pred", "pred", cond), b)
    return Val(k.pure("or.pred", "pred", take_a, take_b), dtype)


# --- Assign ----------------------------------------------------------------------------------


_FLOAT_RANK = ("f16", "bf16", "f32", "f64")


def promote(name: str, dtypes: Sequence[str]) -> str:
    """The result dtype of an op with no explicit dtype (Emmy's promotion, as restated for the
    cases Kernel IR leaves implicit: combine programs, whose arguments share one dtype)."""
    if name in COMPARE:
        return "bool"
    distinct = list(dict.fromkeys(dtypes))
    if len(distinct) == 1:
        return distinct[0]
    floats = {d for d in distinct if d != "bool" and is_float(d)}
    if floats == {"f16", "bf16"}:
        return "f32"
    if floats:
        return max(floats, key=_FLOAT_RANK.index)
    ints = [d for d in distinct if d != "bool"]
    return max(ints, key=size) if ints else "bool"


def _compare(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    x, y = (convert(k, v, "f32").reg for v in args)
    return convert(k, Val(k.pure(f"setp.{COMPARE[name]}.f32", "pred", x, y), "bool"), dtype)


def _where(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    cond = convert(k, args[0], "bool").reg
    x, y = (convert(k, v, dtype).reg for v in args[1:])
    return select(k, cond, x, y, dtype)


def _logic(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    preds = [convert(k, v, "bool").reg for v in args]
    opcode = {"logical_and": "and.pred", "logical_or": "or.pred", "logical_not": "not.pred"}
    return convert(k, Val(k.pure(opcode[name], "pred", *preds), "bool"), dtype)


def _copy(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    return convert(k, args[0], dtype)


_STRUCTURAL: dict[str, Callable[[Kernel, str, Sequence[Val], str], Val]] = {
    **dict.fromkeys(COMPARE, _compare), "where": _where,
    **dict.fromkeys(("logical_and", "logical_or", "logical_not"), _logic),
    **dict.fromkeys(("copy", "pad", "identity", "cast", "to"), _copy),
}


def assign(k: Kernel, name: str, dtype: str | None, args: Sequence[Val]) -> Val:
    """The value of an Assign of op ``name`` over ``args``: compares (in f32), selects, logic
    and copies by their own rules, every other op through ``apply``."""
    name = canonical(name)
    if dtype is None:
        dtype = promote(name, [v.dtype for v in args])
    handler = _STRUCTURAL.get(name)
    if handler is not None:
        return handler(k, name, args, dtype)
    return apply(k, name, args, dtype)


# --- shuffles --------------------------------------------------------------------------------


def shfl(k: Kernel, x: str, typ: str, mode: str, lane: str | int, clamp: int, mask: str) -> str:
    """One ``shfl.sync`` of ``x``. The instruction moves 32-bit words: a 64-bit value moves as
    its two halves, a 16-bit value widened to a word, a predicate as a 0/1 word."""

    def move(word: str, word_typ: str = "u32") -> str:
        out = k.reg(word_typ)
        k.emit(f"shfl.sync.{mode}.b32", (out,), (word, str(lane), str(clamp), mask))
        return out

    if typ == "pred":
        word = move(k.pure("selp.u32", "u32", "1", "0", x))
        return k.pure("setp.ne.u32", "pred", word, "0")
    if size(typ) == 4:
        return move(x, typ)
    out = k.reg(typ)  # the result's register, filled from the moved words
    if size(typ) == 8:
        halves = (k.reg("u32"), k.reg("u32"))
        k.emit("mov.b64", (f"{{{halves[0]}, {halves[1]}}}",), (x,))
        moved = [move(h) for h in halves]
        k.emit("mov.b64", (out,), (f"{{{moved[0]}, {moved[1]}}}",))
    else:
        k.emit("cvt.u16.u32", (out,), (move(k.pure("cvt.u32.u16", "u32", x)),))
    return out

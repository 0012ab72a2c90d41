"""Data values and the instruction sequences of Emmy's elementwise ops.

A data value is a ``Val``: a register and its Emmy dtype (a bool is a predicate register). Emmy's
dtype rule decides where an op computes (reference ``ptxgen/ops.py:173-192``): natively for f16's
simple ops, integer ops and f64; every other op converts its inputs to f32, computes, and converts
the result back once.

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
from functools import partial

from . import fastmath
from .dtypes import FLOAT_TYPES, is_float, is_int, literal, move_type, reg_type, size
from .ptx import Kernel

Op = Callable[..., str]

# Other spellings of Emmy's op names.
ALIASES = {"sub": "subtract", "mul": "multiply", "div": "divide", "max": "maximum",
           "min": "minimum", "sum": "add", "prod": "multiply", "amax": "maximum",
           "amin": "minimum", "true_divide": "divide", "neg": "negative", "pow_": "pow",
           "power": "pow", "rsqrt_": "rsqrt"}
BINARY = {"add", "subtract", "multiply", "divide", "maximum", "minimum", "pow"}
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


def const(k: Kernel, value: float, typ: str) -> str:
    """A register holding ``value`` (16-bit float arithmetic takes no immediates)."""
    return k.pure(f"mov.{move_type(typ)}", typ, literal(value, typ))


# The forms ``--no_fusion`` writes: no rounding modifier, so ptxas may contract them.
UNFUSED = {"add.rn": "add", "sub.rn": "sub", "mul.rn": "mul"}


def arith(k: Kernel, m: str) -> str:
    """Mnemonic ``m`` as this kernel writes it: ``add.rn``/``sub.rn``/``mul.rn`` lose their
    rounding modifier with fusion off; everything else is unchanged."""
    return UNFUSED.get(m, m) if k.no_fusion else m


def _bin(m: str, t: str, k: Kernel, a: str, b: str) -> str:
    return k.pure(f"{arith(k, m)}.{t}", t, a, b)


def _un(m: str, t: str, k: Kernel, x: str) -> str:
    return k.pure(f"{m}.{t}", t, x)


def fma_operands(k: Kernel, t: str, a: str, b: str) -> tuple[str, str, str] | None:
    """``(x, y, c)`` when ``a + b`` is ``x * y + c`` for a multiply of type ``t`` that is still
    reusable here, trying ``a`` first; never with fusion off, and only for f32/f64."""
    if k.no_fusion or t not in ("f32", "f64"):
        return None
    for prod, c in ((a, b), (b, a)):
        key = k.definition(prod)
        if key and key[0] == f"mul.rn.{t}":
            return key[1], key[2], c
    return None


def _add(t: str, k: Kernel, a: str, b: str) -> str:
    if (f := fma_operands(k, t, a, b)) is not None:
        return k.pure(f"fma.rn.{t}", t, *f)
    return _bin("add.rn", t, k, a, b)


def _float_ops(t: str) -> dict[str, Op]:
    def zero(k: Kernel) -> str:
        return const(k, 0.0, t) if t == "f16" else literal(0.0, t)

    return {
        "add": partial(_add, t),
        "subtract": partial(_bin, "sub.rn", t),
        "multiply": partial(_bin, "mul.rn", t),
        "divide": partial(_bin, "div.rn", t),
        "maximum": partial(_bin, "max", t),
        "minimum": partial(_bin, "min", t),
        "relu": lambda k, x: _bin("max", t, k, x, zero(k)),
        "negative": partial(_un, "neg", t),
        "abs": partial(_un, "abs", t),
        "square": lambda k, x: _bin("mul.rn", t, k, x, x),
        "reciprocal": partial(_un, "rcp.rn", t),
        "sqrt": partial(_un, "sqrt.rn", t),
        "floor": partial(_un, "cvt.rmi", t + "." + t) if t != "f16" else None,
        "ceil": partial(_un, "cvt.rpi", t + "." + t) if t != "f16" else None,
        "trunc": partial(_un, "cvt.rzi", t + "." + t) if t != "f16" else None,
        "round": partial(_un, "cvt.rni", t + "." + t) if t != "f16" else None,
    }


def _rounding(m: str, t: str, k: Kernel, x: str) -> str:
    return k.pure(f"{m}.{t}.{t}", t, x)


F32_OPS: dict[str, Op] = {n: f for n, f in _float_ops("f32").items() if f is not None}
F32_OPS |= {"rsqrt": partial(_un, "rsqrt.approx", "f32")}
for _m, _n in (("cvt.rmi", "floor"), ("cvt.rpi", "ceil"), ("cvt.rzi", "trunc"),
               ("cvt.rni", "round")):
    F32_OPS[_n] = partial(_rounding, _m, "f32")
F64_OPS: dict[str, Op] = {n: f for n, f in _float_ops("f64").items() if f is not None}
for _m, _n in (("cvt.rmi", "floor"), ("cvt.rpi", "ceil"), ("cvt.rzi", "trunc"),
               ("cvt.rni", "round")):
    F64_OPS[_n] = partial(_rounding, _m, "f64")
# f16 computes natively only where Emmy does (its simple ops); the rest go through f32.
F16_OPS = {n: f for n, f in _float_ops("f16").items()
           if f is not None and n not in ("divide", "reciprocal", "sqrt", "square", "floor",
                                          "ceil", "trunc", "round")}
# Integer ops Emmy keeps integer: op -> (mnemonic, whether it takes a .b<bits> type).
INT_OPS = {"add": ("add", False), "subtract": ("sub", False), "multiply": ("mul.lo", False),
           "floor_divide": ("div", False), "remainder": ("rem", False), "mod": ("rem", False),
           "left_shift": ("shl", True), "right_shift": ("shr", False),
           "bitwise_and": ("and", True), "bitwise_or": ("or", True),
           "bitwise_xor": ("xor", True), "maximum": ("max", False), "minimum": ("min", False)}


def _int_op(name: str, t: str, k: Kernel, a: str, b: str) -> str:
    m, bits = INT_OPS[name]
    if m in ("shl", "shr") and size(t) != 4:
        raise NotImplementedError(f"{t} op {name}: shift of a non-32-bit integer")
    return k.pure(f"{m}.{f'b{size(t) * 8}' if bits else t}", t, a, b)


def cvt(k: Kernel, x: str, src: str, dst: str) -> str:
    """Register ``x`` from PTX type ``src`` to ``dst`` with C's rules: floats round to nearest,
    float to integer truncates, two 16-bit floats meet in f32 (exact)."""
    if src == dst:
        return x
    if src in FLOAT_TYPES and dst in FLOAT_TYPES and "f32" not in (src, dst):
        return cvt(k, cvt(k, x, src, "f32"), "f32", dst)
    if src == "bf16" and dst == "f32":
        # exact: the bf16 bits are the upper half of the f32 bits. A register pack runs on the
        # integer pipe, where cvt.f32.bf16 would take a slot of the XU pipe that ex2/rcp need.
        zero = k.pure("mov.b16", "b16", "0")
        return k.pure("mov.b32", "f32", f"{{{zero}, {x}}}")
    if src in FLOAT_TYPES and dst in FLOAT_TYPES:
        rnd = "" if size(dst) > size(src) else ".rn"  # widening is exact
    elif dst in FLOAT_TYPES:
        rnd = ".rn"
    elif src in FLOAT_TYPES:
        rnd = ".rzi"
    else:
        rnd = ""
    return k.pure(f"cvt{rnd}.{dst}.{src}", dst, x)


def convert(k: Kernel, v: Val, dtype: str) -> Val:
    """``v`` as Emmy dtype ``dtype``: rounding conversions, bool as 1/0, nonzero as true."""
    if v.dtype == dtype:
        return v
    typ = reg_type(dtype)
    if v.dtype == "bool":
        one, zero = (const(k, 1.0, typ), const(k, 0.0, typ)) if typ in ("f16", "bf16") else (
            literal(1.0, typ), literal(0.0, typ))
        return select(k, v.reg, one, zero, dtype)
    if dtype == "bool":
        x = convert(k, v, "f32" if is_float(v.dtype) else "i32")
        zero = literal(0.0, reg_type(x.dtype))
        return Val(k.pure(f"setp.ne.{reg_type(x.dtype)}", "pred", x.reg, zero), dtype)
    return Val(cvt(k, v.reg, reg_type(v.dtype), typ), dtype)


def select(k: Kernel, cond: str, a: str, b: str, dtype: str) -> Val:
    typ = reg_type(dtype)
    if typ == "pred":
        out = k.pure("or.pred", "pred", k.pure("and.pred", "pred", cond, a),
                     k.pure("and.pred", "pred", k.pure("not.pred", "pred", cond), b))
        return Val(out, dtype)
    return Val(k.pure(f"selp.{move_type(typ)}", typ, a, b, cond), dtype)


def promote(name: str, dtypes: Sequence[str]) -> str:
    """The result dtype of an op with no explicit dtype (Emmy's promotion, as restated for the
    cases Kernel IR leaves implicit: combine programs, whose arguments share one dtype)."""
    if name in COMPARE:
        return "bool"
    ds = list(dict.fromkeys(dtypes))
    if len(ds) == 1:
        return ds[0]
    floats = [d for d in ds if d != "bool" and is_float(d)]
    if floats:
        order = ["f16", "bf16", "f32", "f64"]
        best = max(floats, key=order.index)
        if set(floats) == {"f16", "bf16"}:
            return "f32"
        return best
    ints = [d for d in ds if d != "bool"]
    return max(ints, key=size) if ints else "bool"


def apply(k: Kernel, name: str, args: Sequence[Val], dtype: str) -> Val:
    """name(args) at result ``dtype`` under Emmy's rule: native where Emmy computes there,
    otherwise in f32, converted once."""
    name, typ = canonical(name), reg_type(dtype)
    at, fn = dtype, None
    if typ == "f16" and all(a.dtype == dtype for a in args):
        fn = F16_OPS.get(name)
    elif is_int(dtype) and all(is_int(a.dtype) for a in args) and name in INT_OPS:
        fn = partial(_int_op, name, typ)
    elif dtype == "f64":
        fn = F64_OPS.get(name)
    if fn is None:
        at, fn = "f32", F32_OPS.get(name) or fastmath.F32_FUNCS.get(name)
    if fn is None:
        raise NotImplementedError(f"{at} op {name}")
    arity = 2 if name in BINARY else 1
    if len(args) != arity:
        raise ValueError(f"{at} op {name} takes {arity} argument(s), got {len(args)}")
    out = fn(k, *(convert(k, a, at).reg for a in args))
    return convert(k, Val(out, at), dtype)


def assign(k: Kernel, name: str, dtype: str | None, args: Sequence[Val]) -> Val:
    """The value of an Assign of op ``name`` over ``args`` (compares compute in f32)."""
    name = canonical(name)
    dtype = dtype if dtype is not None else promote(name, [v.dtype for v in args])
    if name in COMPARE:
        x, y = (convert(k, v, "f32").reg for v in args)
        p = Val(k.pure(f"setp.{COMPARE[name]}.f32", "pred", x, y), "bool")
        return convert(k, p, dtype)
    if name == "where":
        cond = convert(k, args[0], "bool").reg
        x, y = (convert(k, v, dtype).reg for v in args[1:])
        return select(k, cond, x, y, dtype)
    if name in ("logical_and", "logical_or"):
        x, y = (convert(k, v, "bool").reg for v in args)
        op = "and.pred" if name == "logical_and" else "or.pred"
        return convert(k, Val(k.pure(op, "pred", x, y), "bool"), dtype)
    if name == "logical_not":
        x = convert(k, args[0], "bool").reg
        return convert(k, Val(k.pure("not.pred", "pred", x), "bool"), dtype)
    if name in ("copy", "pad", "identity", "cast", "to"):
        return convert(k, args[0], dtype)
    return apply(k, name, args, dtype)


# --- shuffles -------------------------------------------------------------------------------


def shfl(k: Kernel, x: str, typ: str, mode: str, lane: str | int, clamp: int, mask: str) -> str:
    """One ``shfl.sync`` of ``x``: 64-bit values move as two halves, 16-bit ones widen."""

    def one(v: str, t: str) -> str:
        out = k.reg(t)
        k.emit(f"shfl.sync.{mode}.b32", (out,), (v, str(lane), str(clamp), mask))
        return out

    if size(typ) == 4:
        return one(x, typ)
    out = k.reg(typ)
    if size(typ) == 8:
        lo, hi = k.reg("u32"), k.reg("u32")
        k.emit("mov.b64", (f"{{{lo}, {hi}}}",), (x,))
        a, b = one(lo, "u32"), one(hi, "u32")
        k.emit("mov.b64", (out,), (f"{{{a}, {b}}}",))
    elif typ == "pred":
        w = k.pure("selp.u32", "u32", "1", "0", x)
        r = one(w, "u32")
        return k.pure("setp.ne.u32", "pred", r, "0")
    else:
        wide = k.pure("cvt.u32.u16", "u32", x)
        k.emit("cvt.u16.u32", (out,), (one(wide, "u32"),))
    return out

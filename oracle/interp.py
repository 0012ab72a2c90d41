"""NumPy oracle: a CPU interpreter of Emmy Kernel IR semantics, vectorised over the threads.

TEST INFRASTRUCTURE, not product code: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import it, as the checker of the CUDA path. Nothing in ptxgen imports it.

It runs a kernel the way the reference lowering defines it (reference ``ptxgen/compiler.py``):

* Tile: the global id ``ctaid*block + tid`` over ``N = prod(extents)`` cells, decoded row-major
  into the axes (``compiler.py:268-302``), with Emmy's grouped raster order for a raster pair;
* Load/Write: row-major flattening (``compiler.py:389-399``), consecutive names at consecutive
  elements, conversion to the buffer's dtype on store, ``atomic`` as an add;
* data ops: Emmy's dtype rule (``ops.py:173-192``): native for f16's simple ops, integer ops and
  f64, otherwise in f32 with one rounding back; bf16 -> f32 exact, f32 -> bf16 nearest even;
* every f32/f64 add/sub/mul/div/sqrt rounds to nearest, and an add whose operand is the result of
  a multiply of the same float type is one fused multiply-add, exactly as ``ptxgen/ops.py:56-71``
  decides it (the multiply must still be reusable: none of its operands written in place since,
  and no loop that writes one entered since); ``oracle.fp.fma_f32`` makes that rounding exact;
* fast math (``fastmath.py``): the same instruction sequences, with each hardware approximation
  (``ex2``, ``lg2``, ``rcp.approx``, ``sin``, ``cos``, ``rsqrt``) modelled as correctly rounded, so
  the oracle differs from the GPU by those instructions' few-ulp errors only;
* WarpShuffle: the xor butterfly of ``length/2 .. 1`` (``compiler.py:445-465``); TreeHalve: the
  shared-memory halving tree (``compiler.py:467-499``); Sync is a no-op, since all threads run in
  lockstep, which any barrier-synchronised, race-free kernel matches;
* loops: every trip, in order, per thread; a thread whose trips end earlier idles (masked).

The interpreter holds one array per name over all threads of the grid, so it suits test-sized
problems (a few million thread-steps in seconds).
"""

from __future__ import annotations

import math
import sys
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "emmy-hackathon-submission_b200"))

from ptxgen.ir import (Accum, Assign, BinaryExpr, CastExpr, Cond, CpAsyncCommit,  # noqa: E402
                       CpAsyncCopy, CpAsyncWait, Expr, FuncCallExpr, Graph, Init, Let, Literal,
                       Load, Loop, Select, Smem, Stmt, StridedLoop, Sync, TernaryExpr, Tile,
                       TreeHalve, Var, WarpShuffle, Write, walk)

from .fp import bf16_round, fma_f32, fma_f64, ftz32, rn32  # noqa: E402

NP = {"f32": np.float32, "f64": np.float64, "f16": np.float16, "bf16": np.float32,
      "i32": np.int64, "u32": np.int64, "i64": np.int64, "u64": np.int64, "i16": np.int64,
      "u16": np.int64, "u8": np.int64, "bool": np.bool_}
FLOATS = ("f32", "f64", "f16", "bf16")
BITS = {"i32": 32, "u32": 32, "i64": 64, "u64": 64, "i16": 16, "u16": 16, "u8": 8}
SIGNED = {"i32", "i64", "i16"}
ALIASES = {"sub": "subtract", "mul": "multiply", "div": "divide", "max": "maximum",
           "min": "minimum", "sum": "add", "prod": "multiply", "amax": "maximum",
           "amin": "minimum", "true_divide": "divide", "neg": "negative", "pow_": "pow",
           "power": "pow"}
IDENTITY = {"add": 0.0, "subtract": 0.0, "multiply": 1.0, "divide": 1.0,
            "maximum": -math.inf, "minimum": math.inf}
COMPARE = {"equal": np.equal, "not_equal": np.not_equal, "greater": np.greater,
           "less": np.less, "greater_equal": np.greater_equal, "less_equal": np.less_equal}
CMP_SYMBOL = {"==": np.equal, "!=": np.not_equal, "<": np.less, "<=": np.less_equal,
              ">": np.greater, ">=": np.greater_equal}
BINARY = {"add", "subtract", "multiply", "divide", "maximum", "minimum", "pow"}
F16_NATIVE = {"add", "subtract", "multiply", "maximum", "minimum", "relu", "negative", "abs"}
INT_OPS = {"add", "subtract", "multiply", "floor_divide", "remainder", "mod", "left_shift",
           "right_shift", "bitwise_and", "bitwise_or", "bitwise_xor", "maximum", "minimum"}
LOG2E32 = np.float32(math.log2(math.e))
LN2_32 = np.float32(math.log(2.0))
SMEM_NAMES = {"float": "f32", "double": "f64", "half": "f16", "__half": "f16",
              "__nv_bfloat16": "bf16", "bfloat16": "bf16", "int": "i32", "unsigned": "u32",
              "unsigned int": "u32", "long long": "i64", "unsigned long long": "u64"}


def canonical(name: str) -> str:
    return ALIASES.get(name, name)


@dataclass
class D:
    """A data value: an array over all threads and its Emmy dtype. ``prod`` holds the operands
    when the value is the result of a multiply the lowering can still fuse into an add."""

    a: np.ndarray
    dtype: str
    prod: tuple[np.ndarray, np.ndarray] | None = None
    deps: frozenset[str] = frozenset()


@dataclass
class Idx:
    """An index value: an int64 array over all threads."""

    a: np.ndarray


@dataclass
class Buf:
    shape: tuple[int, ...]
    dtype: str
    data: np.ndarray  # flat; bf16 as f32 values; shared: [blocks, size]
    shared: bool = False


@dataclass
class Options:
    no_fusion: bool = False


def _wrap(x: np.ndarray, dtype: str) -> np.ndarray:
    bits = BITS[dtype]
    x = np.asarray(x, np.int64)
    if bits == 64:
        return x
    m = x & ((1 << bits) - 1)
    if dtype in SIGNED:
        m = np.where(m >= 1 << (bits - 1), m - (1 << bits), m)
    return m


def to_dtype(x: np.ndarray, src: str, dst: str) -> np.ndarray:
    """Convert an array of Emmy dtype ``src`` to ``dst`` with C's rules (floats round to
    nearest, float to integer truncates; 16-bit floats meet in f32)."""
    if src == dst:
        return x
    if dst == "bool":
        return np.asarray(x) != 0
    if src == "bool":
        x = np.asarray(x).astype(np.float64)
        src = "f64"
    if dst in FLOATS:
        with np.errstate(over="ignore", invalid="ignore"):
            v = np.asarray(x).astype(np.float64) if src not in FLOATS else np.asarray(x)
            if dst == "f64":
                return v.astype(np.float64)
            if dst == "f32":
                return v.astype(np.float32)
            if dst == "f16":
                return v.astype(np.float32).astype(np.float16) if src != "f64" else \
                    v.astype(np.float16)
            return bf16_round(v.astype(np.float32) if src != "f64" else v.astype(np.float32))
    # to integer
    if src in FLOATS:
        with np.errstate(invalid="ignore"):
            v = np.trunc(np.asarray(x, np.float64))
            v = np.nan_to_num(v, nan=0.0, posinf=2.0**62, neginf=-(2.0**62))
        return _wrap(v.astype(np.int64), dst)
    return _wrap(np.asarray(x, np.int64), dst)


def _f32(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32)


# Fast-math sequences of ptxgen/fastmath.py with each approximate instruction correctly rounded.
def _ex2(t: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return ftz32(rn32(np.exp2(ftz32(t).astype(np.float64))))


def _lg2(x: np.ndarray) -> np.ndarray:
    with np.errstate(divide="ignore", invalid="ignore"):
        return rn32(np.log2(ftz32(x).astype(np.float64)))


def _rcp_approx(x: np.ndarray) -> np.ndarray:
    with np.errstate(divide="ignore"):
        return ftz32(rn32(1.0 / ftz32(x).astype(np.float64)))


def fm_exp(x: np.ndarray) -> np.ndarray:
    return _ex2(_f32(x) * LOG2E32)


def fm_log(x: np.ndarray) -> np.ndarray:
    return _lg2(x) * LN2_32


def fm_tanh(x: np.ndarray) -> np.ndarray:
    e = _ex2(_f32(x) * np.float32(2.0 * math.log2(math.e)))
    r = _rcp_approx(e + np.float32(1.0))
    return fma_f32(r, np.float32(-2.0), np.float32(1.0))


def fm_sigmoid(x: np.ndarray) -> np.ndarray:
    e = _ex2(_f32(x) * np.float32(-math.log2(math.e)))
    return _rcp_approx(e + np.float32(1.0))


AS_P = 0.3275911
AS_A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def fm_erf(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    ax = np.abs(x)
    t = _rcp_approx(fma_f32(ax, np.float32(AS_P), np.float32(1.0)))
    poly = np.float32(AS_A[4]) * np.ones_like(x)
    for c in (*reversed(AS_A[:4]), 0.0):
        poly = fma_f32(t, poly, np.float32(c))
    e = fm_exp(-(ax * ax))
    return np.copysign(fma_f32(-poly, e, np.float32(1.0)), x).astype(np.float32)


def fm_pow(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    x, y = _f32(x), _f32(y)
    r = _ex2(_lg2(np.abs(x)) * y)
    whole = np.rint(y) == y
    half = y * np.float32(0.5)
    odd = whole & (np.rint(half) != half)
    neg = x < 0
    r = np.where(neg & odd, -r, r)
    r = np.where(whole | ~neg, r, np.float32(np.nan))
    return np.where(y == 0, np.float32(1.0), r).astype(np.float32)


F32_FUNCS = {
    "exp": fm_exp, "exp2": _ex2, "log": fm_log, "log2": _lg2, "tanh": fm_tanh,
    "sigmoid": fm_sigmoid, "erf": fm_erf, "pow": fm_pow,
    "sin": lambda x: ftz32(rn32(np.sin(ftz32(x).astype(np.float64)))),
    "cos": lambda x: ftz32(rn32(np.cos(ftz32(x).astype(np.float64)))),
    "rsqrt": lambda x: rn32(1.0 / np.sqrt(_f32(x).astype(np.float64))),
}


def _float_op(name: str, t: str, args: list[np.ndarray]) -> np.ndarray:
    dt = np.float64 if t == "f64" else np.float16 if t == "f16" else np.float32
    a = [np.asarray(x, dt) for x in args]
    with np.errstate(all="ignore"):
        if name == "add":
            return a[0] + a[1]
        if name == "subtract":
            return a[0] - a[1]
        if name == "multiply":
            return a[0] * a[1]
        if name == "divide":
            return a[0] / a[1]
        if name == "maximum":
            return np.fmax(a[0], a[1])
        if name == "minimum":
            return np.fmin(a[0], a[1])
        if name == "relu":
            return np.fmax(a[0], dt(0))
        if name == "negative":
            return -a[0]
        if name == "abs":
            return np.abs(a[0])
        if name == "square":
            return a[0] * a[0]
        if name == "reciprocal":
            return dt(1) / a[0]
        if name == "sqrt":
            return np.sqrt(a[0])
        if name == "floor":
            return np.floor(a[0])
        if name == "ceil":
            return np.ceil(a[0])
        if name == "trunc":
            return np.trunc(a[0])
        if name == "round":
            return np.rint(a[0])
    raise NotImplementedError(f"{t} op {name}")


def _int_op(name: str, t: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = np.asarray(a, np.int64), np.asarray(b, np.int64)
    with np.errstate(all="ignore"):
        if name == "add":
            r = a + b
        elif name == "subtract":
            r = a - b
        elif name == "multiply":
            r = a * b
        elif name == "floor_divide":
            r = np.where(b != 0, np.trunc(a / np.where(b == 0, 1, b)), 0).astype(np.int64)
        elif name in ("remainder", "mod"):
            r = np.where(b != 0, np.fmod(a, np.where(b == 0, 1, b)), 0)
        elif name == "left_shift":
            r = a << (b & 31)
        elif name == "right_shift":
            r = a >> (b & 31)
        elif name == "bitwise_and":
            r = a & b
        elif name == "bitwise_or":
            r = a | b
        elif name == "bitwise_xor":
            r = a ^ b
        elif name == "maximum":
            r = np.maximum(a, b)
        else:
            r = np.minimum(a, b)
    return _wrap(r, t)


def promote(name: str, dtypes: Sequence[str]) -> str:
    if name in COMPARE:
        return "bool"
    ds = list(dict.fromkeys(dtypes))
    if len(ds) == 1:
        return ds[0]
    floats = [d for d in ds if d in FLOATS]
    if floats:
        if set(floats) == {"f16", "bf16"}:
            return "f32"
        return max(floats, key=["f16", "bf16", "f32", "f64"].index)
    ints = [d for d in ds if d != "bool"]
    return max(ints, key=lambda d: BITS[d]) if ints else "bool"


class Interpreter:
    """Runs one KernelOp over given input arrays; ``run`` returns the output buffers."""

    def __init__(self, graph: Graph | dict[str, Any], meta: dict[str, Any],
                 inputs: dict[str, np.ndarray], options: Options | None = None,
                 op: Any = None):
        """``op``: run this KernelOp in place of the graph's (a rewritten body of the same
        kernel, as a compiler pass produces it), with its own shared buffers."""
        from ptxgen.compiler import kernel_for_meta

        graph = graph if isinstance(graph, Graph) else Graph.from_dict(graph)
        self.op, self.launch = kernel_for_meta(graph, meta)
        if op is not None:
            self.op = op
        self.opts = options or Options()
        self.block = int(self.launch["block"][0])
        self.grid = int(self.launch["grid"][0])
        self.T = self.block * self.grid
        self.gid = np.arange(self.T, dtype=np.int64)
        self.blk = self.gid // self.block
        self.tid = self.gid % self.block
        self.mem: dict[str, Buf] = {}
        for a in self.launch["args"]:
            shape = tuple(int(s) for s in a["shape"])
            n = int(np.prod(shape)) if shape else 1
            if a["name"] in inputs:
                arr = np.asarray(inputs[a["name"]]).reshape(-1)
                if a["dtype"] == "bf16":
                    data = (arr.astype(np.uint32) << 16).view(np.float32).copy() if \
                        arr.dtype == np.uint16 else bf16_round(arr.astype(np.float32))
                else:
                    data = arr.astype(NP[a["dtype"]]).copy()
            else:
                data = np.zeros(n, NP[a["dtype"]])
            self.mem[a["name"]] = Buf(shape, a["dtype"], data)
        for s in self.op.smem_buffers.values():
            dtype = SMEM_NAMES.get(s.dtype, s.dtype)
            size = int(np.prod(s.extents))
            self.mem[s.name] = Buf(tuple(s.extents), dtype,
                                   np.zeros((self.grid, size), NP[dtype]), shared=True)
        self.env: dict[str, Any] = {}
        self.variables: set[str] = set()
        lane, warp = self.tid & 31, self.tid >> 5
        self.env["lane"], self.env["warp"] = Idx(lane), Idx(warp)

    # --- driver -------------------------------------------------------------------------
    def run(self) -> dict[str, np.ndarray]:
        for name in self.launch.get("zero_outputs", []):
            self.mem[name].data[:] = 0
        self.stmts(self.op.body and [self.op.body], np.ones(self.T, bool))
        out = {}
        for a in self.launch["args"]:
            if a.get("output") or a["name"] in self.op.outputs:
                b = self.mem[a["name"]]
                out[a["name"]] = b.data.reshape(b.shape or (1,))
        return out

    def stmts(self, body: Sequence[Stmt], mask: np.ndarray) -> None:
        for st in body:
            fn = getattr(self, f"do_{type(st).__name__}", None)
            if fn is None:
                raise NotImplementedError(f"oracle: no semantics for {type(st).__name__}")
            fn(st, mask)

    def _scoped(self, body: Sequence[Stmt], mask: np.ndarray) -> None:
        before = set(self.env)
        self.stmts(body, mask)
        for name in set(self.env) - before:
            del self.env[name]

    # --- names --------------------------------------------------------------------------
    def data(self, name: str) -> D:
        v = self.env[name]
        return v if isinstance(v, D) else self._as_data(v)

    def _as_data(self, v: Any) -> D:
        if isinstance(v, D):
            return v
        if isinstance(v, Idx):
            return D(_wrap(v.a, "i32"), "i32")
        if isinstance(v, bool | np.bool_):
            return D(np.full(self.T, bool(v)), "bool")
        raise TypeError(v)

    def define(self, name: str, v: D) -> None:
        """Bind a name; a name copied from a variable carries no fusable product."""
        self.env[name] = v

    def write_var(self, name: str, v: D, mask: np.ndarray) -> None:
        """Write variable ``name`` in place where ``mask`` holds (converting to its dtype)."""
        cur = self.data(name)
        new = to_dtype(v.a, v.dtype, cur.dtype)
        self.env[name] = D(np.where(mask, new, cur.a).astype(cur.a.dtype), cur.dtype)
        self.variables.add(name)
        self.forget(name)

    def forget(self, var: str) -> None:
        """``var`` was written in place: products that read it can no longer fuse."""
        for n, v in self.env.items():
            if isinstance(v, D) and v.prod is not None and var in v.deps:
                self.env[n] = D(v.a, v.dtype)

    def make_var(self, name: str, dtype: str | None = None) -> D:
        v = self.data(name)
        if dtype is not None and v.dtype != dtype:
            v = D(to_dtype(v.a, v.dtype, dtype), dtype)
        v = D(v.a.copy(), v.dtype)
        self.env[name] = v
        self.variables.add(name)
        return v

    # --- launch -------------------------------------------------------------------------
    def do_Tile(self, t: Tile, mask: np.ndarray) -> None:
        n = t.n_elements
        if -(-n // self.block) != self.grid:
            raise ValueError(f"Tile of {n} cells needs {-(-n // self.block)} blocks, "
                             f"meta launches {self.grid}")
        active = mask & (self.gid < n)
        gid = self.gid
        extents = list(t.extents)
        strides = [math.prod(extents[i + 1:]) for i in range(len(extents))]
        axes: dict[str, np.ndarray] = {}
        raster = self._raster(t)
        for i, (axis, e) in enumerate(zip(t.axes, extents, strict=True)):
            if raster is not None and i in raster[:2]:
                continue
            v = gid // strides[i]
            axes[axis.name] = v % e if i else v
        if raster is not None:
            gi, oi, g = raster
            ea, eb = extents[gi], extents[oi]
            sub = gid // strides[max(gi, oi)]
            if min(gi, oi):
                sub = sub % (ea * eb)
            if eb == 1:
                a, b = sub, np.zeros_like(sub)
            else:
                grp, r = sub // (g * eb), sub % (g * eb)
                gsz = np.minimum(ea - grp * g, g) if ea % g else np.full_like(sub, g)
                a, b = grp * g + r % gsz, r // gsz
            axes[t.axes[gi].name], axes[t.axes[oi].name] = a, b
        for name, v in axes.items():
            self.env[name] = Idx(v)
        self._scoped(t.body, active)

    @staticmethod
    def _raster(t: Tile) -> tuple[int, int, int] | None:
        names = [a.name for a in t.axes]
        if not (t.raster_group and t.raster_axes and all(n in names for n in t.raster_axes)):
            return None
        mi, ni = (names.index(n) for n in t.raster_axes)
        if ni != mi + 1:
            return None
        gi, oi = (mi, ni) if t.raster_orient == "m" else (ni, mi)
        g = min(t.raster_group, t.extents[gi])
        return (gi, oi, g) if t.extents[gi] > 1 and g > 1 else None

    def do_Sync(self, s: Sync, mask: np.ndarray) -> None:
        pass

    def do_Smem(self, s: Smem, mask: np.ndarray) -> None:
        pass

    # --- memory -------------------------------------------------------------------------
    def _flat(self, buf: Buf, parts: list[np.ndarray]) -> np.ndarray:
        if len(parts) <= 1:
            return parts[0] if parts else np.zeros(self.T, np.int64)
        flat, stride = np.zeros(self.T, np.int64), 1
        for i, extent in zip(reversed(parts), reversed(buf.shape), strict=True):
            flat, stride = flat + i * stride, stride * int(extent)
        return flat

    def _gather(self, buf: Buf, flat: np.ndarray, mask: np.ndarray) -> np.ndarray:
        out = np.zeros(self.T, buf.data.dtype)
        idx = np.where(mask, flat, 0)
        if buf.shared:
            out[mask] = buf.data[self.blk[mask], idx[mask]]
        else:
            size = buf.data.shape[0]
            if np.any(mask & ((idx < 0) | (idx >= size))):
                raise IndexError(f"oracle: load out of bounds of a {size}-element buffer")
            out[mask] = buf.data[idx[mask]]
        return out

    def _scatter(self, buf: Buf, flat: np.ndarray, vals: np.ndarray, mask: np.ndarray,
                 atomic: bool = False) -> None:
        idx = flat[mask]
        v = vals[mask]
        if buf.shared:
            buf.data[self.blk[mask], idx] = v
            return
        if np.any((idx < 0) | (idx >= buf.data.shape[0])):
            raise IndexError("oracle: store out of bounds")
        if atomic:
            np.add.at(buf.data, idx, v)
        else:
            buf.data[idx] = v

    def do_Load(self, s: Load, mask: np.ndarray) -> None:
        buf = self.mem[s.input]
        dtype = s.dtype.name if s.dtype is not None else buf.dtype
        flat = self._flat(buf, [self.idx(e) for e in s.index])
        for j, name in enumerate(s.names):
            raw = self._gather(buf, flat + j, mask)
            self.env[name] = D(to_dtype(raw, buf.dtype, dtype), dtype)

    def do_Write(self, s: Write, mask: np.ndarray) -> None:
        buf = self.mem[s.output]
        flat = self._flat(buf, [self.idx(e) for e in s.index])
        for j, name in enumerate(s.values):
            v = self.data(name)
            vals = to_dtype(v.a, v.dtype, buf.dtype)
            self._scatter(buf, flat + j, vals, mask, s.atomic)

    def do_CpAsyncCopy(self, s: CpAsyncCopy, mask: np.ndarray) -> None:
        dst, src = self.mem[s.smem], self.mem[s.src]
        idx = [self.idx(e) for e in s.smem_index]
        if s.lane_index is not None:
            idx = [a + self.idx(b) for a, b in zip(idx, s.lane_index, strict=True)]
        d = self._flat(dst, idx)
        sflat = self._flat(src, [self.idx(e) for e in s.src_index])
        esz = {"f32": 4, "f64": 8, "f16": 2, "bf16": 2, "i32": 4, "u32": 4}[src.dtype]
        for j in range(s.nbytes // esz):
            self._scatter(dst, d + j, self._gather(src, sflat + j, mask), mask)

    def do_CpAsyncCommit(self, s: CpAsyncCommit, mask: np.ndarray) -> None:
        pass

    def do_CpAsyncWait(self, s: CpAsyncWait, mask: np.ndarray) -> None:
        pass

    # --- data ---------------------------------------------------------------------------
    def apply(self, name: str, args: list[D], dtype: str, arg_names: Sequence[str] = ()) -> D:
        """name(args) at ``dtype`` under Emmy's rule, with the lowering's fma fusion."""
        name = canonical(name)
        at = dtype
        native = None
        if dtype == "f16" and all(a.dtype == "f16" for a in args) and name in F16_NATIVE:
            native = "f16"
        elif dtype not in FLOATS and dtype != "bool" and \
                all(a.dtype not in FLOATS and a.dtype != "bool" for a in args) and \
                name in INT_OPS:
            native = "int"
        elif dtype == "f64" and name not in F32_FUNCS:
            native = "f64"
        if native is None:
            at = "f32"
        conv = [D(to_dtype(a.a, a.dtype, at), at,
                  a.prod if a.dtype == at else None, a.deps) for a in args]
        if native == "int":
            if len(conv) != 2:
                raise NotImplementedError(f"int op {name}")
            out = D(_int_op(name, at, conv[0].a, conv[1].a), at)
        elif name == "log" and at == "f32":
            # the lowering's log ends in a multiply (lg2(x) * ln 2), which an add can fuse
            lg = _lg2(conv[0].a)
            out = D(lg * LN2_32, at, (lg, np.full_like(lg, LN2_32)), frozenset())
        elif name in F32_FUNCS and at == "f32":
            out = D(F32_FUNCS[name](*[c.a for c in conv]).astype(np.float32), at)
        else:
            if name == "add" and at in ("f32", "f64") and not self.opts.no_fusion:
                for p, c in ((conv[0], conv[1]), (conv[1], conv[0])):
                    if p.prod is not None:
                        fma = fma_f32 if at == "f32" else fma_f64
                        return self._back(D(fma(p.prod[0], p.prod[1], c.a), at), dtype)
            r = _float_op(name, at, [c.a for c in conv])
            out = D(r, at)
            if name in ("multiply", "square") and at in ("f32", "f64"):
                srcs = (conv[0].a, conv[1].a) if name == "multiply" else (conv[0].a, conv[0].a)
                # a multiply that read a variable directly (not through a conversion) goes
                # stale when that variable is written in place
                deps = frozenset(n for n, a in zip(arg_names, args, strict=False)
                                 if n in self.variables and a.dtype == at)
                out = D(r, at, srcs, deps)
        return self._back(out, dtype)

    @staticmethod
    def _back(v: D, dtype: str) -> D:
        if v.dtype == dtype:
            return v
        return D(to_dtype(v.a, v.dtype, dtype), dtype)

    def assign(self, name: str, dtype: str | None, args: list[D],
               arg_names: Sequence[str] = ()) -> D:
        name = canonical(name)
        dtype = dtype if dtype is not None else promote(name, [a.dtype for a in args])
        if name in COMPARE:
            x, y = (to_dtype(a.a, a.dtype, "f32") for a in args)
            return D(to_dtype(COMPARE[name](x, y), "bool", dtype), dtype)
        if name == "where":
            c = to_dtype(args[0].a, args[0].dtype, "bool")
            x, y = (to_dtype(a.a, a.dtype, dtype) for a in args[1:])
            return D(np.where(c, x, y), dtype)
        if name in ("logical_and", "logical_or"):
            x, y = (to_dtype(a.a, a.dtype, "bool") for a in args)
            r = (x & y) if name == "logical_and" else (x | y)
            return D(to_dtype(r, "bool", dtype), dtype)
        if name == "logical_not":
            return D(to_dtype(~to_dtype(args[0].a, args[0].dtype, "bool"), "bool", dtype), dtype)
        if name in ("copy", "pad", "identity", "cast", "to"):
            return D(to_dtype(args[0].a, args[0].dtype, dtype), dtype)
        return self.apply(name, args, dtype, arg_names)

    def do_Assign(self, s: Assign, mask: np.ndarray) -> None:
        args = [self.data(a) for a in s.args]
        self.define(s.name, self.assign(s.op.name, s.dtype.name if s.dtype else None, args,
                                        s.args))

    def do_Let(self, s: Let, mask: np.ndarray) -> None:
        if s.dtype is None:
            v = self.expr(s.value)
            self.env[s.name] = v
            return
        self.define(s.name, self.value(s.value, s.dtype.name))

    def do_Init(self, s: Init, mask: np.ndarray) -> None:
        self._init(s.name, s.identity, s.dtype.name)

    def _init(self, name: str, identity: float | None, dtype: str) -> None:
        if identity is None:
            raise ValueError(f"{name!r} has no identity")
        self.env[name] = D(to_dtype(np.full(self.T, identity, np.float64), "f64", dtype)
                           if dtype in FLOATS else
                           to_dtype(np.full(self.T, identity), "f64", dtype), dtype)
        self.variables.add(name)
        self.forget(name)

    def do_Select(self, s: Select, mask: np.ndarray) -> None:
        self.define(s.name, self.value(TernaryExpr(s.cond, s.if_true, s.if_false), "f32"))

    def do_Accum(self, s: Accum, mask: np.ndarray) -> None:
        name = canonical(s.op.name)
        dtype = s.dtype.name if s.dtype is not None else "f32"
        if s.name not in self.env:
            self._init(s.name, IDENTITY[name], dtype)
        acc = self.make_var(s.name, dtype) if self.data(s.name).dtype != dtype or \
            s.name not in self.variables else self.data(s.name)
        value = self.data(s.value)
        vconv = D(to_dtype(value.a, value.dtype, dtype), dtype,
                  value.prod if value.dtype == dtype else None, value.deps)
        base = acc if s.base is None else self.data(s.base)
        bconv = D(to_dtype(base.a, base.dtype, dtype), dtype,
                  base.prod if base.dtype == dtype else None, base.deps)
        fused = None
        if name == "add" and dtype in ("f32", "f64") and not self.opts.no_fusion:
            for p, c in ((vconv, bconv), (bconv, vconv)):
                if p.prod is not None and p is not acc:
                    fma = fma_f32 if dtype == "f32" else fma_f64
                    fused = fma(p.prod[0], p.prod[1], c.a)
                    break
        if fused is not None:
            r = fused
        elif dtype == "bf16" or (dtype == "f16" and name == "divide"):
            r = to_dtype(_float_op(name, "f32", [to_dtype(bconv.a, dtype, "f32"),
                                                 to_dtype(vconv.a, dtype, "f32")]),
                         "f32", dtype)
        elif dtype in FLOATS:
            r = _float_op(name, dtype, [bconv.a, vconv.a])
        else:
            r = _int_op(name, dtype, bconv.a, vconv.a)
        self.write_var(s.name, D(np.asarray(r), dtype), mask)

    # --- reduce -------------------------------------------------------------------------
    def _combine(self, program: Sequence[Assign], states: Sequence[str], mask: np.ndarray
                 ) -> None:
        for a in program:
            v = self.assign(a.op.name, a.dtype.name if a.dtype else None,
                            [self.data(x) for x in a.args], a.args)
            if a.name in states:
                self.write_var(a.name, v, mask)
            else:
                self.define(a.name, v)

    def do_WarpShuffle(self, s: WarpShuffle, mask: np.ndarray) -> None:
        dtype = s.dtype.name
        for st in s.state:
            self.make_var(st, dtype)
        step = s.length // 2
        while step:
            src = self.gid ^ step
            for st, sb in zip(s.state, s.state_b, strict=True):
                v = self.data(st)
                self.env[sb] = D(v.a[src], v.dtype)
            self._combine(s.combine_states, s.state, mask)
            step //= 2

    def do_TreeHalve(self, s: TreeHalve, mask: np.ndarray) -> None:
        trees = [(self.mem[b], st, sb) for b, st, sb in zip(s.bufs, s.state, s.state_b,
                                                            strict=True)]
        for buf, st, _ in trees:
            self.make_var(st, buf.dtype)
        t = self.idx(Var(s.tid_var))
        scale, root = (1, np.zeros(self.T, np.int64)) if s.inner is None else (
            s.inner[1], self.idx(Var(s.inner[0])))
        half = s.length // 2
        while half:
            active = mask & (t < half)
            mine = t * scale + root
            before = set(self.env)
            for buf, st, sb in trees:
                self.write_var(st, D(self._gather(buf, mine, active), buf.dtype), active)
                self.env[sb] = D(self._gather(buf, mine + half * scale, active), buf.dtype)
            self._combine(s.combine_states, s.state, active)
            for buf, st, _ in trees:
                self._scatter(buf, mine, to_dtype(self.data(st).a, self.data(st).dtype,
                                                  buf.dtype), active)
            for name in set(self.env) - before:
                del self.env[name]
            half //= 2
        for buf, st, _ in trees:
            self.write_var(st, D(self._gather(buf, root, mask), buf.dtype), mask)

    # --- control ------------------------------------------------------------------------
    def do_Cond(self, s: Cond, mask: np.ndarray) -> None:
        p = self.pred(s.cond)
        self._scoped(s.body, mask & p)
        if s.else_body:
            self._scoped(s.else_body, mask & ~p)

    def do_Loop(self, s: Loop | StridedLoop, mask: np.ndarray) -> None:
        if isinstance(s, StridedLoop):
            step = self.idx(s.step) if isinstance(s.step, Expr) else np.full(self.T, s.step)
            start = self.idx(s.start)
            end = np.full(self.T, s.axis.extent.as_static()) if s.end is None else \
                self.idx(s.end)
        else:
            start = np.zeros(self.T, np.int64)
            step = np.ones(self.T, np.int64)
            end = np.full(self.T, s.axis.extent.as_static())
        seen: set[str] = set()
        for st in s.body:
            if isinstance(st, Accum) and st.name not in seen:
                seen.add(st.name)
                if s.seed:
                    dtype = st.dtype.name if st.dtype is not None else "f32"
                    self._init(st.name, IDENTITY[canonical(st.op.name)], dtype)
        written = {n for st in walk(s.body) for n in self._written(st)}
        for n in written & set(self.env):
            if n not in self.variables:
                self.make_var(n)
            self.forget(n)
        axis = start.copy()
        live = mask & (axis < end)
        while np.any(live):
            before = set(self.env)
            self.env[s.axis.name] = Idx(axis)
            self.stmts(s.body, live)
            for name in set(self.env) - before:
                del self.env[name]
            axis = axis + step
            live = live & (axis < end)

    do_StridedLoop = do_Loop

    @staticmethod
    def _written(st: Stmt) -> Sequence[str]:
        if isinstance(st, Accum):
            return (st.name,)
        if isinstance(st, WarpShuffle | TreeHalve):
            return tuple(st.state)
        return ()

    # --- expressions --------------------------------------------------------------------
    def expr(self, e: Expr) -> Any:
        if isinstance(e, Var):
            return self.env[e.name]
        if isinstance(e, Literal):
            if e.dtype == "bool" or isinstance(e.value, bool):
                return np.full(self.T, bool(e.value))
            if e.dtype == "int" or isinstance(e.value, int):
                return Idx(np.full(self.T, int(e.value), np.int64))
            return D(np.full(self.T, e.value, np.float32), "f32")
        if isinstance(e, BinaryExpr):
            return self._binary(e)
        if isinstance(e, TernaryExpr):
            p = self.pred(e.cond)
            a, b = self.expr(e.if_true), self.expr(e.if_false)
            if isinstance(a, Idx) and isinstance(b, Idx):
                return Idx(np.where(p, a.a, b.a))
            va, vb = self._as_data(self._boolwrap(a)), self._as_data(self._boolwrap(b))
            dtype = va.dtype if va.dtype == vb.dtype else "f32"
            return D(np.where(p, to_dtype(va.a, va.dtype, dtype), to_dtype(vb.a, vb.dtype, dtype)),
                     dtype)
        if isinstance(e, FuncCallExpr):
            return self.apply(e.name, [self.value(a, "f32") for a in e.args], "f32")
        if isinstance(e, CastExpr) and e.dtype == "float":
            return self.value(e.expr, "f32")
        raise NotImplementedError(f"oracle: expression {e!r}")

    @staticmethod
    def _boolwrap(v: Any) -> Any:
        if isinstance(v, np.ndarray) and v.dtype == np.bool_:
            return D(v, "bool")
        return v

    def _binary(self, e: BinaryExpr) -> Any:
        if e.op in ("&&", "||"):
            a, b = self.pred(e.left), self.pred(e.right)
            return (a & b) if e.op == "&&" else (a | b)
        a, b = self.expr(e.left), self.expr(e.right)
        if isinstance(a, Idx) and isinstance(b, Idx):
            x, y = a.a, b.a
            if e.op in CMP_SYMBOL:
                return CMP_SYMBOL[e.op](x, y)
            if e.op == "+":
                return Idx(x + y)
            if e.op == "-":
                return Idx(x - y)
            if e.op == "*":
                return Idx(x * y)
            if e.op in ("/", "//"):
                return Idx(x // y)
            if e.op == "%":
                return Idx(x % y)
            raise NotImplementedError(f"oracle: index expression {e!r}")
        da = self._as_data(self._boolwrap(a))
        db = self._as_data(self._boolwrap(b))
        x, y = to_dtype(da.a, da.dtype, "f32"), to_dtype(db.a, db.dtype, "f32")
        if e.op in CMP_SYMBOL:
            return CMP_SYMBOL[e.op](x, y)
        sym = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide"}
        if e.op in sym:
            return self.apply(sym[e.op], [D(x, "f32"), D(y, "f32")], "f32")
        raise NotImplementedError(f"oracle: f32 expression {e!r}")

    def value(self, e: Expr, dtype: str) -> D:
        if isinstance(e, Literal) and e.dtype != "bool" and not isinstance(e.value, bool):
            return D(to_dtype(np.full(self.T, float(e.value)), "f64", dtype)
                     if dtype != "f32" else np.full(self.T, np.float32(e.value)), dtype)
        v = self._as_data(self._boolwrap(self.expr(e)))
        return D(to_dtype(v.a, v.dtype, dtype), dtype)

    def idx(self, e: Expr) -> np.ndarray:
        v = self.expr(e)
        if isinstance(v, Idx):
            return v.a
        if isinstance(v, D) and v.dtype not in FLOATS and v.dtype != "bool":
            return np.asarray(v.a, np.int64)
        raise NotImplementedError(f"oracle: index expression {e!r} is not an integer")

    def pred(self, e: Expr) -> np.ndarray:
        v = self.expr(e)
        if isinstance(v, np.ndarray) and v.dtype == np.bool_:
            return v
        if isinstance(v, Idx):
            return v.a != 0
        if isinstance(v, D):
            return to_dtype(v.a, v.dtype, "bool")
        return np.full(self.T, bool(v))


def run_kernel(graph: Graph | dict[str, Any], meta: dict[str, Any],
               inputs: dict[str, np.ndarray], no_fusion: bool = False) -> dict[str, np.ndarray]:
    """The output buffers of the meta.json kernel on ``inputs`` (bf16 as uint16 bits or f32)."""
    return Interpreter(graph, meta, inputs, Options(no_fusion=no_fusion)).run()


def run_problem(graphs: dict[str, Graph | dict[str, Any]], meta: dict[str, Any],
                inputs: dict[str, np.ndarray], no_fusion: bool = False
                ) -> dict[str, np.ndarray]:
    """Every buffer a meta.json problem of several kernels writes: each kernel, in meta.json
    order, runs on the inputs and on what the kernels before it wrote (its intermediates)."""
    env = dict(inputs)
    for k in meta["kernels"]:
        env.update(run_kernel(graphs[k["entry"]], meta, env, no_fusion=no_fusion))
    return {name: v for name, v in env.items() if name not in inputs}

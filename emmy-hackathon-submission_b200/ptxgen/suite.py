"""Kernel IR for the reference's problem categories beyond the five benchmark configurations.

The reference defines its problems as torch expressions, each with a NumPy formula of the
expected output and a tolerance (reference ``tools/expressions_open.py``,
``tools/expressions_closed.py``). Emmy traces each expression into Kernel IR, and the compiler
lowers that. Emmy is absent here, so this module writes Kernel IR of the same kinds directly, in
the statement shapes of the shipped IRs (``ptxgen.problems`` documents them):

* pointwise chains over one flat Tile axis, with row and column broadcasts and ConstantOp
  scalars (the ``p`` category: every op of the lowering's table, f32/f64/f16/bf16 and mixed
  dtypes, odd sizes that need the tail guard);
* one-block-per-row reductions and fused row passes (``r`` and ``f``: sum, mean, amax, sum of
  squares, softmax, log-softmax, RMS norm, layer norm, L2 norm), with rows that are not a
  multiple of the block;
* column and middle-axis reductions (a Loop over the reduced axis per output element) and a
  grid-stride reduction with an atomic Write;
* small f32 matmuls through the SIMT nest (the ``m`` category's shapes);
* fused attention, softmax(q @ kt * scale) @ v, in the shipped a01/a03 nest's shape: per query
  row an inner product over d for each key, an online-softmax update of the running max, the
  denominator and the numerators, then one reciprocal scaling (the ``a`` category, batched and
  multi-head included);
* problems of two kernels chained through ``intermediate`` buffers (reference
  ``tools/generate.py:142-144``): the grid-kernel reduce plan (per-block partials, then one
  block over them) and a two-pass softmax (row statistics, then a pointwise normalisation).

Each case keeps the reference id it stands for, its NumPy formula (restated from the
reference's ``ref`` of that id, computing in the inputs' dtypes as it does), the reference's
rtol/atol, and the bar its GPU result meets against the oracle's run of the same IR.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .ir import (Accum, Assign, Axis, BinaryExpr, Cond, Dim, Init, Let, Literal, Load, Loop,
                 Stmt, StridedLoop, TensorSpec, Tile, Write, constant_node, dt, input_node,
                 kernel_node)
from .problems import GELU_C, GELU_K, I, ProblemSpec, V, _arg, _block_reduce, _spec, add, div, \
    matmul, mul, op, rem

# --- case container ----------------------------------------------------------------------------


@dataclass
class SuiteCase:
    """A generated problem with its NumPy formula and bars."""

    spec: ProblemSpec
    ref: Callable[..., np.ndarray]  # formula of the output from the inputs, in their dtypes
    rtol: float  # the reference's tolerance of its formula
    atol: float
    bar: tuple[str, float]  # GPU against the oracle: ("exact" | "ulp" | "rel", bound)
    note: str = ""

    @property
    def out(self) -> str:
        return self.spec.meta["graph_outputs"][0]

    @property
    def out_dtype(self) -> str:
        return next(a["dtype"] for a in self.spec.kernel["args"] if a["name"] == self.out)


@dataclass
class In:
    """A graph input: ``bcast`` "rows" indexes it by the output row, "cols" by the column."""

    name: str
    dtype: str
    shape: tuple[int, ...]
    dist: Sequence[Any] = ("normal", 0.0, 1.0)
    bcast: str | None = None


@dataclass
class Step:
    name: str
    fn: str
    args: tuple[str, ...]
    dtype: str | None = "f32"


def S(name: str, fn: str, *args: str, dtype: str | None = "f32") -> Step:  # noqa: N802
    return Step(name, fn, tuple(args), dtype)


# --- pointwise ---------------------------------------------------------------------------------


@dataclass
class Pointwise:
    pid: str
    code: str
    inputs: list[In]
    out: tuple[str, str, tuple[int, ...]]  # name, dtype, shape
    steps: list[Step]
    result: str
    consts: dict[str, float] = field(default_factory=dict)
    unroll: int = 4
    block: int = 256

    def build(self) -> ProblemSpec:
        oname, odt, oshape = self.out
        n, cols = math.prod(oshape), oshape[-1]
        u = self.unroll if n % self.unroll == 0 and cols % self.unroll == 0 else 1
        a0 = V("a0")
        body: list[Stmt] = [Load((c,), c, (I(0),), dt("f32")) for c in self.consts]
        names = {i.name for i in self.inputs} | {s.name for s in self.steps}
        for j in range(u):
            sfx = f"__u{j}"
            flat = add(mul(a0, I(u)), I(j)) if u > 1 else a0
            for i in self.inputs:
                idx = {None: flat, "cols": rem(flat, I(cols)), "rows": div(flat, I(cols))}
                body.append(Load((i.name + sfx,), i.name, (idx[i.bcast],), dt(i.dtype)))
            for s in self.steps:
                args = tuple(a + sfx if a in names else a for a in s.args)
                body.append(Assign(s.name + sfx, op(s.fn), args, dt(s.dtype) if s.dtype
                                   else None))
        rdt = next((s.dtype for s in self.steps if s.name == self.result), None) or \
            next(i.dtype for i in self.inputs if i.name == self.result)
        widx = (add(mul(a0, I(u)), I(0)),) if u > 1 else (a0,)
        body.append(Write(oname, widx, tuple(f"{self.result}__u{j}" for j in range(u)),
                          dt(rdt)))
        tile = Tile((Axis("a0", Dim(n // u)),), tuple(body), None)
        args = [_arg(c, "f32", [1], data=[v]) for c, v in self.consts.items()]
        args += [_arg(i.name, i.dtype, i.shape, seed=k, dist=list(i.dist))
                 for k, i in enumerate(self.inputs)]
        args.append(_arg(oname, odt, oshape, output=True))
        return _spec(self.pid, self.code, 0, 0, f"k_{self.pid}", tile, args,
                     [i.name for i in self.inputs], [oname], dict(self.consts), self.block)


# --- row-wise (one block per row) ----------------------------------------------------------------


@dataclass
class Rowwise:
    """Passes over the rows of x [rows, cols], one block per row. A pass is
    ``("reduce", acc, op, steps, value)`` -- a strided sweep accumulating ``value`` and a block
    reduction; ``("scalar", step)`` -- a per-row value; ``("write", steps, value)`` -- a sweep
    writing ``value`` into out [rows, cols]; or ``("row", value)`` -- out [rows] from thread 0.
    Steps name the sweep's element of x ``xv``."""

    pid: str
    code: str
    x: In
    out: tuple[str, str]  # name, dtype
    passes: list[tuple[Any, ...]]
    consts: dict[str, float] = field(default_factory=dict)
    block: int = 128
    cols_in: tuple[str, ...] = ()  # f32 inputs of shape [cols], read by column in write sweeps

    def build(self) -> ProblemSpec:
        rows, cols = self.x.shape
        a0, t = V("a0"), V("a1_co")
        xdt = dt(self.x.dtype)
        odt = dt(self.out[1])
        body: list[Stmt] = [Load((c,), c, (I(0),), dt("f32")) for c in self.consts]
        body.append(Let("n_cols", Literal(float(cols), "float"), dt("f32")))
        per_row = False

        def sweep(stmts: list[Stmt]) -> StridedLoop:
            return StridedLoop(Axis("a1", Dim(cols)), t, I(self.block), tuple(stmts), False,
                               None, True)

        for k, p in enumerate(self.passes):
            # each sweep loads x under its own name
            xv = f"xv{k}"

            names = {"xv": xv, **{c: f"{c}{k}" for c in self.cols_in}}

            def steps(ss: Sequence[Step], names: dict[str, str] = names) -> list[Stmt]:
                return [Assign(s.name, op(s.fn), tuple(names.get(a, a) for a in s.args),
                               dt(s.dtype) if s.dtype else None) for s in ss]

            def val(v: str, xv: str = xv) -> str:
                return xv if v == "xv" else v

            load = Load((xv,), "x", (a0, V("a1")), xdt)
            if p[0] == "reduce":
                _, acc, fn, ss, value = p
                body.append(sweep([load, *steps(ss),
                                   Accum(acc, val(value), op(fn), dt("f32"), ("a1",), None)]))
                body += _block_reduce(acc, fn, self.block, f"{acc}_smem")
            elif p[0] == "scalar":
                body += steps([p[1]])
            elif p[0] == "write":
                _, ss, value = p
                col_loads = [Load((f"{c}{k}",), c, (V("a1"),), dt("f32")) for c in self.cols_in]
                body.append(sweep([load, *col_loads, *steps(ss),
                                   Write(self.out[0], (a0, V("a1")), (val(value),), odt)]))
            elif p[0] == "row":
                per_row = True
                body.append(Cond(BinaryExpr("==", t, I(0)),
                                 (Write(self.out[0], (a0,), (p[1],), odt),), ()))
            else:
                raise ValueError(f"pass {k}: {p[0]!r}")
        tile = Tile((Axis("a0", Dim(rows)), Axis("a1_co", Dim(self.block))), tuple(body),
                    self.block)
        oshape = [rows] if per_row else [rows, cols]
        args = [_arg(c, "f32", [1], data=[v]) for c, v in self.consts.items()]
        args += [_arg("x", self.x.dtype, self.x.shape, seed=0, dist=list(self.x.dist))]
        args += [_arg(c, "f32", [cols], seed=k + 1) for k, c in enumerate(self.cols_in)]
        args.append(_arg(self.out[0], self.out[1], oshape, output=True))
        return _spec(self.pid, self.code, 0, 0, f"k_{self.pid}", tile, args,
                     ["x", *self.cols_in], [self.out[0]], dict(self.consts), self.block)


# --- reductions along other axes -------------------------------------------------------------


def axis_reduce(pid: str, code: str, shape: tuple[int, int, int], fn: str, mean: bool,
                dtype: str = "f32", block: int = 128) -> ProblemSpec:
    """out[a, c] = fn over b of x[a, b, c] (mean: divided by the extent of b): one thread per
    output element, a Loop over the reduced axis into an Init'ed accumulator. A leading extent
    of 1 makes it a column reduction of a [b, c] matrix."""
    na, nb, nc = shape
    a0 = V("a0")
    ia, ic = div(a0, I(nc)), rem(a0, I(nc))
    identity = {"add": 0.0, "maximum": -math.inf, "minimum": math.inf}[fn]
    body: list[Stmt] = [
        Init("acc0", identity, dt("f32")),
        Loop(Axis("a1", Dim(nb)), (Load(("xv",), "x", (ia, V("a1"), ic), dt(dtype)),
                                   Accum("acc0", "xv", op(fn), dt("f32"), ("a1",), None))),
    ]
    value = "acc0"
    if mean:
        body += [Let("n_b", Literal(float(nb), "float"), dt("f32")),
                 Assign("mean0", op("divide"), ("acc0", "n_b"), dt("f32"))]
        value = "mean0"
    body.append(Write("out", (a0,), (value,), dt("f32")))
    tile = Tile((Axis("a0", Dim(na * nc)),), tuple(body), None)
    args = [_arg("x", dtype, [na, nb, nc], seed=0), _arg("out", "f32", [na, nc], output=True)]
    return _spec(pid, code, 0, 0, f"k_{pid}", tile, args, ["x"], ["out"], {}, block)


def grid_reduce(pid: str, code: str, n: int, square: bool, block: int = 256,
                blocks: int = 64) -> ProblemSpec:
    """sum(x) or sum(x*x) over n f32: a grid-stride sweep per thread, a block reduction and an
    atomic add of each block's total into the zeroed output (Emmy's grid-atomic plan)."""
    ab, at = V("a0_b"), V("a0_t")
    sweep: list[Stmt] = [Load(("xv",), "x", (V("a0"),), dt("f32"))]
    value = "xv"
    if square:
        sweep.append(Assign("sq", op("multiply"), ("xv", "xv"), dt("f32")))
        value = "sq"
    sweep.append(Accum("acc0", value, op("add"), dt("f32"), ("a0",), None))
    body: list[Stmt] = [
        StridedLoop(Axis("a0", Dim(n)), add(mul(ab, I(block)), at), I(block * blocks),
                    tuple(sweep), False, None, True),
        *_block_reduce("acc0", "add", block, "acc0_smem"),
        Cond(BinaryExpr("==", at, I(0)), (Write("out", (), ("acc0",), dt("f32"), True),), ()),
    ]
    tile = Tile((Axis("a0_b", Dim(blocks)), Axis("a0_t", Dim(block))), tuple(body), block)
    args = [_arg("x", "f32", [n], seed=0), _arg("out", "f32", [1], output=True)]
    return _spec(pid, code, 0, 0, f"k_{pid}", tile, args, ["x"], ["out"], {}, block,
                 zero_outputs=["out"])


# --- the cases -----------------------------------------------------------------------------------

SQRT1_2 = 1.0 / math.sqrt(2.0)


def _erf(x: np.ndarray) -> np.ndarray:
    return np.vectorize(math.erf, otypes=[np.float64])(x)


def _d(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float64)


def _softmax(x: np.ndarray) -> np.ndarray:
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def _pw(pid: str, code: str, inputs: list[In], out: tuple[str, str, tuple[int, ...]],
        steps: list[Step], result: str, ref: Callable[..., np.ndarray], rtol: float,
        atol: float, bar: tuple[str, float], consts: dict[str, float] | None = None,
        note: str = "") -> Callable[[], SuiteCase]:
    return lambda: SuiteCase(Pointwise(pid, code, inputs, out, steps, result,
                                       consts or {}).build(), ref, rtol, atol, bar, note)


def _x(n: int | tuple[int, ...], dtype: str = "f32", name: str = "x", **kw: Any) -> In:
    return In(name, dtype, (n,) if isinstance(n, int) else n, **kw)


EXACT, FAST, FAST_REL = ("exact", 0.0), ("ulp", 4.0), ("rel", 2e-5)
f16x, bf16x = "f16", "bf16"

POINTWISE: dict[str, Callable[[], SuiteCase]] = {
    "p00_small_sub": _pw("p00_small_sub", "torch.randn(64) - torch.randn(64)",
                         [_x(64), _x(64, name="y")], ("out", "f32", (64,)),
                         [S("v0", "subtract", "x", "y")], "v0",
                         lambda x, y: x - y, 0, 0, EXACT),
    "p01_odd_add": _pw("p01_odd_add", "torch.randn(1000) + torch.randn(1000)",
                       [_x(1000), _x(1000, name="y")], ("out", "f32", (1000,)),
                       [S("v0", "add", "x", "y")], "v0", lambda x, y: x + y, 0, 0, EXACT),
    "p02_v2_mul": _pw("p02_v2_mul", "torch.randn(1538) * torch.randn(1538)",
                      [_x(1538), _x(1538, name="y")], ("out", "f32", (1538,)),
                      [S("v0", "multiply", "x", "y")], "v0", lambda x, y: x * y, 0, 0, EXACT),
    "p03_div": _pw("p03_div", "x / y", [_x(2048), _x(2048, name="y")], ("out", "f32", (2048,)),
                   [S("v0", "divide", "x", "y")], "v0", lambda x, y: x / y, 1e-6, 1e-6, EXACT),
    "p04_max_min": _pw("p04_max_min", "torch.maximum(x, y) - torch.minimum(x, y)",
                       [_x(4096), _x(4096, name="y")], ("out", "f32", (4096,)),
                       [S("v0", "maximum", "x", "y"), S("v1", "minimum", "x", "y"),
                        S("v2", "subtract", "v0", "v1")], "v2",
                       lambda x, y: np.maximum(x, y) - np.minimum(x, y), 0, 0, EXACT),
    "p06_bias_bcast": _pw("p06_bias_bcast", "x + b (x [64, 256], b [256])",
                          [_x((64, 256)), In("b", "f32", (256,), bcast="cols")],
                          ("out", "f32", (64, 256)), [S("v0", "add", "x", "b")], "v0",
                          lambda x, b: x + b, 0, 0, EXACT),
    "p07_fma3": _pw("p07_fma3", "a * b + c", [_x(8192, name="a"), _x(8192, name="b"),
                                              _x(8192, name="c")], ("out", "f32", (8192,)),
                    [S("v0", "multiply", "a", "b"), S("v1", "add", "v0", "c")], "v1",
                    lambda a, b, c: a * b + c, 1e-6, 1e-6, EXACT),
    # this backend fuses only an add of a product: a subtract of one stays a mul and a sub
    "p09_fms": _pw("p09_fms", "a * b - c", [_x(8192, name="a"), _x(8192, name="b"),
                                            _x(8192, name="c")], ("out", "f32", (8192,)),
                   [S("v0", "multiply", "a", "b"), S("v1", "subtract", "v0", "c")], "v1",
                   lambda a, b, c: a * b - c, 1e-6, 1e-6, EXACT),
    "p08_relu_affine_odd": _pw("p08_relu_affine_odd", "torch.relu(x * 0.5 - 0.25)",
                               [_x(3000)], ("out", "f32", (3000,)),
                               [S("v0", "multiply", "x", "mul_c1"),
                                S("v1", "subtract", "v0", "sub_c1"), S("v2", "relu", "v1")],
                               "v2", lambda x: np.maximum(x * 0.5 - 0.25, 0), 1e-6, 1e-6, EXACT,
                               {"mul_c1": 0.5, "sub_c1": 0.25}),
    "p09_exp": _pw("p09_exp", "torch.exp(x)", [_x(4096)], ("out", "f32", (4096,)),
                   [S("v0", "exp", "x")], "v0", np.exp, 1e-5, 1e-5, FAST),
    "p10_inv_norm": _pw("p10_inv_norm", "1.0 / torch.sqrt(x * x + 1.0)", [_x(2048)],
                        ("out", "f32", (2048,)),
                        [S("v0", "multiply", "x", "x"), S("v1", "add", "v0", "add_c1"),
                         S("v2", "sqrt", "v1"), S("v3", "divide", "div_c1", "v2")], "v3",
                        lambda x: 1.0 / np.sqrt(x * x + 1.0), 1e-5, 1e-5, EXACT,
                        {"add_c1": 1.0, "div_c1": 1.0}),
    "p12_neg": _pw("p12_neg", "-x", [_x(1024)], ("out", "f32", (1024,)),
                   [S("v0", "negative", "x")], "v0", lambda x: -x, 0, 0, EXACT),
    "p13_square": _pw("p13_square", "torch.square(x)", [_x(2048)], ("out", "f32", (2048,)),
                      [S("v0", "square", "x")], "v0", lambda x: x * x, 0, 0, EXACT),
    "p14_abs": _pw("p14_abs", "torch.abs(x)", [_x(2048)], ("out", "f32", (2048,)),
                   [S("v0", "abs", "x")], "v0", np.abs, 0, 0, EXACT),
    "p15_rsqrt": _pw("p15_rsqrt", "torch.rsqrt(x * x + 1.0)", [_x(2048)],
                     ("out", "f32", (2048,)),
                     [S("v0", "multiply", "x", "x"), S("v1", "add", "v0", "add_c1"),
                      S("v2", "rsqrt", "v1")], "v2", lambda x: 1.0 / np.sqrt(x * x + 1.0),
                     1e-5, 1e-5, FAST, {"add_c1": 1.0}),
    "p16_log": _pw("p16_log", "torch.log(x * x + 1.0) * 0.5", [_x(2048)],
                   ("out", "f32", (2048,)),
                   [S("v0", "multiply", "x", "x"), S("v1", "add", "v0", "add_c1"),
                    S("v2", "log", "v1"), S("v3", "multiply", "v2", "mul_c1")], "v3",
                   lambda x: np.log(x * x + 1.0) * 0.5, 1e-5, 1e-5, FAST_REL,
                   {"add_c1": 1.0, "mul_c1": 0.5}),
    "p17_sin_cos": _pw("p17_sin_cos", "torch.sin(x) + torch.cos(y)",
                       [_x(4096), _x(4096, name="y")], ("out", "f32", (4096,)),
                       [S("v0", "sin", "x"), S("v1", "cos", "y"), S("v2", "add", "v0", "v1")],
                       "v2", lambda x, y: np.sin(x) + np.cos(y), 1e-5, 1e-5, FAST_REL),
    "p18_tanh": _pw("p18_tanh", "torch.tanh(x)", [_x(4096)], ("out", "f32", (4096,)),
                    [S("v0", "tanh", "x")], "v0", np.tanh, 1e-5, 1e-5, FAST_REL),
    "p19_sigmoid": _pw("p19_sigmoid", "torch.sigmoid(x)", [_x(4096)], ("out", "f32", (4096,)),
                       [S("v0", "sigmoid", "x")], "v0", lambda x: 1 / (1 + np.exp(-x)),
                       1e-5, 1e-5, FAST),
    "p20_silu_odd": _pw("p20_silu_odd", "torch.nn.functional.silu(x)", [_x(3000)],
                        ("out", "f32", (3000,)),
                        [S("v0", "sigmoid", "x"), S("v1", "multiply", "x", "v0")], "v1",
                        lambda x: x / (1 + np.exp(-x)), 1e-5, 1e-5, FAST),
    "p21_gelu": _pw("p21_gelu", "torch.nn.functional.gelu(x)", [_x(4096)],
                    ("out", "f32", (4096,)),
                    [S("v0", "multiply", "x", "c_rsqrt2"), S("v1", "erf", "v0"),
                     S("v2", "add", "v1", "c_one"), S("v3", "multiply", "x", "c_half"),
                     S("v4", "multiply", "v3", "v2")], "v4",
                    lambda x: 0.5 * x * (1.0 + _erf(x * SQRT1_2)), 1e-5, 1e-5, FAST_REL,
                    {"c_rsqrt2": SQRT1_2, "c_one": 1.0, "c_half": 0.5},
                    "erf by Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7), as the reference's "
                    "fastmath.erf"),
    "p23_sigmoid_gate": _pw("p23_sigmoid_gate", "torch.sigmoid(x) * torch.tanh(y)",
                            [_x((64, 256)), _x((64, 256), name="y")],
                            ("out", "f32", (64, 256)),
                            [S("v0", "sigmoid", "x"), S("v1", "tanh", "y"),
                             S("v2", "multiply", "v0", "v1")], "v2",
                            lambda x, y: np.tanh(y) / (1 + np.exp(-x)), 1e-5, 1e-5, FAST_REL),
    "p24_add_f64": _pw("p24_add_f64", "f64 a + b", [_x(4096, "f64", name="a"),
                                                    _x(4096, "f64", name="b")],
                       ("out", "f64", (4096,)), [S("v0", "add", "a", "b", dtype="f64")], "v0",
                       lambda a, b: a + b, 0, 0, EXACT),
    "p25_fma_f64_odd": _pw("p25_fma_f64_odd", "f64 a * b + c",
                           [_x(3000, "f64", name="a"), _x(3000, "f64", name="b"),
                            _x(3000, "f64", name="c")], ("out", "f64", (3000,)),
                           [S("v0", "multiply", "a", "b", dtype="f64"),
                            S("v1", "add", "v0", "c", dtype="f64")], "v1",
                           lambda a, b, c: a * b + c, 1e-12, 1e-12, EXACT),
    "p26_exp_f64": _pw("p26_exp_f64", "torch.exp(x) in f64", [_x(4096, "f64")],
                       ("out", "f64", (4096,)), [S("v0", "exp", "x", dtype="f64")], "v0",
                       np.exp, 1e-6, 1e-6, FAST_REL,
                       note="the reference's dtype rule computes an f64 op without an f64 PTX "
                            "form (exp) in f32 (reference ptxgen/ops.py:173-192), so the "
                            "formula holds to f32 accuracy, not the reference's rtol 1e-10"),
    "p27_add_bf16": _pw("p27_add_bf16", "bf16 a + b", [_x(2048, bf16x, name="a"),
                                                       _x(2048, bf16x, name="b")],
                        ("out", "bf16", (2048,)), [S("v0", "add", "a", "b", dtype="bf16")],
                        "v0", lambda a, b: a + b, 1e-2, 1e-2, EXACT),
    "p28_relu_affine_bf16_odd": _pw("p28_relu_affine_bf16_odd", "relu(bf16 x * 0.5 - 0.25)",
                                    [_x(3000, bf16x)], ("out", "bf16", (3000,)),
                                    [S("v0", "multiply", "x", "mul_c1", dtype="bf16"),
                                     S("v1", "subtract", "v0", "sub_c1", dtype="bf16"),
                                     S("v2", "relu", "v1", dtype="bf16")], "v2",
                                    lambda x: np.maximum(x * 0.5 - 0.25, 0), 1e-2, 1e-2, EXACT,
                                    {"mul_c1": 0.5, "sub_c1": 0.25}),
    "p29_sigmoid_bf16": _pw("p29_sigmoid_bf16", "torch.sigmoid(bf16 x)", [_x(4096, bf16x)],
                            ("out", "bf16", (4096,)), [S("v0", "sigmoid", "x", dtype="bf16")],
                            "v0", lambda x: 1 / (1 + np.exp(-x)), 1e-2, 1e-2, ("ulp", 1)),
    "p30_add_f16": _pw("p30_add_f16", "f16 a + b", [_x(2048, f16x, name="a"),
                                                    _x(2048, f16x, name="b")],
                       ("out", "f16", (2048,)), [S("v0", "add", "a", "b", dtype="f16")], "v0",
                       lambda a, b: a + b, 1e-3, 1e-3, EXACT),
    "p31_tanh_f16": _pw("p31_tanh_f16", "torch.tanh(f16 x)", [_x(4096, f16x)],
                        ("out", "f16", (4096,)), [S("v0", "tanh", "x", dtype="f16")], "v0",
                        np.tanh, 1e-3, 1e-3, ("rel", 1e-3)),
    "p32_bf16_to_f32": _pw("p32_bf16_to_f32", "x.float() * y (x bf16)",
                           [_x(4096, bf16x), _x(4096, name="y")], ("out", "f32", (4096,)),
                           [S("v0", "cast", "x"), S("v1", "multiply", "v0", "y")], "v1",
                           lambda x, y: x * y, 1e-6, 1e-6, EXACT),
    "p37_div": _pw("p37_div", "a / (b.abs() + 1.0)", [_x(1024, name="a"), _x(1024, name="b")],
                   ("out", "f32", (1024,)),
                   [S("v0", "abs", "b"), S("v1", "add", "v0", "add_c1"),
                    S("v2", "divide", "a", "v1")], "v2",
                   lambda a, b: a / (np.abs(b) + 1.0), 1e-6, 1e-6, EXACT, {"add_c1": 1.0}),
    "p44_leaky_where": _pw("p44_leaky_where", "torch.where(x > 0, x, 0.01 * x)", [_x(4096)],
                           ("out", "f32", (4096,)),
                           [S("v0", "greater", "x", "c_zero", dtype="bool"),
                            S("v1", "multiply", "x", "c_slope"),
                            S("v2", "where", "v0", "x", "v1")], "v2",
                           lambda x: np.where(x > 0, x, 0.01 * x), 1e-6, 1e-6, EXACT,
                           {"c_zero": 0.0, "c_slope": 0.01}),
    "p50_clamp": _pw("p50_clamp", "torch.clamp(x, -0.5, 0.5)", [_x(4096)],
                     ("out", "f32", (4096,)),
                     [S("v0", "maximum", "x", "c_lo"), S("v1", "minimum", "v0", "c_hi")], "v1",
                     lambda x: np.clip(x, -0.5, 0.5), 0, 0, EXACT,
                     {"c_lo": -0.5, "c_hi": 0.5}),
    "p52_swiglu": _pw("p52_swiglu", "silu(a) * b", [_x((32, 512), name="a"),
                                                    _x((32, 512), name="b")],
                      ("out", "f32", (32, 512)),
                      [S("v0", "sigmoid", "a"), S("v1", "multiply", "a", "v0"),
                       S("v2", "multiply", "v1", "b")], "v2",
                      lambda a, b: a / (1 + np.exp(-a)) * b, 1e-5, 1e-5, FAST_REL),
    "p54_residual_scale": _pw("p54_residual_scale", "x + 0.5 * r * s (s per row)",
                              [_x((64, 256)), _x((64, 256), name="r"),
                               In("s", "f32", (64,), bcast="rows")],
                              ("out", "f32", (64, 256)),
                              [S("v0", "multiply", "r", "c_half"),
                               S("v1", "multiply", "v0", "s"), S("v2", "add", "x", "v1")],
                              "v2", lambda x, r, s: x + 0.5 * r * s[:, None], 1e-6, 1e-6,
                              EXACT, {"c_half": 0.5}),
    "p57_pow": _pw("p57_pow", "torch.pow(x.abs() + 0.5, 1.5)", [_x(4096)],
                   ("out", "f32", (4096,)),
                   [S("v0", "abs", "x"), S("v1", "add", "v0", "c_half"),
                    S("v2", "pow", "v1", "c_exp")], "v2",
                   lambda x: (np.abs(x) + 0.5) ** 1.5, 1e-5, 1e-5, FAST_REL,
                   {"c_half": 0.5, "c_exp": 1.5}),
    "p61_f16_silu": _pw("p61_f16_silu", "silu(f16 x)", [_x(4096, f16x)],
                        ("out", "f16", (4096,)),
                        [S("v0", "sigmoid", "x", dtype="f16"),
                         S("v1", "multiply", "x", "v0", dtype="f16")], "v1",
                        lambda x: x / (1 + np.exp(-x)), 1e-3, 1e-3, ("rel", 1e-3)),
    "p00_scalar_add": _pw("p00_scalar_add", "torch.randn(128) + torch.randn(128)",
                          [_x(128, name="a"), _x(128, name="b")], ("out", "f32", (128,)),
                          [S("v0", "add", "a", "b")], "v0", lambda a, b: a + b, 0, 0, EXACT),
    "p01_vector_add": _pw("p01_vector_add", "torch.randn(1024) + torch.randn(1024)",
                          [_x(1024, name="a"), _x(1024, name="b")], ("out", "f32", (1024,)),
                          [S("v0", "add", "a", "b")], "v0", lambda a, b: a + b, 0, 0, EXACT),
    "p03_relu_mul": _pw("p03_relu_mul", "torch.relu(x) * y", [_x(2048), _x(2048, name="y")],
                        ("out", "f32", (2048,)),
                        [S("v0", "relu", "x"), S("v1", "multiply", "v0", "y")], "v1",
                        lambda x, y: np.maximum(x, 0) * y, 0, 0, EXACT),
    # --- the reference's remaining pointwise ids (formulas in f64 where its ``ref`` lifts
    # to f64, cast back to f32) ---
    "p05_add_2d": _pw("p05_add_2d", "torch.randn(64, 128) + torch.randn(64, 128)",
                      [_x((64, 128), name="a"), _x((64, 128), name="b")],
                      ("out", "f32", (64, 128)), [S("v0", "add", "a", "b")], "v0",
                      lambda a, b: a + b, 0, 0, EXACT),
    "p11_big_add": _pw("p11_big_add", "torch.randn(1 << 20) + torch.randn(1 << 20)",
                       [_x(1 << 20, name="a"), _x(1 << 20, name="b")],
                       ("out", "f32", (1 << 20,)), [S("v0", "add", "a", "b")], "v0",
                       lambda a, b: a + b, 0, 0, EXACT),
    "p22_gelu_tanh": _pw("p22_gelu_tanh", 'gelu(torch.randn(4096), approximate="tanh")',
                         [_x(4096)], ("out", "f32", (4096,)),
                         [S("v0", "multiply", "x", "x"), S("v1", "multiply", "v0", "x"),
                          S("v2", "multiply", "c_cube", "v1"), S("v3", "add", "x", "v2"),
                          S("v4", "multiply", "c_k", "v3"), S("v5", "tanh", "v4"),
                          S("v6", "add", "v5", "c_one"), S("v7", "multiply", "c_half", "x"),
                          S("v8", "multiply", "v7", "v6")], "v8",
                         lambda x: (0.5 * x * (1.0 + np.tanh(GELU_K * (
                             x + GELU_C * x.astype(np.float64) ** 3)))).astype(np.float32),
                         1e-5, 1e-5, FAST_REL,
                         {"c_cube": GELU_C, "c_k": GELU_K, "c_one": 1.0, "c_half": 0.5}),
    "p33_sub_2d": _pw("p33_sub_2d", "x - y (x, y [64, 128])",
                      [_x((64, 128)), _x((64, 128), name="y")], ("out", "f32", (64, 128)),
                      [S("v0", "subtract", "x", "y")], "v0", lambda x, y: x - y, 0, 0, EXACT),
    "p34_sigmoid": _pw("p34_sigmoid", "torch.sigmoid(torch.randn(2048))", [_x(2048)],
                       ("out", "f32", (2048,)), [S("v0", "sigmoid", "x")], "v0",
                       lambda x: (1 / (1 + np.exp(-_d(x)))).astype(np.float32), 1e-5, 1e-6,
                       FAST),
    "p35_tanh": _pw("p35_tanh", "torch.tanh(torch.randn(2048))", [_x(2048)],
                    ("out", "f32", (2048,)), [S("v0", "tanh", "x")], "v0",
                    lambda x: np.tanh(_d(x)).astype(np.float32), 1e-5, 1e-6, FAST_REL),
    "p36_silu": _pw("p36_silu", "x * torch.sigmoid(x)", [_x(4096)], ("out", "f32", (4096,)),
                    [S("v0", "sigmoid", "x"), S("v1", "multiply", "x", "v0")], "v1",
                    lambda x: (_d(x) / (1 + np.exp(-_d(x)))).astype(np.float32), 1e-5, 1e-6,
                    FAST),
    "p38_bias_bcast": _pw("p38_bias_bcast", "x + b (x [32, 256], b [256])",
                          [_x((32, 256)), In("b", "f32", (256,), bcast="cols")],
                          ("out", "f32", (32, 256)), [S("v0", "add", "x", "b")], "v0",
                          lambda x, b: x + b, 0, 0, EXACT),
    "p39_odd_mul": _pw("p39_odd_mul", "torch.randn(1000) * torch.randn(1000)",
                       [_x(1000, name="a"), _x(1000, name="b")], ("out", "f32", (1000,)),
                       [S("v0", "multiply", "a", "b")], "v0", lambda a, b: a * b, 0, 0, EXACT),
    "p40_odd_add_const": _pw("p40_odd_add_const", "torch.randn(999) + 1.5", [_x(999)],
                             ("out", "f32", (999,)), [S("v0", "add", "x", "add_c1")], "v0",
                             lambda x: x + np.float32(1.5), 0, 0, EXACT, {"add_c1": 1.5}),
    "p41_maximum": _pw("p41_maximum", "torch.maximum(torch.randn(2048), torch.randn(2048))",
                       [_x(2048, name="a"), _x(2048, name="b")], ("out", "f32", (2048,)),
                       [S("v0", "maximum", "a", "b")], "v0", np.maximum, 0, 0, EXACT),
    "p42_sqrt_abs": _pw("p42_sqrt_abs", "torch.sqrt(torch.randn(2048).abs())", [_x(2048)],
                        ("out", "f32", (2048,)), [S("v0", "abs", "x"), S("v1", "sqrt", "v0")],
                        "v1", lambda x: np.sqrt(np.abs(x)), 1e-6, 1e-6, EXACT),
    "p43_square_shift": _pw("p43_square_shift", "(x - 0.5) * (x - 0.5)", [_x(4096)],
                            ("out", "f32", (4096,)),
                            [S("v0", "subtract", "x", "sub_c1"),
                             S("v1", "multiply", "v0", "v0")], "v1",
                            lambda x: (x - np.float32(0.5)) * (x - np.float32(0.5)), 1e-6,
                            1e-6, EXACT, {"sub_c1": 0.5}),
    "p45_rsqrt": _pw("p45_rsqrt", "torch.rsqrt(torch.randn(1024).abs() + 1.0)", [_x(1024)],
                     ("out", "f32", (1024,)),
                     [S("v0", "abs", "x"), S("v1", "add", "v0", "add_c1"),
                      S("v2", "rsqrt", "v1")], "v2",
                     lambda x: (1 / np.sqrt(np.abs(_d(x)) + 1.0)).astype(np.float32), 1e-5,
                     1e-6, FAST, {"add_c1": 1.0}),
    "p46_log": _pw("p46_log", "torch.log(torch.randn(1024).abs() + 1.0)", [_x(1024)],
                   ("out", "f32", (1024,)),
                   [S("v0", "abs", "x"), S("v1", "add", "v0", "add_c1"), S("v2", "log", "v1")],
                   "v2", lambda x: np.log(np.abs(_d(x)) + 1.0).astype(np.float32), 1e-5, 1e-6,
                   FAST_REL, {"add_c1": 1.0}),
    "p47_gelu": _pw("p47_gelu", "torch.nn.functional.gelu(torch.randn(2048))", [_x(2048)],
                    ("out", "f32", (2048,)),
                    [S("v0", "multiply", "x", "c_rsqrt2"), S("v1", "erf", "v0"),
                     S("v2", "add", "v1", "c_one"), S("v3", "multiply", "x", "c_half"),
                     S("v4", "multiply", "v3", "v2")], "v4",
                    lambda x: (0.5 * _d(x) * (1 + _erf(_d(x) / np.sqrt(2.0)))).astype(
                        np.float32), 1e-4, 1e-5, FAST_REL,
                    {"c_rsqrt2": SQRT1_2, "c_one": 1.0, "c_half": 0.5}),
    "p48_3d_mul": _pw("p48_3d_mul", "torch.randn(4, 16, 64) * torch.randn(4, 16, 64)",
                      [_x((4, 16, 64), name="a"), _x((4, 16, 64), name="b")],
                      ("out", "f32", (4, 16, 64)), [S("v0", "multiply", "a", "b")], "v0",
                      lambda a, b: a * b, 0, 0, EXACT),
    "p49_fma3": _pw("p49_fma3", "a * b + c (512)", [_x(512, name="a"), _x(512, name="b"),
                                                    _x(512, name="c")], ("out", "f32", (512,)),
                    [S("v0", "multiply", "a", "b"), S("v1", "add", "v0", "c")], "v1",
                    lambda a, b, c: a * b + c, 1e-6, 1e-6, EXACT),
    "p51_neg_abs": _pw("p51_neg_abs", "-x.abs()", [_x(3000)], ("out", "f32", (3000,)),
                       [S("v0", "abs", "x"), S("v1", "negative", "v0")], "v1",
                       lambda x: -np.abs(x), 0, 0, EXACT),
    "p53_sig_tanh": _pw("p53_sig_tanh", "torch.sigmoid(x) * torch.tanh(x) (x [4, 64])",
                        [_x((4, 64))], ("out", "f32", (4, 64)),
                        [S("v0", "sigmoid", "x"), S("v1", "tanh", "x"),
                         S("v2", "multiply", "v0", "v1")], "v2",
                        lambda x: (np.tanh(_d(x)) / (1 + np.exp(-_d(x)))).astype(np.float32),
                        1e-5, 1e-6, FAST_REL),
    "p55_f16_add": _pw("p55_f16_add", "f16 a + b (1024)", [_x(1024, f16x, name="a"),
                                                          _x(1024, f16x, name="b")],
                       ("out", "f16", (1024,)), [S("v0", "add", "a", "b", dtype="f16")], "v0",
                       lambda a, b: (a + b).astype(np.float32), 1e-3, 1e-3, EXACT),
    "p56_scalar_chain": _pw("p56_scalar_chain", "(x * 0.5 + 0.25) * 3.0 - 1.0", [_x(4096)],
                            ("out", "f32", (4096,)),
                            [S("v0", "multiply", "x", "mul_c1"), S("v1", "add", "v0", "add_c1"),
                             S("v2", "multiply", "v1", "mul_c2"),
                             S("v3", "subtract", "v2", "sub_c1")], "v3",
                            lambda x: (x * np.float32(0.5) + np.float32(0.25)) * np.float32(3.0)
                            - np.float32(1.0), 1e-6, 1e-6, EXACT,
                            {"mul_c1": 0.5, "add_c1": 0.25, "mul_c2": 3.0, "sub_c1": 1.0}),
    "p58_rsqrt_eps": _pw("p58_rsqrt_eps", "1.0 / torch.sqrt(torch.randn(1024).abs() + 1e-3)",
                         [_x(1024)], ("out", "f32", (1024,)),
                         [S("v0", "abs", "x"), S("v1", "add", "v0", "add_c1"),
                          S("v2", "sqrt", "v1"), S("v3", "divide", "div_c1", "v2")], "v3",
                         lambda x: (1 / np.sqrt(np.abs(_d(x)) + 1e-3)).astype(np.float32),
                         1e-5, 1e-6, EXACT, {"add_c1": 1e-3, "div_c1": 1.0}),
    "p59_large": _pw("p59_large", "torch.randn(1 << 20) * 2.0", [_x(1 << 20)],
                     ("out", "f32", (1 << 20,)), [S("v0", "multiply", "x", "mul_c1")], "v0",
                     lambda x: x * np.float32(2.0), 0, 0, EXACT, {"mul_c1": 2.0}),
    "p60_tiny": _pw("p60_tiny", "torch.randn(7) + torch.randn(7)",
                    [_x(7, name="a"), _x(7, name="b")], ("out", "f32", (7,)),
                    [S("v0", "add", "a", "b")], "v0", lambda a, b: a + b, 0, 0, EXACT),
}


def _rw(pid: str, code: str, shape: tuple[int, int], out: tuple[str, str],
        passes: list[tuple[Any, ...]], ref: Callable[..., np.ndarray], rtol: float, atol: float,
        bar: tuple[str, float], block: int = 128, dtype: str = "f32",
        consts: dict[str, float] | None = None,
        cols_in: tuple[str, ...] = ()) -> Callable[[], SuiteCase]:
    return lambda: SuiteCase(Rowwise(pid, code, In("x", dtype, shape), out, passes,
                                     consts or {}, block, cols_in).build(), ref, rtol, atol, bar)


def _softmax_passes(pre: Callable[[str, str], list[Step]] | None = None,
                    out_cast: str | None = None) -> list[tuple[Any, ...]]:
    """max, sum of exp(s - max), then exp(s - max) / sum, where s is x or ``pre``'s last step
    (``pre(name, x)`` gives the steps making s under ``name``); ``out_cast`` casts the result."""
    def s_of(tag: str) -> tuple[list[Step], str]:
        if pre is None:
            return [], "xv"
        ss = pre(f"s{tag}", "xv")
        return ss, ss[-1].name
    s0, v0 = s_of("0")
    s1, v1 = s_of("1")
    s2, v2 = s_of("2")
    write = [*s2, S("d2", "subtract", v2, "acc0"), S("e2", "exp", "d2"),
             S("y", "multiply", "e2", "r")]
    if out_cast:
        write.append(S("yc", "cast", "y", dtype=out_cast))
    return [("reduce", "acc0", "maximum", s0, v0),
            ("reduce", "acc1", "add", [*s1, S("d", "subtract", v1, "acc0"), S("e", "exp", "d")],
             "e"),
            ("scalar", S("r", "reciprocal", "acc1")),
            ("write", write, "yc" if out_cast else "y")]


SUM = ("reduce", "acc0", "add", [], "xv")
MAX = ("reduce", "acc0", "maximum", [], "xv")
SUMSQ = ("reduce", "acc0", "add", [S("sq", "multiply", "xv", "xv")], "sq")
ATOMIC = ("rel", 1e-6)

ROWWISE: dict[str, Callable[[], SuiteCase]] = {
    "r02_row_mean": _rw("r02_row_mean", "x.mean(dim=-1)", (64, 1024), ("out", "f32"),
                        [SUM, ("scalar", S("m", "divide", "acc0", "n_cols")), ("row", "m")],
                        lambda x: x.mean(-1), 1e-5, 1e-5, EXACT),
    "r03_row_amax": _rw("r03_row_amax", "x.amax(dim=-1)", (64, 1000), ("out", "f32"),
                        [MAX, ("row", "acc0")], lambda x: x.max(-1), 0, 0, EXACT),
    "r04_row_sum_odd": _rw("r04_row_sum_odd", "x.sum(dim=-1)", (37, 777), ("out", "f32"),
                           [SUM, ("row", "acc0")], lambda x: x.sum(-1), 1e-5, 1e-5, EXACT),
    "r05_sum_squares": _rw("r05_sum_squares", "(x * x).sum(dim=-1)", (32, 2048),
                           ("out", "f32"), [SUMSQ, ("row", "acc0")],
                           lambda x: (x * x).sum(-1), 1e-5, 1e-5, EXACT),
    "r11_t64_rows": _rw("r11_t64_rows", "x.sum(dim=-1), 64 threads a row", (128, 512),
                        ("out", "f32"), [SUM, ("row", "acc0")], lambda x: x.sum(-1),
                        1e-5, 1e-5, EXACT, block=64),
    "r12_t32_rows": _rw("r12_t32_rows", "x.sum(dim=-1), one warp a row", (128, 256),
                        ("out", "f32"), [SUM, ("row", "acc0")], lambda x: x.sum(-1),
                        1e-5, 1e-5, EXACT, block=32),
    "r21_f16_rowsum": _rw("r21_f16_rowsum", "f16 x.sum(dim=-1) in f32", (32, 1024),
                          ("out", "f32"), [SUM, ("row", "acc0")], lambda x: x.sum(-1),
                          1e-3, 1e-3, EXACT, dtype="f16"),
    "f00_softmax_1000": _rw("f00_softmax_1000", "torch.softmax(x, dim=-1)", (32, 1000),
                            ("out", "f32"),
                            [MAX, ("reduce", "acc1", "add", [S("d", "subtract", "xv", "acc0"),
                                                            S("e", "exp", "d")], "e"),
                             ("scalar", S("r", "reciprocal", "acc1")),
                             ("write", [S("d2", "subtract", "xv", "acc0"), S("e2", "exp", "d2"),
                                        S("y", "multiply", "e2", "r")], "y")],
                            _softmax, 1e-3, 1e-5, FAST_REL),
    "f01_rmsnorm_2048": _rw("f01_rmsnorm_2048", "x * rsqrt(mean(x^2) + 1e-6)", (16, 2048),
                            ("out", "f32"),
                            [SUMSQ, ("scalar", S("ms", "divide", "acc0", "n_cols")),
                             ("scalar", S("mse", "add", "ms", "c_eps")),
                             ("scalar", S("inv", "rsqrt", "mse")),
                             ("write", [S("y", "multiply", "xv", "inv")], "y")],
                            lambda x: x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6),
                            1e-4, 1e-5, FAST_REL, consts={"c_eps": 1e-6}),
    "f04_l2norm_eps": _rw("f04_l2norm_eps", "x / (x.norm(dim=-1) + 1e-6)", (32, 1024),
                          ("out", "f32"),
                          [SUMSQ, ("scalar", S("nrm", "sqrt", "acc0")),
                           ("scalar", S("den", "add", "nrm", "c_eps")),
                           ("write", [S("y", "divide", "xv", "den")], "y")],
                          lambda x: x / (np.sqrt((x * x).sum(-1, keepdims=True)) + 1e-6),
                          1e-5, 1e-5, EXACT, consts={"c_eps": 1e-6}),
    "f08_layernorm": _rw("f08_layernorm", "torch.nn.functional.layer_norm(x, (768,))",
                         (16, 768), ("out", "f32"),
                         [SUM, ("scalar", S("mu", "divide", "acc0", "n_cols")),
                          ("reduce", "acc1", "add", [S("c", "subtract", "xv", "mu"),
                                                     S("c2", "multiply", "c", "c")], "c2"),
                          ("scalar", S("var", "divide", "acc1", "n_cols")),
                          ("scalar", S("vare", "add", "var", "c_eps")),
                          ("scalar", S("inv", "rsqrt", "vare")),
                          ("write", [S("cc", "subtract", "xv", "mu"),
                                     S("y", "multiply", "cc", "inv")], "y")],
                         lambda x: (x - x.mean(-1, keepdims=True))
                         / np.sqrt(x.var(-1, keepdims=True) + 1e-5),
                         1e-4, 1e-4, FAST_REL, consts={"c_eps": 1e-5}),
    "f12_log_softmax": _rw("f12_log_softmax", "torch.log_softmax(x, dim=-1)", (32, 512),
                           ("out", "f32"),
                           [MAX, ("reduce", "acc1", "add", [S("d", "subtract", "xv", "acc0"),
                                                           S("e", "exp", "d")], "e"),
                            ("scalar", S("lse", "log", "acc1")),
                            ("write", [S("d2", "subtract", "xv", "acc0"),
                                       S("y", "subtract", "d2", "lse")], "y")],
                           lambda x: np.log(_softmax(x)), 1e-4, 1e-5, FAST_REL),
    # --- the reference's remaining row-wise, fused and whole-tensor ids; a whole-tensor
    # reduction is one row of one block (the reference's single-block plans), and leading axes
    # of a higher-rank input are flattened into rows ---
    "r01_array_sum": _rw("r01_array_sum", "torch.randn(1024).sum()", (1, 1024), ("out", "f32"),
                         [SUM, ("row", "acc0")], lambda x: _d(x).sum().astype(np.float32),
                         1e-4, 1e-4, EXACT),
    "r03_mean": _rw("r03_mean", "torch.randn(32768).mean()", (1, 32768), ("out", "f32"),
                    [SUM, ("scalar", S("m", "divide", "acc0", "n_cols")), ("row", "m")],
                    lambda x: _d(x).mean().astype(np.float32), 1e-4, 1e-4, EXACT),
    "r04_row_sum": _rw("r04_row_sum", "torch.randn(64, 512).sum(-1)", (64, 512),
                       ("out", "f32"), [SUM, ("row", "acc0")],
                       lambda x: _d(x).sum(-1).astype(np.float32), 1e-4, 1e-4, EXACT),
    "r00_sum_2048": _rw("r00_sum_2048", "torch.randn(2048).sum()", (1, 2048), ("out", "f32"),
                        [SUM, ("row", "acc0")], lambda x: _d(x).sum().astype(np.float32),
                        1e-4, 1e-4, EXACT),
    "r01_sum_odd": _rw("r01_sum_odd", "torch.randn(1000).sum()", (1, 1000), ("out", "f32"),
                       [SUM, ("row", "acc0")], lambda x: _d(x).sum().astype(np.float32),
                       1e-4, 1e-4, EXACT),
    "r07_sum_unpinned": _rw("r07_sum_unpinned", "torch.randn(65536).sum()", (1, 65536),
                            ("out", "f32"), [SUM, ("row", "acc0")],
                            lambda x: _d(x).sum().astype(np.float32), 1e-3, 1e-3, EXACT,
                            block=256),
    "r08_row_sum_short": _rw("r08_row_sum_short", "torch.randn(64, 32).sum(-1)", (64, 32),
                             ("out", "f32"), [SUM, ("row", "acc0")],
                             lambda x: _d(x).sum(-1).astype(np.float32), 1e-4, 1e-4, EXACT),
    "r09_row_sum_unpinned": _rw("r09_row_sum_unpinned", "torch.randn(256, 512).sum(-1)",
                                (256, 512), ("out", "f32"), [SUM, ("row", "acc0")],
                                lambda x: _d(x).sum(-1).astype(np.float32), 1e-4, 1e-4,
                                EXACT),
    "r10_t256": _rw("r10_t256", "torch.randn(4096).sum(), 256 threads", (1, 4096),
                    ("out", "f32"), [SUM, ("row", "acc0")],
                    lambda x: _d(x).sum().astype(np.float32), 1e-4, 1e-4, EXACT, block=256),
    "r13_t512_mean": _rw("r13_t512_mean", "torch.randn(65536).mean(), 512 threads",
                         (1, 65536), ("out", "f32"),
                         [SUM, ("scalar", S("m", "divide", "acc0", "n_cols")), ("row", "m")],
                         lambda x: _d(x).mean().astype(np.float32), 1e-4, 1e-4, EXACT,
                         block=512),
    "r14_coop_t": _rw("r14_coop_t", "torch.randn(64, 512).sum(-1), cooperating threads",
                      (64, 512), ("out", "f32"), [SUM, ("row", "acc0")],
                      lambda x: _d(x).sum(-1).astype(np.float32), 1e-4, 1e-4, EXACT),
    "r15_coop_r2": _rw("r15_coop_r2", "torch.randn(8192).sum(), cooperating threads",
                       (1, 8192), ("out", "f32"), [SUM, ("row", "acc0")],
                       lambda x: _d(x).sum().astype(np.float32), 1e-4, 1e-4, EXACT),
    "r18_amax_4d": _rw("r18_amax_4d", "torch.randn(2, 4, 8, 256).amax(-1)", (64, 256),
                       ("out", "f32"), [MAX, ("row", "acc0")], lambda x: x.max(-1), 0, 0,
                       EXACT),
    "r20_sig_tanh_sum": _rw("r20_sig_tanh_sum", "(sigmoid(x) * tanh(x)).sum(-1) (x [4, 64])",
                            (4, 64), ("out", "f32"),
                            [("reduce", "acc0", "add",
                              [S("sg", "sigmoid", "xv"), S("th", "tanh", "xv"),
                               S("pr", "multiply", "sg", "th")], "pr"), ("row", "acc0")],
                            lambda x: (np.tanh(_d(x)) / (1 + np.exp(-_d(x)))).sum(-1).astype(
                                np.float32), 1e-4, 1e-4, FAST_REL, block=64),
    "f01_rmsnorm": _rw("f01_rmsnorm", "x / sqrt((x * x).mean(-1) + 1e-5) * w (x [64, 1024])",
                       (64, 1024), ("out", "f32"),
                       [SUMSQ, ("scalar", S("ms", "divide", "acc0", "n_cols")),
                        ("scalar", S("mse", "add", "ms", "c_eps")),
                        ("scalar", S("den", "sqrt", "mse")),
                        ("write", [S("q", "divide", "xv", "den"), S("y", "multiply", "q", "w")],
                         "y")],
                       lambda x, w: (x / np.sqrt((_d(x) ** 2).mean(-1, keepdims=True) + 1e-5)
                                     * w).astype(np.float32), 1e-3, 1e-4, EXACT,
                       consts={"c_eps": 1e-5}, cols_in=("w",)),
    "f02_row_softmax": _rw("f02_row_softmax", "torch.softmax(torch.randn(64, 256), dim=-1)",
                           (64, 256), ("out", "f32"), _softmax_passes(),
                           lambda x: _softmax(_d(x)).astype(np.float32), 1e-3, 1e-5, FAST_REL),
    "f03_l2norm": _rw("f03_l2norm", "x / sqrt((x * x).sum(-1)) (x [64, 512])", (64, 512),
                      ("out", "f32"),
                      [SUMSQ, ("scalar", S("nrm", "sqrt", "acc0")),
                       ("write", [S("y", "divide", "xv", "nrm")], "y")],
                      lambda x: (x / np.sqrt((_d(x) ** 2).sum(-1, keepdims=True))).astype(
                          np.float32), 1e-3, 1e-4, EXACT),
    "f02_center": _rw("f02_center", "x - x.mean(-1, keepdim=True) (x [64, 256])", (64, 256),
                      ("out", "f32"),
                      [SUM, ("scalar", S("mu", "divide", "acc0", "n_cols")),
                       ("write", [S("y", "subtract", "xv", "mu")], "y")],
                      lambda x: (_d(x) - _d(x).mean(-1, keepdims=True)).astype(np.float32),
                      1e-3, 1e-5, EXACT),
    "f03_softmax_narrow": _rw("f03_softmax_narrow", "torch.softmax(torch.randn(128, 64), -1)",
                              (128, 64), ("out", "f32"), _softmax_passes(),
                              lambda x: _softmax(_d(x)).astype(np.float32), 1e-3, 1e-5,
                              FAST_REL, block=64),
    "f05_softmax_temp": _rw("f05_softmax_temp", "torch.softmax(x * 0.5, dim=-1) (x [64, 512])",
                            (64, 512), ("out", "f32"),
                            _softmax_passes(lambda nm, x: [S(nm, "multiply", x, "c_t")]),
                            lambda x: _softmax(_d(x) * 0.5).astype(np.float32), 1e-3, 1e-5,
                            FAST_REL, consts={"c_t": 0.5}),
    "f06_rmsnorm_pow": _rw("f06_rmsnorm_pow", "x * pow(mean(pow(x, 2), -1) + 1e-6, -0.5) "
                           "(x [2, 64, 256])", (128, 256), ("out", "f32"),
                           [SUMSQ, ("scalar", S("ms", "divide", "acc0", "n_cols")),
                            ("scalar", S("mse", "add", "ms", "c_eps")),
                            ("scalar", S("inv", "pow", "mse", "c_p")),
                            ("write", [S("y", "multiply", "xv", "inv")], "y")],
                           lambda x: (_d(x) / np.sqrt((_d(x) ** 2).mean(-1, keepdims=True)
                                                      + 1e-6)).astype(np.float32),
                           1e-3, 1e-4, FAST_REL, consts={"c_eps": 1e-6, "c_p": -0.5}),
    "f07_softmax_4d": _rw("f07_softmax_4d", "torch.softmax(torch.randn(2, 4, 16, 128), -1)",
                          (128, 128), ("out", "f32"), _softmax_passes(),
                          lambda x: _softmax(_d(x)).astype(np.float32), 1e-3, 1e-5, FAST_REL),
    "f08_layernorm_affine": _rw("f08_layernorm_affine",
                                "d / sqrt((d * d).mean(-1) + 1e-5) * w + b, d = x - x.mean(-1) "
                                "(x [32, 256])", (32, 256), ("out", "f32"),
                                [SUM, ("scalar", S("mu", "divide", "acc0", "n_cols")),
                                 ("reduce", "acc1", "add", [S("c", "subtract", "xv", "mu"),
                                                            S("c2", "multiply", "c", "c")],
                                  "c2"),
                                 ("scalar", S("var", "divide", "acc1", "n_cols")),
                                 ("scalar", S("vare", "add", "var", "c_eps")),
                                 ("scalar", S("den", "sqrt", "vare")),
                                 ("write", [S("cc", "subtract", "xv", "mu"),
                                            S("q", "divide", "cc", "den"),
                                            S("qw", "multiply", "q", "w"),
                                            S("y", "add", "qw", "b")], "y")],
                                lambda x, w, b: ((_d(x) - _d(x).mean(-1, keepdims=True))
                                                 / np.sqrt(_d(x).var(-1, keepdims=True) + 1e-5)
                                                 * w + b).astype(np.float32),
                                1e-3, 1e-4, EXACT, consts={"c_eps": 1e-5}, cols_in=("w", "b")),
    "f09_softmax_wide": _rw("f09_softmax_wide", "torch.softmax(torch.randn(8, 4096), dim=-1)",
                            (8, 4096), ("out", "f32"), _softmax_passes(),
                            lambda x: _softmax(_d(x)).astype(np.float32), 1e-3, 1e-6, FAST_REL,
                            block=256),
    "f10_normalize_sum": _rw("f10_normalize_sum", "a / a.sum(-1, keepdim=True), a = x.abs() "
                             "(x [64, 128])", (64, 128), ("out", "f32"),
                             [("reduce", "acc0", "add", [S("a", "abs", "xv")], "a"),
                              ("write", [S("a2", "abs", "xv"), S("y", "divide", "a2", "acc0")],
                               "y")],
                             lambda x: (np.abs(_d(x)) / np.abs(_d(x)).sum(-1, keepdims=True)
                                        ).astype(np.float32), 1e-3, 1e-5, EXACT),
    "f11_softmax_f16": _rw("f11_softmax_f16", "torch.softmax(f16 x [64, 256], dim=-1)",
                           (64, 256), ("out", "f16"),
                           _softmax_passes(lambda nm, x: [S(nm, "cast", x)], out_cast="f16"),
                           lambda x: _softmax(_d(x)).astype(np.float16).astype(np.float32),
                           5e-3, 1e-4, ("rel", 1e-3), dtype="f16"),
}

AXES: dict[str, Callable[[], SuiteCase]] = {
    "r06_col_sum": lambda: SuiteCase(axis_reduce("r06_col_sum", "x.sum(dim=0)", (1, 512, 384),
                                                 "add", False), lambda x: x.sum(1),
                                     1e-4, 1e-4, EXACT),
    "r18_amax_mid": lambda: SuiteCase(axis_reduce("r18_amax_mid", "x.amax(dim=1)",
                                                  (8, 64, 96), "maximum", False),
                                      lambda x: x.max(1), 0, 0, EXACT),
    "r19_mean_mid_axis": lambda: SuiteCase(axis_reduce("r19_mean_mid_axis", "x.mean(dim=1)",
                                                       (16, 100, 48), "add", True),
                                           lambda x: x.mean(1), 1e-5, 1e-5, EXACT),
    "r16_grid_atomic": lambda: SuiteCase(grid_reduce("r16_grid_atomic", "x.sum()", 1 << 18,
                                                     False), lambda x: np.atleast_1d(x.sum()),
                                         1e-5, 1e-5, ATOMIC),
    "r05b_grid_sum_squares": lambda: SuiteCase(grid_reduce("r05b_grid_sum_squares",
                                                           "(x * x).sum()", 100_003, True),
                                               lambda x: np.atleast_1d((x * x).sum()),
                                               1e-5, 1e-5, ATOMIC),
}


def dot_nest(pid: str, code: str, m: int, n: int, k: int, batch: int = 1,
             linear: bool = False, bias: bool = False, relu: bool = False,
             block: int = 128) -> ProblemSpec:
    """out[(b,) i, j] = sum over k of a[(b,) i, k] * B[(b,) k, j], with B = w[j, k] for
    ``F.linear`` (``linear``), then + bias[j] and relu: one thread per output element and a Loop
    over k into an Init'ed accumulator, the plan for matmuls too small or too ragged for block
    tiles (matrix-vector products, odd shapes, few rows)."""
    a0, a1 = V("a0"), V("a1")
    j = rem(a0, I(n))
    i = rem(div(a0, I(n)), I(m)) if batch > 1 else div(a0, I(n))
    bi: tuple[Any, ...] = (div(a0, I(m * n)),) if batch > 1 else ()
    lead = [batch] if batch > 1 else []
    bname = "w" if linear else "b"
    body: list[Stmt] = [
        Init("acc0", 0.0, dt("f32")),
        Loop(Axis("a1", Dim(k)), (
            Load(("av",), "a", (*bi, i, a1), dt("f32")),
            Load(("bv",), bname, (j, a1) if linear else (*bi, a1, j), dt("f32")),
            Assign("pr", op("multiply"), ("av", "bv"), dt("f32")),
            Accum("acc0", "pr", op("add"), dt("f32"), ("a1",), None))),
    ]
    value = "acc0"
    if bias:
        body += [Load(("bb",), "bias", (j,), dt("f32")),
                 Assign("yb", op("add"), (value, "bb"), dt("f32"))]
        value = "yb"
    if relu:
        body.append(Assign("yr", op("relu"), (value,), dt("f32")))
        value = "yr"
    body.append(Write("out", (*bi, i, j), (value,), dt("f32")))
    tile = Tile((Axis("a0", Dim(batch * m * n)),), tuple(body), None)
    args = [_arg("a", "f32", lead + [m, k], seed=0),
            _arg(bname, "f32", [n, k] if linear else lead + [k, n], seed=1)]
    if bias:
        args.append(_arg("bias", "f32", [n], seed=2))
    args.append(_arg("out", "f32", lead + [m, n], output=True))
    return _spec(pid, code, 0, 0, f"k_{pid}", tile, args, [a["name"] for a in args[:-1]],
                 ["out"], {}, block)


def _dn(pid: str, code: str, m: int, n: int, k: int, ref: Callable[..., np.ndarray],
        atol: float = 1e-3, **kw: Any) -> Callable[[], SuiteCase]:
    return lambda: SuiteCase(dot_nest(pid, code, m, n, k, **kw), ref, 1e-3, atol, EXACT)


def _mm(pid: str, m: int, n: int, k: int, **kw: Any) -> Callable[[], SuiteCase]:
    def make() -> SuiteCase:
        spec = matmul(m, n, k, dtype="f32", raster_group=None, **kw)
        spec.meta["id"] = pid
        return SuiteCase(spec, lambda x0, x1: (_d(x0) @ _d(x1)).astype(np.float32), 1e-3,
                         1e-3, EXACT)
    return make


def m06_1024sq(m: int = 1024, n: int = 1024) -> ProblemSpec:
    """The reference's ``m06_1024sq`` (f32 [1024, 1024] @ [1024, 1024]) in the m01 nest with
    128 x 128 block tiles; ``m``, ``n`` smaller give the same nest over fewer tiles (a tile of C
    depends only on its rows of A and columns of B, so a one-tile problem reproduces any tile of
    the full one bit for bit)."""
    spec = matmul(m, n, 1024, dtype="f32", raster_group=None, bm=128, bn=128, bk=16,
                  block=256, b_std=1.0)
    spec.meta["id"] = "m06_1024sq"
    return spec


MATMUL: dict[str, Callable[[], SuiteCase]] = {
    "m00_256x128x256": _mm("m00_256x128x256", 256, 256, 128, bm=64, bn=64, bk=16, block=256),
    "m01_64sq": _mm("m01_64sq", 64, 64, 64, bm=64, bn=64, bk=16, block=256),
    "m03_tall": _mm("m03_tall", 1024, 32, 64, bm=64, bn=32, bk=16, block=128),
    "m04_deep_k": _mm("m04_deep_k", 32, 128, 1024, bm=32, bn=64, bk=32, block=128),
    # the reference's remaining matmul ids; square and rectangular shapes that divide into
    # block tiles take the m01 nest, the rest one thread per output element
    "m02_matmul_rect": _mm("m02_matmul_rect", 128, 64, 256, bm=64, bn=64, bk=16, block=256,
                           b_std=1.0),
    "m02_odd": _dn("m02_odd", "torch.randn(96, 80) @ torch.randn(80, 48)", 96, 48, 80,
                   lambda a, b: (_d(a) @ _d(b)).astype(np.float32)),
    "m05_bias": _dn("m05_bias", "a @ b + c (a, b [128, 128], c [128])", 128, 128, 128,
                    lambda a, b, c: (_d(a) @ _d(b) + _d(c)).astype(np.float32), bias=True),
    "m07_linear_b1": _dn("m07_linear_b1", "F.linear(x [1, 64], w [32, 64])", 1, 32, 64,
                         lambda x, w: (_d(x) @ _d(w).T).astype(np.float32), linear=True),
    "m08_linear_b5": _dn("m08_linear_b5", "F.linear(x [5, 96], w [72, 96])", 5, 72, 96,
                         lambda x, w: (_d(x) @ _d(w).T).astype(np.float32), linear=True),
    "m09_matvec_wide": _dn("m09_matvec_wide", "torch.randn(1, 1024) @ torch.randn(1024, 3072)",
                           1, 3072, 1024, lambda a, b: (_d(a) @ _d(b)).astype(np.float32)),
    "m10_bmm": _dn("m10_bmm", "torch.bmm(torch.randn(4, 64, 32), torch.randn(4, 32, 48))",
                   64, 48, 32, lambda a, b: (_d(a) @ _d(b)).astype(np.float32), batch=4),
    "m11_linear_deep": _dn("m11_linear_deep", "F.linear(x [1, 4096], w [512, 4096])", 1, 512,
                           4096, lambda x, w: (_d(x) @ _d(w).T).astype(np.float32), atol=2e-3,
                           linear=True),
    "m12_linear_bias": _dn("m12_linear_bias", "F.linear(x [16, 128], w [64, 128], b [64])",
                           16, 64, 128,
                           lambda x, w, b: (_d(x) @ _d(w).T + _d(b)).astype(np.float32),
                           linear=True, bias=True),
    "m13_matmul_relu": _dn("m13_matmul_relu",
                           "torch.relu(torch.randn(128, 64) @ torch.randn(64, 128))", 128, 128,
                           64, lambda a, b: np.maximum(_d(a) @ _d(b), 0).astype(np.float32),
                           relu=True),
}




def ref_inputs(case: SuiteCase, inputs: dict[str, np.ndarray]) -> list[np.ndarray]:
    """The case's graph inputs in graph-input order, in their own dtypes (bf16 as the f32
    values of its bits), so a formula computes in NumPy the way the reference's does."""
    from .problems import bf16_values

    out = []
    for name in case.spec.meta["graph_inputs"]:
        a = next(x for x in case.spec.kernel["args"] if x["name"] == name)
        v = inputs[name]
        out.append(bf16_values(v) if a["dtype"] == "bf16" else v)
    return out


# --- fused attention ---------------------------------------------------------------------------


def attention(pid: str, code: str, b: int, m: int, n: int, d: int, dv: int, scale: str,
              value: float, rb: int, r: int, cb: int, c: int) -> ProblemSpec:
    """softmax(q @ kt * s) @ v over f32 q [b, m, d], kt [b, d, n], v [b, n, dv] (b = 1: 2-D),
    in the shipped a01 nest's shape (reference ``examples/op_fusion/a01_attention``): a Tile over
    (batch,) row blocks of ``rb``, column blocks of ``cb`` and threads holding ``r`` rows x ``c``
    columns; per key a1 an inner-product Loop over d per row, then per (row, column) the online
    update -- running max ``mx``, alpha = exp(mx_old - mx_new), beta = exp(s - mx_new), the
    denominator ``den`` <- alpha*den + beta and the numerator ``num`` <- alpha*num + beta*v --
    and after the keys num / den. ``scale`` is "div" (s = score / value, as a reciprocal of the
    ConstantOp), "mul" (s = score * value) or "none"."""
    bt = b > 1
    axes = ([Axis("ab", Dim(b))] if bt else []) + [
        Axis("a0_b", Dim(m // rb)), Axis("a5_b", Dim(dv // cb)),
        Axis("a0_u", Dim(rb // r)), Axis("a5_u", Dim(cb // c))]
    block = (rb // r) * (cb // c)
    bi: tuple[Any, ...] = (V("ab"),) if bt else ()
    row = lambda i: add(add(mul(V("a0_b"), I(rb)), mul(V("a0_u"), I(r))), I(i))  # noqa: E731
    col = add(mul(V("a5_b"), I(cb)), mul(V("a5_u"), I(c)))
    body: list[Stmt] = []
    consts: dict[str, float] = {}
    if scale == "div":
        consts["div_c1"] = value
        body += [Load(("sc_in",), "div_c1", (I(0),), dt("f32")),
                 Assign("sc", op("reciprocal"), ("sc_in",), dt("f32"))]
    elif scale == "mul":
        consts["mul_c1"] = value
        body.append(Load(("sc",), "mul_c1", (I(0),), dt("f32")))
    keys: list[Stmt] = []
    for i in range(r):
        keys.append(Loop(Axis("a2", Dim(d)), (
            Load((f"q__r{i}",), "q", (*bi, row(i), V("a2")), dt("f32")),
            Load((f"k__r{i}",), "kt", (*bi, V("a2"), V("a1")), dt("f32")),
            Assign(f"qk__r{i}", op("multiply"), (f"k__r{i}", f"q__r{i}"), dt("f32")),
            Accum(f"dot__r{i}", f"qk__r{i}", op("add"), dt("f32"), ("a2",), None))))
    keys.append(Load(tuple(f"v__c{j}" for j in range(c)), "v", (*bi, V("a1"), col), dt("f32")))
    for i in range(r):
        s_ = f"dot__r{i}"
        if scale != "none":
            keys.append(Assign(f"s__r{i}", op("multiply"), (s_, "sc"), dt("f32")))
            s_ = f"s__r{i}"
        for j in range(c):
            u = f"__r{i}c{j}"
            keys += [
                Let(f"one{u}", Literal(1.0, "float"), dt("f32")),
                Assign(f"gn{u}", op("maximum"), (s_, f"mx{u}"), dt("f32")),
                Assign(f"dg{u}", op("subtract"), (f"mx{u}", f"gn{u}"), dt("f32")),
                Assign(f"alpha{u}", op("exp"), (f"dg{u}",), dt("f32")),
                Assign(f"dgo{u}", op("subtract"), (s_, f"gn{u}"), dt("f32")),
                Assign(f"beta{u}", op("exp"), (f"dgo{u}",), dt("f32")),
                Assign(f"den_sa{u}", op("multiply"), (f"alpha{u}", f"den{u}"), dt("f32")),
                Assign(f"den_sb{u}", op("multiply"), (f"beta{u}", f"one{u}"), dt("f32")),
                Accum(f"den{u}", f"den_sb{u}", op("add"), dt("f32"), ("a1",), f"den_sa{u}"),
                Assign(f"num_sa{u}", op("multiply"), (f"alpha{u}", f"num{u}"), dt("f32")),
                Assign(f"num_sb{u}", op("multiply"), (f"beta{u}", f"v__c{j}"), dt("f32")),
                Accum(f"num{u}", f"num_sb{u}", op("add"), dt("f32"), ("a1",), f"num_sa{u}"),
                Accum(f"mx{u}", s_, op("maximum"), dt("f32"), ("a1",), None),
            ]
    body.append(Loop(Axis("a1", Dim(n)), tuple(keys)))
    for i in range(r):
        for j in range(c):
            u = f"__r{i}c{j}"
            body += [Assign(f"rcp{u}", op("reciprocal"), (f"den{u}",), dt("f32")),
                     Assign(f"o{u}", op("multiply"), (f"num{u}", f"rcp{u}"), dt("f32")),
                     Write("out", (*bi, row(i), add(col, I(j))), (f"o{u}",), dt("f32"))]
    tile = Tile(tuple(axes), tuple(body), block)
    lead = [b] if bt else []
    args = [_arg(k, "f32", [1], data=[v]) for k, v in consts.items()]
    args += [_arg("q", "f32", lead + [m, d], seed=0), _arg("kt", "f32", lead + [d, n], seed=1),
             _arg("v", "f32", lead + [n, dv], seed=2),
             _arg("out", "f32", lead + [m, dv], output=True)]
    return _spec(pid, code, 1e-3, 1e-4, f"k_{pid}", tile, args, ["q", "kt", "v"], ["out"],
                 consts, block)


def _attn(scale: float) -> Callable[..., np.ndarray]:
    def ref(q: np.ndarray, kt: np.ndarray, v: np.ndarray) -> np.ndarray:
        q, kt, v = (x.astype(np.float64) for x in (q, kt, v))
        return (_softmax(q @ kt * scale) @ v).astype(np.float32)
    return ref


def _at(pid: str, shape: tuple[int, int, int, int, int], scale: str, value: float,
        layout: tuple[int, int, int, int]) -> Callable[[], SuiteCase]:
    b, m, n, d, dv = shape
    factor = {"div": 1.0 / value if value else 1.0, "mul": value, "none": 1.0}[scale]
    code = (f"q [{b}, {m}, {d}], kt [{b}, {d}, {n}], v [{b}, {n}, {dv}]: "
            f"torch.softmax(q @ kt {'/' if scale == 'div' else '*'} {value}, dim=-1) @ v")
    return lambda: SuiteCase(attention(pid, code, b, m, n, d, dv, scale, value, *layout),
                             _attn(factor), 1e-3, 1e-4, FAST_REL)


ATTENTION: dict[str, Callable[[], SuiteCase]] = {
    "a00_small": _at("a00_small", (1, 32, 32, 16, 16), "div", 4.0, (32, 4, 16, 2)),
    "a01_256": _at("a01_256", (1, 256, 256, 64, 64), "div", 8.0, (32, 4, 64, 2)),
    "a02_rect": _at("a02_rect", (1, 64, 128, 32, 64), "mul", 0.1767767, (32, 4, 64, 2)),
    "a03_noscale": _at("a03_noscale", (1, 64, 64, 64, 64), "none", 0.0, (32, 4, 64, 2)),
    "a04_batched": _at("a04_batched", (2, 64, 64, 32, 32), "div", 5.656854, (32, 4, 32, 2)),
    "a05_heads": _at("a05_heads", (4, 32, 48, 16, 16), "mul", 0.25, (32, 4, 16, 2)),
    "a06_long_kv": _at("a06_long_kv", (1, 16, 512, 64, 64), "div", 8.0, (16, 2, 64, 2)),
    "a07_tall_q": _at("a07_tall_q", (1, 256, 64, 16, 16), "div", 4.0, (64, 4, 16, 2)),
    "a02_attention_128": _at("a02_attention_128", (1, 128, 128, 32, 32), "div", 5.656854,
                             (32, 4, 32, 2)),
}


# --- problems of several kernels ---------------------------------------------------------------


@dataclass
class MultiSpec:
    """A problem of several kernels: one Kernel IR graph per kernel entry, one meta.json."""

    graphs: dict[str, dict[str, Any]]
    meta: dict[str, Any]

    def write(self, directory: Any) -> Any:
        import json
        from pathlib import Path

        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        for entry, g in self.graphs.items():
            (d / f"{entry}.ir.json").write_text(json.dumps(g, indent=2))
        (d / "meta.json").write_text(json.dumps(self.meta, indent=1))
        return d


@dataclass
class Kern:
    entry: str
    tile: Tile
    args: list[dict[str, Any]]  # in arg order; outputs marked, chained buffers "intermediate"
    block: int
    zero_outputs: Sequence[str] = ()


def _multi(pid: str, code: str, kernels: list[Kern], inputs: list[str], outputs: list[str],
           consts: dict[str, float]) -> MultiSpec:
    """Per-kernel graphs and the meta.json of a chained problem, as the reference's packager
    lays it out: one ``<entry>.ir.json`` per kernel, meta.json's kernels in launch order."""
    graphs, metas = {}, []
    for k in kernels:
        specs = {a["name"]: TensorSpec(a["name"], tuple(a["shape"]), a["dtype"]) for a in k.args}
        nodes: dict[str, Any] = {}
        for a in k.args:
            if "data" in a:
                nodes[a["name"]] = constant_node(a["name"], consts[a["name"]])
            elif not a.get("output"):
                nodes[a["name"]] = input_node(specs[a["name"]])
        outs = [a["name"] for a in k.args if a.get("output")]
        nodes[outs[0]] = kernel_node(k.entry, k.tile,
                                     [a["name"] for a in k.args if not a.get("output")],
                                     [specs[o] for o in outs])
        graphs[k.entry] = {"inputs": [a["name"] for a in k.args
                                      if not a.get("output") and "data" not in a],
                           "outputs": outs, "nodes": nodes}
        metas.append({"node": outs[0], "entry": k.entry, "arg_order": [a["name"] for a in k.args],
                      "grid": [-(-k.tile.n_elements // k.block), 1, 1], "block": [k.block, 1, 1],
                      "smem_bytes": 0, "zero_outputs": list(k.zero_outputs), "args": k.args,
                      "final": bool(set(outs) & set(outputs))})
    meta = {"id": pid, "code": code, "rtol": 0, "atol": 0, "graph_inputs": inputs,
            "graph_outputs": outputs, "kernels": metas}
    return MultiSpec(graphs, meta)


def grid_kernel_sum(n: int = 1 << 20, block: int = 256, blocks: int = 128) -> MultiSpec:
    """sum(x) by the grid-kernel plan: kernel 1 reduces a grid-stride share per block and
    writes each block's total into ``partials`` [blocks]; kernel 2, one block, sums those. No
    atomics, so the result is deterministic."""
    ab, at = V("a0_b"), V("a0_t")
    k1 = Tile((Axis("a0_b", Dim(blocks)), Axis("a0_t", Dim(block))), (
        StridedLoop(Axis("a0", Dim(n)), add(mul(ab, I(block)), at), I(block * blocks),
                    (Load(("xv",), "x", (V("a0"),), dt("f32")),
                     Accum("acc0", "xv", op("add"), dt("f32"), ("a0",), None)),
                    False, None, True),
        *_block_reduce("acc0", "add", block, "acc0_smem"),
        Cond(BinaryExpr("==", at, I(0)), (Write("partials", (ab,), ("acc0",), dt("f32")),), ()),
    ), block)
    t2 = V("a0_t")
    k2 = Tile((Axis("a0_b", Dim(1)), Axis("a0_t", Dim(block))), (
        StridedLoop(Axis("a1", Dim(blocks)), t2, I(block),
                    (Load(("pv",), "partials", (V("a1"),), dt("f32")),
                     Accum("acc1", "pv", op("add"), dt("f32"), ("a1",), None)),
                    False, None, True),
        *_block_reduce("acc1", "add", block, "acc1_smem"),
        Cond(BinaryExpr("==", t2, I(0)), (Write("out", (), ("acc1",), dt("f32")),), ()),
    ), block)
    return _multi("r17_grid_kernel", "x.sum() (grid-kernel reduce plan)", [
        Kern("k_sum_partials", k1, [_arg("x", "f32", [n], seed=0),
                                    _arg("partials", "f32", [blocks], output=True)], block),
        Kern("k_sum_final", k2, [_arg("partials", "f32", [blocks], intermediate=True),
                                 _arg("out", "f32", [1], output=True)], block),
    ], ["x"], ["out"], {})


def two_pass_softmax(rows: int = 64, cols: int = 1024, block: int = 128) -> MultiSpec:
    """softmax(x, dim=-1) in two kernels: a row pass writes each row's max and sum of
    exp(x - max) into ``row_max`` and ``row_sum`` [rows]; a pointwise pass over all elements
    reads them by row and writes exp(x - max) / sum."""
    a0, t = V("a0"), V("a1_co")
    sweep = lambda body: StridedLoop(Axis("a1", Dim(cols)), t, I(block), tuple(body),  # noqa
                                     False, None, True)
    k1 = Tile((Axis("a0", Dim(rows)), Axis("a1_co", Dim(block))), (
        sweep([Load(("x0",), "x", (a0, V("a1")), dt("f32")),
               Accum("acc0", "x0", op("maximum"), dt("f32"), ("a1",), None)]),
        *_block_reduce("acc0", "maximum", block, "acc0_smem"),
        sweep([Load(("x1",), "x", (a0, V("a1")), dt("f32")),
               Assign("d", op("subtract"), ("x1", "acc0"), dt("f32")),
               Assign("e", op("exp"), ("d",), dt("f32")),
               Accum("acc1", "e", op("add"), dt("f32"), ("a1",), None)]),
        *_block_reduce("acc1", "add", block, "acc1_smem"),
        Cond(BinaryExpr("==", t, I(0)), (Write("row_max", (a0,), ("acc0",), dt("f32")),
                                          Write("row_sum", (a0,), ("acc1",), dt("f32"))), ()),
    ), block)
    e0, pw = V("a0"), 256
    k2 = Tile((Axis("a0", Dim(rows * cols)),), (
        Load(("xv",), "x", (e0,), dt("f32")),
        Load(("mx",), "row_max", (div(e0, I(cols)),), dt("f32")),
        Load(("sm",), "row_sum", (div(e0, I(cols)),), dt("f32")),
        Assign("d", op("subtract"), ("xv", "mx"), dt("f32")),
        Assign("e", op("exp"), ("d",), dt("f32")),
        Assign("y", op("divide"), ("e", "sm"), dt("f32")),
        Write("out", (e0,), ("y",), dt("f32")),
    ), None)
    return _multi("f13_softmax_two_pass", "torch.softmax(x, dim=-1) in two kernels", [
        Kern("k_softmax_stats", k1, [_arg("x", "f32", [rows, cols], seed=0),
                                     _arg("row_max", "f32", [rows], output=True),
                                     _arg("row_sum", "f32", [rows], output=True)], block),
        Kern("k_softmax_normalise", k2, [_arg("x", "f32", [rows, cols], seed=0),
                                         _arg("row_max", "f32", [rows], intermediate=True),
                                         _arg("row_sum", "f32", [rows], intermediate=True),
                                         _arg("out", "f32", [rows, cols], output=True)], pw),
    ], ["x"], ["out"], {})


@dataclass
class MultiCase:
    spec: MultiSpec
    ref: Callable[..., np.ndarray]
    rtol: float
    atol: float
    bar: tuple[str, float]


MULTI: dict[str, Callable[[], MultiCase]] = {
    "r17_grid_kernel": lambda: MultiCase(grid_kernel_sum(), lambda x: np.atleast_1d(x.sum()),
                                         1e-5, 1e-5, EXACT),
    "f13_softmax_two_pass": lambda: MultiCase(two_pass_softmax(), _softmax, 1e-3, 1e-5,
                                              FAST_REL),
}


SUITE: dict[str, Callable[[], SuiteCase]] = {**POINTWISE, **ROWWISE, **AXES, **MATMUL,
                                             **ATTENTION}

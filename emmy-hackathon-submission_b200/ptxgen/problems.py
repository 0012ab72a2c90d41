"""Kernel IR problems for the benchmark configurations, written the way Emmy writes them.

Emmy (``emmy-ml``), which traces a torch expression into Kernel IR, is not available, so this
module builds the ``<kernel>.ir.json`` + ``meta.json`` pair of each configuration directly, in
Emmy's repr format and in the shapes of the shipped IRs (reference ``examples/``):

* ``pointwise_add``  -- ``p02``'s shape: one Tile axis, an unrolled body of ``unroll`` consecutive
  elements, one vector Write;
* ``gelu_chain``     -- the same shape over bf16 ``x`` with a per-row f32 scale, gelu's tanh form
  decomposed into primitive ops plus ``tanh`` as Emmy decomposes it;
* ``row_softmax``    -- one block per row: a max pass and a sum-of-exp pass, each a StridedLoop +
  WarpShuffle + shared slots + TreeHalve (``r02``'s reduction shape), then the normalising pass;
* ``full_sum``       -- ``r02``'s shape over many blocks, each block adding its total into the
  zeroed output with an atomic Write (Emmy's grid-atomic plan);
* ``matmul``         -- ``m01``'s shape: a block tile of C per CTA, a ring of cp.async stages of A
  and B tiles in shared memory, a K loop of FMAs over register tiles; optionally split along K
  with atomic Writes into the zeroed C.

The meta.json schema is the reference's (``tools/generate.py:99-107,130-146,196-198``); each
argument may add a ``dist`` (``["normal", mean, std]`` or ``["uniform", lo, hi]``) that replaces
``standard_normal`` in the seeding rule (``default_rng(index of the input)``,
``tools/generate.py:152-157``). bf16 inputs are generated in f32 and rounded to nearest even.
"""

from __future__ import annotations

import json
import math
from collections.abc import Sequence
from pathlib import Path
from typing import Any

import numpy as np

from .ir import (Accum, Assign, Axis, BinaryExpr, Cond, CpAsyncCommit, CpAsyncCopy, CpAsyncWait,
                 Dim, ElementwiseImpl, Expr, Graph, Init, Let, Literal, Load, Loop, Smem,
                 Stmt, StridedLoop, Sync, TensorSpec, TernaryExpr, Tile, TreeHalve, Var,
                 WarpShuffle, Window, Write, constant_node, dt, input_node, kernel_node)

# --- expression helpers ----------------------------------------------------------------------


def V(name: str) -> Var:
    return Var(name)


def I(value: int) -> Literal:  # noqa: E743 - an integer literal
    return Literal(value, "int")


def add(a: Expr, b: Expr) -> BinaryExpr:
    return BinaryExpr("+", a, b)


def mul(a: Expr, b: Expr) -> BinaryExpr:
    return BinaryExpr("*", a, b)


def div(a: Expr, b: Expr) -> BinaryExpr:
    return BinaryExpr("/", a, b)


def rem(a: Expr, b: Expr) -> BinaryExpr:
    return BinaryExpr("%", a, b)


def op(name: str) -> ElementwiseImpl:
    return ElementwiseImpl(name)


def assign(name: str, fn: str, args: Sequence[str], dtype: str | None = "f32") -> Assign:
    return Assign(name, op(fn), tuple(args), dt(dtype) if dtype else None)


# --- problem container -----------------------------------------------------------------------


class ProblemSpec:
    """A generated problem: its graph JSON and meta.json."""

    def __init__(self, graph: dict[str, Any], meta: dict[str, Any]):
        self.graph, self.meta = graph, meta

    @property
    def kernel(self) -> dict[str, Any]:
        return self.meta["kernels"][0]

    @property
    def entry(self) -> str:
        return self.kernel["entry"]

    def write(self, directory: str | Path) -> Path:
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        (d / f"{self.entry}.ir.json").write_text(json.dumps(self.graph, indent=2))
        (d / "meta.json").write_text(json.dumps(self.meta, indent=1))
        return d

    def graph_obj(self) -> Graph:
        return Graph.from_dict(self.graph)


def _arg(name: str, dtype: str, shape: Sequence[int], **kw: Any) -> dict[str, Any]:
    return {"name": name, "dtype": dtype, "shape": list(shape), **kw}


def _spec(pid: str, code: str, rtol: float, atol: float, entry: str, tile: Tile,
          args: list[dict[str, Any]], inputs: list[str], outputs: list[str],
          consts: dict[str, float], block: int, smem_bytes: int = 0,
          zero_outputs: Sequence[str] = ()) -> ProblemSpec:
    nodes: dict[str, Any] = {}
    for name, value in consts.items():
        nodes[name] = constant_node(name, value)
    specs = {a["name"]: TensorSpec(a["name"], tuple(a["shape"]), a["dtype"]) for a in args}
    for name in inputs:
        nodes[name] = input_node(specs[name])
    out_node = outputs[0]
    nodes[out_node] = kernel_node(entry, tile, [a["name"] for a in args if not a.get("output")],
                                  [specs[o] for o in outputs])
    graph = {"inputs": inputs, "outputs": outputs, "nodes": nodes}
    grid = -(-tile.n_elements // block)
    kern = {"node": out_node, "entry": entry, "arg_order": [a["name"] for a in args],
            "grid": [grid, 1, 1], "block": [block, 1, 1], "smem_bytes": smem_bytes,
            "zero_outputs": list(zero_outputs), "args": args, "final": True}
    meta = {"id": pid, "code": code, "rtol": rtol, "atol": atol, "graph_inputs": inputs,
            "graph_outputs": outputs, "kernels": [kern]}
    return ProblemSpec(graph, meta)


# --- config 1: f32 pointwise add --------------------------------------------------------------


def pointwise_add(n: int = 2**24, block: int = 256, unroll: int = 4, dtype: str = "f32",
                  dist: Sequence[Any] = ("uniform", -1.0, 1.0)) -> ProblemSpec:
    """z = x + y over n elements, ``unroll`` consecutive elements per Tile cell."""
    if n % unroll:
        unroll = 1
    cells = n // unroll
    a0 = V("a0")
    body: list[Stmt] = []
    for j in range(unroll):
        idx = (add(mul(a0, I(unroll)), I(j)),) if unroll > 1 else (a0,)
        body += [Load((f"in0__u{j}",), "x", idx, dt(dtype)),
                 Load((f"in1__u{j}",), "y", idx, dt(dtype)),
                 assign(f"v0__u{j}", "add", (f"in0__u{j}", f"in1__u{j}"), dtype)]
    widx = (add(mul(a0, I(unroll)), I(0)),) if unroll > 1 else (a0,)
    body.append(Write("add", widx, tuple(f"v0__u{j}" for j in range(unroll)), dt(dtype)))
    tile = Tile((Axis("a0", Dim(cells)),), tuple(body), None)
    args = [_arg("x", dtype, [n], seed=0, dist=list(dist)),
            _arg("y", dtype, [n], seed=1, dist=list(dist)),
            _arg("add", dtype, [n], output=True)]
    return _spec("c1_vector_add", f"torch.rand({n}) + torch.rand({n})", 0, 0,
                 "k_add_pointwise", tile, args, ["x", "y"], ["add"], {}, block)


# --- config 2: bf16 gelu_tanh(a*x + b) * s ---------------------------------------------------

GELU_C = 0.044715
GELU_K = math.sqrt(2.0 / math.pi)


def gelu_chain(rows: int = 8192, cols: int = 8192, block: int = 256, unroll: int = 16,
               a: float | None = None, b: float | None = None) -> ProblemSpec:
    """y = gelu_tanh(a*x + b) * s[row] over a [rows, cols] bf16 x, computed in f32, y bf16."""
    rng = np.random.default_rng(1234)
    a = float(np.float32(rng.uniform(-2, 2))) if a is None else a
    b = float(np.float32(rng.uniform(-2, 2))) if b is None else b
    n = rows * cols
    if n % unroll or cols % unroll:
        unroll = 1
    a0 = V("a0")
    body: list[Stmt] = [
        Load(("in_a",), "mul_c1", (I(0),), dt("f32")),
        Load(("in_b",), "add_c1", (I(0),), dt("f32")),
        Let("c_cube", Literal(GELU_C, "float"), dt("f32")),
        Let("c_sqrt2pi", Literal(GELU_K, "float"), dt("f32")),
        Let("c_half", Literal(0.5, "float"), dt("f32")),
        Let("c_one", Literal(1.0, "float"), dt("f32")),
    ]
    for j in range(unroll):
        u = f"__u{j}"
        flat = add(mul(a0, I(unroll)), I(j)) if unroll > 1 else a0
        body += [
            Load((f"in_x{u}",), "x", (flat,), dt("bf16")),
            Load((f"in_s{u}",), "s", (div(flat, I(cols)),), dt("f32")),
            assign(f"v0{u}", "multiply", ("in_a", f"in_x{u}")),
            assign(f"v1{u}", "add", (f"v0{u}", "in_b")),
            assign(f"v2{u}", "multiply", (f"v1{u}", f"v1{u}")),
            assign(f"v3{u}", "multiply", (f"v2{u}", f"v1{u}")),
            assign(f"v4{u}", "multiply", ("c_cube", f"v3{u}")),
            assign(f"v5{u}", "add", (f"v1{u}", f"v4{u}")),
            assign(f"v6{u}", "multiply", ("c_sqrt2pi", f"v5{u}")),
            assign(f"v7{u}", "tanh", (f"v6{u}",)),
            assign(f"v8{u}", "add", (f"v7{u}", "c_one")),
            assign(f"v9{u}", "multiply", ("c_half", f"v1{u}")),
            assign(f"v10{u}", "multiply", (f"v9{u}", f"v8{u}")),
            assign(f"v11{u}", "multiply", (f"v10{u}", f"in_s{u}")),
        ]
    widx = (add(mul(a0, I(unroll)), I(0)),) if unroll > 1 else (a0,)
    body.append(Write("mul_1", widx, tuple(f"v11__u{j}" for j in range(unroll)), dt("f32")))
    tile = Tile((Axis("a0", Dim(n // unroll)),), tuple(body), None)
    args = [_arg("mul_c1", "f32", [1], data=[a]), _arg("add_c1", "f32", [1], data=[b]),
            _arg("x", "bf16", [rows, cols], seed=0, dist=["normal", 0.0, 1.0]),
            _arg("s", "f32", [rows], seed=1, dist=["uniform", 0.5, 1.5]),
            _arg("mul_1", "bf16", [rows, cols], output=True)]
    code = (f"x = torch.randn({rows}, {cols}, dtype=torch.bfloat16); s = torch.rand({rows}, 1); "
            f"torch.nn.functional.gelu({a!r} * x + {b!r}, approximate='tanh') * s")
    return _spec("c2_gelu_chain", code, 1e-2, 1e-2, "k_gelu_chain", tile, args, ["x", "s"],
                 ["mul_1"], {"mul_c1": a, "add_c1": b}, block)


# --- shared reduction tail (r02 shape) --------------------------------------------------------


def _block_reduce(acc: str, fn: str, block: int, smem: str) -> list[Stmt]:
    """WarpShuffle over 32 lanes, lane 0 of each warp to shared slot ``warp``, Sync, then a
    TreeHalve over the block's warps (reference ``examples/cse/r02_big_sum/*.ir.txt``)."""
    warps = block // 32
    combine = (Assign(acc, op(fn), (acc, f"{acc}__o"), None),)
    out: list[Stmt] = [
        WarpShuffle((acc,), (f"{acc}__o",), combine, 32, dt("f32")),
        Smem(smem, (warps,), "float", 0),
        Cond(BinaryExpr("==", V("lane"), I(0)),
             (Write(smem, (V("warp"),), (acc,), dt("f32")),), ()),
        Sync(0, None, False),
    ]
    if warps > 1:
        out.append(TreeHalve((smem,), (acc,), (f"{acc}__o",), combine, warps, "warp", dt("f32"),
                             0, None, None))
    else:
        out.append(Load((f"{acc}__w",), smem, (I(0),), dt("f32")))
    return out


# --- config 3: row softmax -------------------------------------------------------------------


def row_softmax(rows: int = 16384, cols: int = 4096, block: int = 256,
                std: float = 3.0) -> ProblemSpec:
    """y = softmax(x, dim=-1) over [rows, cols] f32, one block per row."""
    if block % 32 or cols % block:
        raise ValueError("row_softmax wants block a multiple of 32 dividing cols")
    a0, t = V("a0"), V("a1_co")

    def sweep(name: str, body: tuple[Stmt, ...]) -> StridedLoop:
        return StridedLoop(Axis(name, Dim(cols)), t, I(block), body, False, None, True)

    body: list[Stmt] = [
        sweep("a1", (Load(("in0",), "x", (a0, V("a1")), dt("f32")),
                     Accum("acc0", "in0", op("maximum"), dt("f32"), ("a1",), None))),
        *_block_reduce("acc0", "maximum", block, "acc0_smem"),
        sweep("a1", (Load(("in1",), "x", (a0, V("a1")), dt("f32")),
                     assign("v0", "subtract", ("in1", "acc0")),
                     assign("v1", "exp", ("v0",)),
                     Accum("acc1", "v1", op("add"), dt("f32"), ("a1",), None))),
        *_block_reduce("acc1", "add", block, "acc1_smem"),
        assign("v2", "reciprocal", ("acc1",)),
        sweep("a1", (Load(("in2",), "x", (a0, V("a1")), dt("f32")),
                     assign("v3", "subtract", ("in2", "acc0")),
                     assign("v4", "exp", ("v3",)),
                     assign("v5", "multiply", ("v4", "v2")),
                     Write("softmax", (a0, V("a1")), ("v5",), dt("f32")))),
    ]
    tile = Tile((Axis("a0", Dim(rows)), Axis("a1_co", Dim(block))), tuple(body), block)
    args = [_arg("x", "f32", [rows, cols], seed=0, dist=["normal", 0.0, std]),
            _arg("softmax", "f32", [rows, cols], output=True)]
    return _spec("c3_row_softmax", f"torch.softmax(torch.randn({rows}, {cols}) * {std}, dim=-1)",
                 1e-3, 1e-5, "k_softmax_reduce", tile, args, ["x"], ["softmax"], {}, block)


# --- config 4: full-tensor sum ---------------------------------------------------------------


def full_sum(n: int = 2**30, block: int = 256, blocks: int = 148 * 8) -> ProblemSpec:
    """sum(x) over n f32 elements: a grid-stride StridedLoop per thread, a block reduction, and
    one atomic add of each block's total into the zeroed output."""
    if block % 32:
        raise ValueError("full_sum wants block a multiple of 32")
    threads = block * blocks
    ab, at = V("a0_b"), V("a0_t")
    body: list[Stmt] = [
        StridedLoop(Axis("a0", Dim(n)), add(mul(ab, I(block)), at), I(threads),
                    (Load(("in0",), "x", (V("a0"),), dt("f32")),
                     Accum("acc0", "in0", op("add"), dt("f32"), ("a0",), None)),
                    False, None, True),
        *_block_reduce("acc0", "add", block, "acc0_smem"),
        Cond(BinaryExpr("==", at, I(0)),
             (Write("sum_1", (), ("acc0",), dt("f32"), True),), ()),
    ]
    tile = Tile((Axis("a0_b", Dim(blocks)), Axis("a0_t", Dim(block))), tuple(body), block)
    args = [_arg("x", "f32", [n], seed=0, dist=["uniform", 0.0, 1.0]),
            _arg("sum_1", "f32", [1], output=True)]
    return _spec("c4_full_sum", f"torch.rand({n}).sum()", 1e-5, 1e-5, "k_sum_1_reduce", tile,
                 args, ["x"], ["sum_1"], {}, block, zero_outputs=["sum_1"])


# --- config 5: matmul (m01 shape) ------------------------------------------------------------


def matmul(m: int = 8192, n: int = 8192, k: int = 8192, dtype: str = "bf16",
           bm: int = 128, bn: int = 256, bk: int = 64, stages: int = 4, block: int = 256,
           split_k: int = 1, raster_group: int | None = 8,
           b_std: float | None = None) -> ProblemSpec:
    """C[m, n] = A[m, k] @ B[k, n] with f32 accumulation and output, in m01's SIMT shape: each
    block owns a bm x bn tile of C, each thread a (bm/ty) x (bn/tx) register tile; A and B tiles
    stream through a ring of ``stages`` shared-memory stages filled by 16-byte cp.async copies.
    With ``split_k`` > 1 the K range is split across blocks, which add their partial tiles into
    the zeroed C with atomic Writes."""
    esz = 2 if dtype in ("bf16", "f16") else 4
    per = 16 // esz  # elements per 16-byte copy
    if m % bm or n % bn or k % (bk * split_k):
        raise ValueError("matmul: m, n, k must be multiples of the block tile")
    tx = min(32, bn // 2)  # threads along n
    ty = block // tx  # threads along m
    if ty * tx != block or bm % ty or bn % tx:
        raise ValueError("matmul: block does not tile the block tile")
    rm, rn = bm // ty, bn // tx  # register tile per thread
    ksplit = k // split_k
    if (bm * bk) % (per * block) or (bk * bn) % (per * block):
        raise ValueError("matmul: tiles do not split into whole 16-byte copies per thread")

    ab, nb, au, nu = V("a0_b"), V("a1_b"), V("a0_u"), V("a1_u")
    tid = add(mul(au, I(tx)), nu)
    kbase: Expr = I(0) if split_k == 1 else mul(V("ak_s"), I(ksplit))
    # a thread's 16-byte copy: row and column of its lane within a copy pass
    a_row, a_col = div(mul(tid, I(per)), I(bk)), rem(mul(tid, I(per)), I(bk))
    b_row, b_col = div(mul(tid, I(per)), I(bn)), rem(mul(tid, I(per)), I(bn))
    a_pass, b_pass = block * per // bk, block * per // bn  # rows one pass covers

    def copies(stage: Expr, kk: Expr) -> list[Stmt]:
        out: list[Stmt] = []
        for r0 in range(0, bm, a_pass):
            out.append(CpAsyncCopy(
                "_a_smem", (add(mul(stage, I(bm)), I(r0)), I(0)), "x0",
                (add(mul(ab, I(bm)), add(a_row, I(r0))), add(add(kbase, kk), a_col)),
                16, "NONE", (a_row, a_col), None))
        for r0 in range(0, bk, b_pass):
            out.append(CpAsyncCopy(
                "_b_smem", (add(mul(stage, I(bk)), I(r0)), I(0)), "x1",
                (add(add(kbase, kk), add(b_row, I(r0))), add(mul(nb, I(bn)), b_col)),
                16, "NONE", (b_row, b_col), None))
        return out

    acc = lambda i, j: f"acc0__c{i}_{j}"  # noqa: E731
    body: list[Stmt] = [Init(acc(i, j), 0.0, dt("f32")) for i in range(rm) for j in range(rn)]
    body += [Smem("_a_smem", (stages * bm, bk), _cname(dtype), 16),
             Smem("_b_smem", (stages * bk, bn), _cname(dtype), 16)]
    for s in range(stages - 1):  # past the end the prologue re-reads the last K tile
        body += copies(I(s), I(min(s * bk, ksplit - bk)))
        body.append(CpAsyncCommit())
    ks = V("_ks")
    nxt = add(ks, I((stages - 1) * bk))
    stage_next = rem(add(div(ks, I(bk)), I(stages - 1)), I(stages))
    # past the end the copy re-reads the last K tile, so every thread issues the same groups
    kk_next = TernaryExpr(BinaryExpr("<", nxt, I(ksplit)), nxt, I(ksplit - bk))
    stage_now = rem(div(ks, I(bk)), I(stages))
    inner: list[Stmt] = []
    for i in range(rm):
        row = add(mul(stage_now, I(bm)), add(mul(au, I(rm)), I(i)))
        inner.append(Load((f"in0__r{i}",), "_a_smem", (row, V("_ki")), dt(dtype)))
    for j in range(rn):
        inner.append(Load((f"in1__c{j}",), "_b_smem",
                          (add(mul(stage_now, I(bk)), V("_ki")), add(mul(nu, I(rn)), I(j))),
                          dt(dtype)))
    for i in range(rm):
        for j in range(rn):
            inner += [assign(f"acc0__v__c{i}_{j}", "multiply", (f"in0__r{i}", f"in1__c{j}")),
                      Accum(acc(i, j), f"acc0__v__c{i}_{j}", op("add"), dt("f32"), ("_ki",),
                            None)]
    body.append(StridedLoop(
        Axis("_ks", Dim(ksplit)), I(0), I(bk), (
            *copies(stage_next, kk_next), CpAsyncCommit(), CpAsyncWait(stages - 1),
            Sync(0, None, False),
            Loop(Axis("_ki", Dim(bk)), tuple(inner), False, False),
            Sync(0, None, False)), False, None, False))
    atomic = split_k > 1
    for i in range(rm):
        row = add(mul(ab, I(bm)), add(mul(au, I(rm)), I(i)))
        col = add(mul(nb, I(bn)), add(mul(nu, I(rn)), I(0)))
        body.append(Write("matmul", (row, col), tuple(acc(i, j) for j in range(rn)), dt("f32"),
                          atomic))
    mb, nbk = m // bm, n // bn

    def window(name: str, ext: int, parent: str, pext: int) -> Axis:
        return Axis(name, Dim(ext), Window(Axis(parent, Dim(pext)), None, None, False))

    axes = [window("a0_b", mb, "a0", m), window("a1_b", nbk, "a1", n),
            Axis("a0_u", Dim(ty)), Axis("a1_u", Dim(tx))]
    if split_k > 1:
        axes.insert(0, Axis("ak_s", Dim(split_k)))
    raster = ("a0_b", "a1_b") if raster_group else None
    tile = Tile(tuple(axes), tuple(body), block, 0, raster, raster_group, "m")
    # the shared tiles plus 2 KiB, which a kernel aligning its tiles to 1 KiB and keeping its
    # barriers beside them can use
    smem = stages * (bm * bk + bk * bn) * esz + 2048
    b_dist = ["normal", 0.0, b_std if b_std is not None else 1.0 / math.sqrt(k)]
    args = [_arg("x1", dtype, [k, n], seed=1, dist=b_dist),
            _arg("x0", dtype, [m, k], seed=0, dist=["normal", 0.0, 1.0]),
            _arg("matmul", "f32", [m, n], output=True)]
    pid = "c5_matmul" if split_k == 1 else "c5b_matmul_splitk"
    tdt = {"bf16": "torch.bfloat16", "f16": "torch.float16", "f32": "torch.float32"}[dtype]
    code = f"torch.randn({m}, {k}, dtype={tdt}) @ torch.randn({k}, {n}, dtype={tdt})"
    return _spec(pid, code, 1e-2, 1e-2, f"k_matmul_{m}x{n}x{k}" + (
        f"_s{split_k}" if split_k > 1 else ""), tile, args, ["x0", "x1"], ["matmul"], {}, block,
        smem_bytes=smem if smem > 48 * 1024 else 0,
        zero_outputs=["matmul"] if atomic else [])


def _cname(dtype: str) -> str:
    return {"bf16": "__nv_bfloat16", "f16": "half", "f32": "float"}[dtype]


# --- the benchmark configurations -------------------------------------------------------------

CONFIGS = {
    "c1_vector_add": lambda: pointwise_add(),
    "c2_gelu_chain": lambda: gelu_chain(),
    "c3_row_softmax": lambda: row_softmax(),
    "c4_full_sum": lambda: full_sum(),
    "c5_matmul": lambda: matmul(),
    "c5b_matmul_splitk": lambda: matmul(1024, 1024, 65536, split_k=4, raster_group=None),
}


# --- seeded inputs ---------------------------------------------------------------------------

_NP = {"f32": np.float32, "f64": np.float64, "f16": np.float16, "i32": np.int32,
       "i64": np.int64, "u8": np.uint8}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to bf16, nearest even, as raw uint16 bits."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_values(bits: np.ndarray) -> np.ndarray:
    """bf16 raw bits as the f32 values they hold."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def seeded_input(arg: dict[str, Any], chunk: int = 1 << 24) -> np.ndarray:
    """The host array of a meta.json argument: ``data`` for a constant, else
    ``default_rng(seed)`` drawn from its ``dist`` (standard normal by default); bf16 comes back
    as uint16 bits."""
    shape = [int(s) for s in arg["shape"]] or [1]
    dtype = arg["dtype"]
    if "data" in arg:
        vals = np.asarray(arg["data"], dtype=np.float64).reshape(shape)
        return bf16_bits(vals.astype(np.float32)) if dtype == "bf16" else vals.astype(_NP[dtype])
    rng = np.random.default_rng(int(arg.get("seed", 0)))
    dist = arg.get("dist", ["normal", 0.0, 1.0])
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.uint16 if dtype == "bf16" else _NP[dtype])
    for lo in range(0, n, chunk):
        cnt = min(chunk, n - lo)
        if dist[0] == "uniform":
            v = rng.uniform(dist[1], dist[2], cnt)
        else:
            v = rng.standard_normal(cnt) * dist[2] + dist[1]
        out[lo:lo + cnt] = bf16_bits(v.astype(np.float32)) if dtype == "bf16" else v
    return out.reshape(shape)

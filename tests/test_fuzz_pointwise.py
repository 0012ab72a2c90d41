"""Seeded random pointwise chains and row reductions through the generic lowering: a
differential test of the compiler against the oracle on Kernel IR nobody wrote by hand.

Each seed draws a chain of 2 to 9 IEEE round-to-nearest operations (add, subtract, multiply,
divide, maximum, minimum, abs, negative, relu, square, sqrt of an abs) over f32 or f64 inputs
of a random shape: flat sizes from 1 to 5000 or [rows, cols] with row and column broadcasts,
ConstantOp scalars, 1- to 8-wide unrolled bodies and blocks of 64 to 512 threads. Products
that feed adds meet the lowering's fma rule, packed f32x2 pairs, vector loads and stores and
tail guards wherever the shape leads them. Row reductions draw the rows, the row length (up to
3000, mostly ragged against the block) and the block (32 to 1024 threads), and reduce by sum, max
or sum of squares of x or |x|, then write the row's value or x divided by it plus one. Nests
draw matmuls with one thread per output element (random shapes, batch, ``F.linear`` layout, bias,
relu) and sums, maxima, minima and means over the middle axis of a 3-D input.

On the CPU every chain compiles under each flag set and assembles for sm_100a. On the GPU the
kernel's output equals the oracle's bit for bit (IEEE operations only, so nothing is
approximate), or under ``--no_fusion`` the oracle's with products rounded or fused, since ptxas
may contract there."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import gpu_run, oracle_run, reference_inputs
from test_compile import FLAG_SETS, ptxas

from ptxgen.compiler import to_ptx
from ptxgen.ir import Graph
from ptxgen.problems import ProblemSpec
from ptxgen.suite import In, Pointwise, Rowwise, S, axis_reduce, dot_nest

SEEDS = list(range(32))
BINARY = ["add", "subtract", "multiply", "divide", "maximum", "minimum"]
UNARY = ["abs", "negative", "relu", "square", "sqrt_abs"]


def random_chain(seed: int) -> ProblemSpec:
    rng = np.random.default_rng(1000 + seed)
    dtype = "f64" if rng.random() < 0.25 else "f32"

    # most sizes a multiple of 8, so unrolled bodies and vector accesses come into play
    def size(hi: int) -> int:
        return 8 * int(rng.integers(1, hi // 8 + 1)) if rng.random() < 0.6 else \
            int(rng.integers(1, hi + 1))
    if rng.random() < 0.5:
        shape: tuple[int, ...] = (size(5000),)
    else:
        shape = (int(rng.integers(1, 65)), size(300))
    inputs = [In(f"x{i}", dtype, shape) for i in range(int(rng.integers(1, 4)))]
    if len(shape) == 2 and rng.random() < 0.5:
        bc = str(rng.choice(["rows", "cols"]))
        inputs.append(In("bb", dtype, (shape[0] if bc == "rows" else shape[1],), bcast=bc))
    consts = {f"c{i}": float(rng.choice([0.5, 1.25, -3.0, 2.0, 1e-3, 7.5]))
              for i in range(int(rng.integers(0, 3)))}
    names = [i.name for i in inputs] + list(consts)
    steps = []
    for k in range(int(rng.integers(2, 10))):
        # lean on recent values so the chain stays connected
        pick = lambda: names[-1 - int(rng.integers(0, min(3, len(names))))]  # noqa: E731
        if rng.random() < 0.65:
            fn = str(rng.choice(BINARY, p=[0.25, 0.15, 0.3, 0.1, 0.1, 0.1]))
            steps.append(S(f"v{k}", fn, pick(), pick(), dtype=dtype))
        else:
            fn = str(rng.choice(UNARY))
            if fn == "sqrt_abs":
                steps.append(S(f"a{k}", "abs", pick(), dtype=dtype))
                steps.append(S(f"v{k}", "sqrt", f"a{k}", dtype=dtype))
            else:
                steps.append(S(f"v{k}", fn, pick(), dtype=dtype))
        names.append(f"v{k}")
    unroll, block = int(rng.choice([1, 2, 4, 8])), int(rng.choice([64, 128, 256, 512]))
    pw = Pointwise(f"z{seed:02d}_random_chain", "random IEEE chain", inputs,
                   ("out", dtype, shape), steps, steps[-1].name, consts, unroll, block)
    return pw.build()


def random_rows(seed: int) -> ProblemSpec:
    """One block per row of x [rows, cols]: a sum, max or sum of squares (of x or |x|) through
    the block reduction, then either the row's value or a sweep writing x normalised by it."""
    rng = np.random.default_rng(5000 + seed)
    block = int(rng.choice([32, 64, 128, 256, 512, 1024]))
    rows, cols = int(rng.integers(1, 48)), int(rng.integers(1, 3000))
    pre = [S("ax", "abs", "xv")] if rng.random() < 0.3 else []
    val = pre[-1].name if pre else "xv"
    kind = str(rng.choice(["add", "maximum", "sumsq"]))
    if kind == "sumsq":
        pre = [*pre, S("sq", "multiply", val, val)]
        val, kind = "sq", "add"
    passes: list[tuple] = [("reduce", "acc0", kind, pre, val)]
    consts = {"c_one": 1.0}
    if rng.random() < 0.5:
        passes.append(("row", "acc0"))
    else:
        passes += [("scalar", S("den", "add", "acc0", "c_one")),
                   ("write", [S("y", "divide", "xv", "den")], "y")]
    return Rowwise(f"z{seed:02d}_random_rows", "random row reduction", In("x", "f32", (rows, cols)),
                   ("out", "f32"), passes, consts, block).build()


def random_dot(seed: int) -> ProblemSpec:
    """A matmul with one thread per output element (``suite.dot_nest``): random m, n, k,
    batch, ``F.linear`` layout, bias, relu and block."""
    rng = np.random.default_rng(9000 + seed)
    m, n, k = (int(rng.integers(1, hi)) for hi in (70, 70, 300))
    return dot_nest(f"z{seed:02d}_random_dot", "random matmul", m, n, k,
                    batch=int(rng.choice([1, 1, 2, 3])), linear=bool(rng.random() < 0.4),
                    bias=bool(rng.random() < 0.4), relu=bool(rng.random() < 0.3),
                    block=int(rng.choice([32, 64, 128, 256])))


def random_axis(seed: int) -> ProblemSpec:
    """A reduction over the middle axis of x [a, b, c] (``suite.axis_reduce``): sum, max or min,
    or a mean, over random extents."""
    rng = np.random.default_rng(13000 + seed)
    shape = tuple(int(rng.integers(1, hi)) for hi in (9, 200, 97))
    fn = str(rng.choice(["add", "maximum", "minimum"]))
    return axis_reduce(f"z{seed:02d}_random_axis", "random axis reduction", shape, fn,
                       mean=fn == "add" and bool(rng.random() < 0.5),
                       block=int(rng.choice([32, 64, 128, 256])))


EXTRA = {"dot": random_dot, "axis": random_axis}


@pytest.mark.parametrize("seed", SEEDS)
def test_random_chain_compiles_and_assembles(seed: int, tmp_path) -> None:
    spec = random_chain(seed)
    for flags in FLAG_SETS:
        ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta, **flags)
        assert ".target sm_100a" in ptx
        ptxas(ptx, tmp_path)


@pytest.mark.parametrize("seed", SEEDS[:16])
def test_random_rows_compile_and_assemble(seed: int, tmp_path) -> None:
    spec = random_rows(seed)
    for flags in FLAG_SETS:
        ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta, **flags)
        assert ".target sm_100a" in ptx
        ptxas(ptx, tmp_path)


@pytest.mark.parametrize("kind", sorted(EXTRA))
@pytest.mark.parametrize("seed", SEEDS[:12])
def test_random_nests_compile_and_assemble(kind: str, seed: int, tmp_path) -> None:
    spec = EXTRA[kind](seed)
    for flags in FLAG_SETS:
        ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta, **flags)
        assert ".target sm_100a" in ptx
        ptxas(ptx, tmp_path)


def test_random_chains_cover_the_lowering() -> None:
    """The seeds reach both dtypes, broadcasts, constants, vector widths and ragged sizes."""
    specs = [random_chain(s) for s in SEEDS]
    args = [a for sp in specs for a in sp.kernel["args"]]
    assert {a["dtype"] for a in args if not a.get("data")} >= {"f32", "f64"}
    assert any(len(a["shape"]) == 2 for a in args)
    assert any("data" in a for a in args)
    ptx = "\n".join(to_ptx(Graph.from_dict(sp.graph), sp.meta) for sp in specs)
    for form in ("ld.global.nc.v4", "fma.rn", "div.rn", "sqrt.rn", ".f32x2"):
        assert form in ptx, form


@pytest.mark.gpu
@pytest.mark.parametrize("seed", SEEDS)
@pytest.mark.parametrize("flags", FLAG_SETS, ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_random_chain_matches_oracle(cuda, seed: int, flags: dict) -> None:
    from test_gpu_parity import check_flags

    spec = random_chain(seed)
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64, **flags)["out"]

    def run(nf: bool) -> np.ndarray:
        return oracle_run(spec.graph, spec.meta, ins, no_fusion=nf)["out"]

    dtype = next(a["dtype"] for a in spec.kernel["args"] if a["name"] == "out")
    check_flags("exact", got, run, dtype, 0, flags)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", SEEDS[:16])
@pytest.mark.parametrize("flags", FLAG_SETS, ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_random_rows_match_oracle(cuda, seed: int, flags: dict) -> None:
    """Single-block reductions add in one fixed order (a warp's shuffle ladder, then the
    halving tree over warps), so the GPU equals the oracle bit for bit."""
    from test_gpu_parity import check_flags

    spec = random_rows(seed)
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64, **flags)["out"]

    def run(nf: bool) -> np.ndarray:
        return oracle_run(spec.graph, spec.meta, ins, no_fusion=nf)["out"]

    check_flags("exact", got, run, "f32", 0, flags)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", sorted(EXTRA))
@pytest.mark.parametrize("seed", SEEDS[:12])
@pytest.mark.parametrize("flags", FLAG_SETS, ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_random_nests_match_oracle(cuda, kind: str, seed: int, flags: dict) -> None:
    """Each output element's loop adds in index order, so the GPU equals the oracle bit for
    bit."""
    from test_gpu_parity import check_flags

    spec = EXTRA[kind](seed)
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64, **flags)["out"]

    def run(nf: bool) -> np.ndarray:
        return oracle_run(spec.graph, spec.meta, ins, no_fusion=nf)["out"]

    check_flags("exact", got, run, "f32", 0, flags)

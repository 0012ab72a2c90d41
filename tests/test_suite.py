"""The op/dtype suite (``ptxgen.suite``) on the CPU: every case compiles to PTX that ptxas
accepts for sm_100a under each flag set, and the oracle's run of its Kernel IR meets the
reference's NumPy formula for that problem within the reference's tolerance. This pins each
generated IR to the reference's problem and the oracle to its semantics; the GPU tests then hold
the kernels to the oracle."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import oracle_run, reference_inputs
from test_compile import FLAG_SETS, assert_plain_tma, ptxas

from ptxgen.compiler import to_ptx
from ptxgen.ir import Graph
from ptxgen.suite import MULTI, SUITE, ref_inputs


def as_values(case, got: np.ndarray) -> np.ndarray:
    from ptxgen.problems import bf16_values

    return bf16_values(got) if case.out_dtype == "bf16" else got


@pytest.mark.parametrize("name", sorted(SUITE))
def test_suite_compiles(name: str, tmp_path) -> None:
    spec = SUITE[name]().spec
    for flags in FLAG_SETS:
        ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta, **flags)
        assert ".target sm_100a" in ptx
        assert_plain_tma(ptx)
        if not flags:
            ptxas(ptx, tmp_path)


@pytest.mark.parametrize("name", sorted(SUITE))
def test_suite_oracle_meets_reference_formula(name: str) -> None:
    case = SUITE[name]()
    ins = reference_inputs(case.spec.meta)
    got = as_values(case, oracle_run(case.spec.graph, case.spec.meta, ins)[case.out])
    want = np.asarray(case.ref(*ref_inputs(case, ins)))
    got, want = got.astype(np.float64).reshape(want.shape), want.astype(np.float64)
    np.testing.assert_allclose(got, want, rtol=case.rtol, atol=case.atol)


def test_packed_sub_of_a_product_stays_scalar() -> None:
    """A multiply this backend does not fuse must stay two roundings: the SLP pass keeps an
    add or sub that reads a product scalar (its explicit .rn forbids ptxas to contract), since
    the packed f32x2 forms came out contracted on a B200. ``a * b - c`` is such a case: only an
    add of a product fuses."""
    spec = SUITE["p09_fms"]().spec
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    assert ".f32x2" not in ptx and "fma.rn" not in ptx
    assert ptx.count("mul.rn.f32 ") == ptx.count("sub.rn.f32 ") == 4


def test_no_fusion_writes_the_reference_forms() -> None:
    """``--no_fusion`` writes a multiply and an add without a rounding modifier, as the
    reference does, so ptxas may contract them; with fusion on they are one ``fma.rn``."""
    spec = SUITE["p07_fma3"]().spec
    plain = to_ptx(Graph.from_dict(spec.graph), spec.meta, no_fusion=True)
    fused = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    def ops(ptx: str) -> list[str]:
        return [ln.split()[0] for ln in ptx.splitlines() if ln.startswith("\t") and
                not ln.startswith("\t.")]

    assert ops(plain).count("mul.f32") == ops(plain).count("add.f32") == 4
    assert not any(".rn" in o or o.startswith("fma") for o in ops(plain))
    lanes = ops(fused).count("fma.rn.f32") + 2 * ops(fused).count("fma.rn.f32x2")
    assert "mul.rn.f32" not in ops(fused) and lanes == 4


# --- problems of several kernels ---------------------------------------------------------------


def multi_inputs(meta) -> dict[str, np.ndarray]:
    from ptxgen.problems import seeded_input
    from ptxgen.runtime import problem_args

    return {n: seeded_input(a) for n, a in problem_args(meta).items()
            if not a.get("output") and not a.get("intermediate")}


@pytest.mark.parametrize("name", sorted(MULTI))
def test_multi_kernel_problem_compiles_and_meets_formula(name: str, tmp_path) -> None:
    from oracle.interp import run_problem

    case = MULTI[name]()
    for k in case.spec.meta["kernels"]:
        ptxas(to_ptx(Graph.from_dict(case.spec.graphs[k["entry"]]), case.spec.meta), tmp_path)
    ins = multi_inputs(case.spec.meta)
    out = run_problem(case.spec.graphs, case.spec.meta, ins)["out"]
    want = np.asarray(case.ref(*[ins[n] for n in case.spec.meta["graph_inputs"]]))
    np.testing.assert_allclose(out.reshape(want.shape), want, rtol=case.rtol, atol=case.atol)


def test_multi_kernel_dir_through_the_cli(tmp_path) -> None:
    """The drop-in CLI compiles each kernel of a chained problem from its own IR file, reading
    the shared meta.json beside it (reference compile.py:58-69)."""
    import subprocess
    import sys

    from conftest import ROOT

    case = MULTI["f13_softmax_two_pass"]()
    d = case.spec.write(tmp_path / "f13")
    for k in case.spec.meta["kernels"]:
        r = subprocess.run([sys.executable, str(ROOT / "compile.py"),
                            str(d / f"{k['entry']}.ir.json")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert f".visible .entry {k['entry']}(" in r.stdout


def test_intermediate_without_producer_is_rejected() -> None:
    from ptxgen.runtime import problem_args

    meta = MULTI["r17_grid_kernel"]().spec.meta
    meta["kernels"] = meta["kernels"][1:]  # the consumer alone
    with pytest.raises(ValueError, match="intermediate"):
        problem_args(meta)

"""The benchmark configurations at their full sizes, through properties that do not depend on
the size.

* Configs 2 and 3: every output row depends only on its own input row (and config 2's per-row
  scale), so the first, the last and random rows of the full-size GPU output are checked
  against the oracle's run of the same kernel on just those rows, at the small cases' bars
  (one bf16 ulp; rel 2e-5). Each of config 3's 16384 rows also sums to 1.
* Config 4: the sum of all 2^30 elements against an f64 sum of the same data (rel 1e-5).
* Configs 5 and 5b: sampled full rows of C against the f64 product of the same bf16 operands
  (rel 1e-2 per element, floor 1e-3 of the largest |C| in those rows).
* The reference's ``m06_1024sq`` (an f32 1024^3 matmul on the SIMT nest, whose oracle run at
  full size takes most of a minute): a tile of C depends only on its rows of A and columns of B,
  so three 128 x 128 tiles of the full-size GPU result are checked bit for bit against the
  oracle's run of the one-tile problem on those rows and columns.

The independence these checks rest on is itself checked on the CPU: the oracle's run on picked
rows (or one tile) equals its run on the whole problem.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import gpu_run, oracle_run, reference_inputs

from ptxgen import problems


def picked_rows(rows: int, count: int = 16, seed: int = 7) -> np.ndarray:
    """The first and last rows and ``count`` others, sorted."""
    rng = np.random.default_rng(seed)
    return np.array(sorted({0, rows - 1, *rng.choice(rows, count, replace=False).tolist()}))


def gelu_on_rows(spec: problems.ProblemSpec, ins: dict[str, np.ndarray], rows: np.ndarray
                 ) -> tuple[problems.ProblemSpec, dict[str, np.ndarray]]:
    """Config 2's kernel over only ``rows`` of ``ins`` (same constants a, b)."""
    cols = int(ins["x"].shape[1])
    a, b = float(ins["mul_c1"][0]), float(ins["add_c1"][0])
    small = problems.gelu_chain(len(rows), cols, a=a, b=b)
    return small, {"mul_c1": ins["mul_c1"], "add_c1": ins["add_c1"],
                   "x": np.ascontiguousarray(ins["x"][rows]), "s": ins["s"][rows]}


def test_oracle_rows_are_independent() -> None:
    """The oracle's output rows of configs 2 and 3 on picked rows equal its rows of the whole
    problem: the premise of the full-size row checks."""
    spec = problems.gelu_chain(40, 256)
    ins = reference_inputs(spec.meta)
    whole = oracle_run(spec.graph, spec.meta, ins)["mul_1"]
    rows = picked_rows(40, 6)
    small, sub = gelu_on_rows(spec, ins, rows)
    assert np.array_equal(oracle_run(small.graph, small.meta, sub)["mul_1"], whole[rows])

    spec = problems.row_softmax(24, 1024)
    ins = reference_inputs(spec.meta)
    whole = oracle_run(spec.graph, spec.meta, ins)["softmax"]
    rows = picked_rows(24, 5)
    small = problems.row_softmax(len(rows), 1024)
    got = oracle_run(small.graph, small.meta, {"x": np.ascontiguousarray(ins["x"][rows])})
    assert np.array_equal(got["softmax"], whole[rows])

    from ptxgen.suite import m06_1024sq

    spec = m06_1024sq(256, 256)
    ins = reference_inputs(spec.meta)
    whole = oracle_run(spec.graph, spec.meta, ins)["matmul"]
    tile = oracle_run(m06_1024sq(128, 128).graph, m06_1024sq(128, 128).meta,
                      m06_tile_inputs(ins, 1, 1))["matmul"]
    assert np.array_equal(tile, whole[128:, 128:])


@pytest.mark.gpu
def test_c2_full_size_rows(cuda) -> None:
    from test_gpu_parity import check

    spec = problems.CONFIGS["c2_gelu_chain"]()
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins)["mul_1"]
    rows = picked_rows(got.shape[0])
    small, sub = gelu_on_rows(spec, ins, rows)
    want = oracle_run(small.graph, small.meta, sub)["mul_1"]
    check("ulp", got[rows], want, "bf16", 1)


@pytest.mark.gpu
def test_c3_full_size_rows(cuda) -> None:
    from test_gpu_parity import check

    spec = problems.CONFIGS["c3_row_softmax"]()
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins)["softmax"]
    sums = got.astype(np.float64).sum(axis=1)
    assert np.abs(sums - 1).max() < 1e-4, np.abs(sums - 1).max()
    rows = picked_rows(got.shape[0])
    cols = got.shape[1]
    small = problems.row_softmax(len(rows), cols)
    want = oracle_run(small.graph, small.meta,
                      {"x": np.ascontiguousarray(ins["x"][rows])})["softmax"]
    check("rel", got[rows], want, "f32", 2e-5)


@pytest.mark.gpu
def test_c4_full_size_against_f64(cuda) -> None:
    """2^30 f32 elements ~ U(0,1) drawn on the device; the kernel's sum against torch's f64
    sum of the same tensor (the checker only)."""
    import torch

    from ptxgen.runtime import Problem

    spec = problems.CONFIGS["c4_full_sum"]()
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    gen = torch.Generator(device=cuda)
    gen.manual_seed(0)
    tensors["x"].uniform_(0.0, 1.0, generator=gen)
    tensors["sum_1"].fill_(float("nan"))
    prob.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    got = float(tensors["sum_1"][0])
    want = float(torch.sum(tensors["x"], dtype=torch.float64))
    assert abs(got / want - 1) < 1e-5, (got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["c5_matmul", "c5b_matmul_splitk", "c5_matmul/4", "c5_matmul/8"])
def test_gemm_full_size_rows(cuda, key: str) -> None:
    """Config 5 at 8192^3, and the 1/4 and 1/8 shares one rank of a strong-scaled run holds
    (2048 and 1024 rows): the picked rows of C (first, last and 16 seeded picks); config 5b
    (1024 x 1024 x 65536, split-K): every row of C. Each against the f64 product of the same
    bf16 operands, at the GEMM bar."""
    from test_gpu_gemm import assert_gemm_close

    from oracle.fp import bf16_bits_to_f32
    from ptxgen import shard

    name, _, share = key.partition("/")
    spec = shard.local_problem(name, int(share or 1)).spec
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins)["matmul"]
    rows = picked_rows(got.shape[0]) if name == "c5_matmul" else np.arange(got.shape[0])
    a = bf16_bits_to_f32(ins["x0"][rows]).astype(np.float64)
    b = bf16_bits_to_f32(ins["x1"]).astype(np.float64)
    worst = assert_gemm_close(got[rows], a @ b)
    print(f"{key}: {len(rows)} rows, max |err| / max |C| = {worst:.3e}")


def m06_tile_inputs(ins: dict[str, np.ndarray], r: int, c: int) -> dict[str, np.ndarray]:
    """The operands of the one-tile problem for tile (r, c) of the 128 x 128 tiling."""
    return {"x0": np.ascontiguousarray(ins["x0"][128 * r:128 * (r + 1)]),
            "x1": np.ascontiguousarray(ins["x1"][:, 128 * c:128 * (c + 1)])}


def test_m06_tile_oracle_meets_reference_formula() -> None:
    """The reference's m06_1024sq formula (f64 product, rtol/atol 1e-3) on one tile, through
    the oracle's run of the one-tile problem."""
    from ptxgen.suite import m06_1024sq

    ins = reference_inputs(m06_1024sq().meta)
    small = m06_1024sq(128, 128)
    got = oracle_run(small.graph, small.meta, m06_tile_inputs(ins, 7, 7))["matmul"]
    want = ins["x0"][896:].astype(np.float64) @ ins["x1"][:, 896:].astype(np.float64)
    np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
def test_m06_1024sq_tiles(cuda) -> None:
    """m06_1024sq at its full size on the GPU: its first and last 128 x 128 tiles equal, bit for
    bit, the oracle's run of the one-tile problem on those rows and columns."""
    from test_gpu_parity import check

    from ptxgen.suite import m06_1024sq

    spec = m06_1024sq()
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64)["matmul"]
    small = m06_1024sq(128, 128)
    for r, c in [(0, 0), (7, 7), (3, 5)]:
        want = oracle_run(small.graph, small.meta, m06_tile_inputs(ins, r, c))["matmul"]
        check("exact", got[128 * r:128 * (r + 1), 128 * c:128 * (c + 1)], want, "f32")

"""Warp rows fetched 8 bytes a lane through shared memory (``ptxgen.stage``).

A per-thread grid-stride sum (each thread writes its own sum, so the result does not depend on
any atomic order) over a grid of several waves takes the rewrite with whole blocks, and keeps its
scalar loads with a partial last block or in a grid of one wave. On the GPU the staged sums must
equal the oracle's bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import reference_inputs

from ptxgen import problems
from ptxgen.compiler import to_ptx
from ptxgen.ir import (Accum, Axis, Dim, ElementwiseImpl, Graph, Load, StridedLoop, Tile, Var,
                       Write, dt)

F32 = dt("f32")


def per_thread_sum(threads: int, n: int, block: int) -> problems.ProblemSpec:
    """out[t] = x[t] + x[t + threads] + ... over n elements, in that order, one thread per t."""
    from ptxgen.problems import _arg, _spec

    t = Var("a0")
    loop = StridedLoop(Axis("i", Dim(n)), t, threads,
                       (Load(("xv",), "x", (Var("i"),), F32),
                        Accum("acc", "xv", ElementwiseImpl("add"), F32, ("i",), None)),
                       False, None, True)
    tile = Tile((Axis("a0", Dim(threads)),), (loop, Write("out", (t,), ("acc",), F32)), None)
    args = [_arg("x", "f32", [n], seed=0, dist=["uniform", 0.0, 1.0]),
            _arg("out", "f32", [threads], output=True)]
    return _spec("stage_sum", "per-thread grid-stride sums", 0, 0, "k_stage_sum", tile, args,
                 ["x"], ["out"], {}, block)


def loop_of(ptx: str) -> str:
    return ptx[ptx.index("$L_loop_1:"):ptx.index("$L_loop_end_2:")]


WAVES = 160 * 256  # 160 blocks of 256 threads: more blocks than the B200's 148 SMs


def test_whole_blocks_are_staged() -> None:
    spec = per_thread_sum(WAVES, WAVES * 64, 256)
    loop = loop_of(to_ptx(Graph.from_dict(spec.graph), spec.meta))
    assert loop.count("bar.warp.sync") == 2 and "ld.global.nc.v2.f32" in loop
    assert "ld.global.nc.f32" not in loop


def test_partial_last_block_keeps_scalar_loads() -> None:
    """A grid 100 threads short of whole blocks of 256: the last block's threads past the end
    skip the body, so a warp sync there would wait on lanes that never come."""
    spec = per_thread_sum(WAVES - 100, (WAVES - 100) * 64, 256)
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    assert "bar.warp.sync" not in ptx and "ld.global.nc.f32" in ptx


def test_one_wave_keeps_its_unroll() -> None:
    """4 blocks: an SM holds too few warps to cover a staged trip's round of loads, stores and
    syncs (the shipped r02, one block, took 26.7 us staged against 14.3 unrolled)."""
    spec = per_thread_sum(1024, 1024 * 4096, 256)
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    assert "bar.warp.sync" not in ptx


def test_flags_keep_it_where_they_keep_the_loop() -> None:
    """The rewrite changes no value, so, like the copy ring, it stays under the flags that keep
    the counted loop (with CSE off every address is recomputed and there is no pointer)."""
    spec = per_thread_sum(WAVES, WAVES * 64, 256)
    g = Graph.from_dict(spec.graph)
    assert "bar.warp.sync" in to_ptx(g, spec.meta, no_fusion=True)
    assert "bar.warp.sync" not in to_ptx(g, spec.meta, no_cse=True)


@pytest.mark.gpu
@pytest.mark.parametrize("threads,block,trips", [(WAVES, 256, 64), (150 * 512, 512, 40),
                                                (WAVES, 256, 4096 // 32)])
def test_staged_sums_equal_the_oracle(cuda, threads: int, block: int, trips: int) -> None:
    from conftest import gpu_run, oracle_run

    spec = per_thread_sum(threads, threads * trips, block)
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    assert "bar.warp.sync" in ptx
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=16, ptx=ptx)["out"]
    want = oracle_run(spec.graph, spec.meta, ins)["out"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_strided_rows_keep_scalar_loads() -> None:
    """A loop over every other element: a warp's lanes read 4 bytes out of each 8, not one
    contiguous row, so nothing is staged."""
    from ptxgen.ir import BinaryExpr, Literal
    from ptxgen.problems import _arg, _spec

    t, threads = Var("a0"), WAVES
    n = threads * 64
    loop = StridedLoop(Axis("i", Dim(n)), t, threads,
                       (Load(("xv",), "x", (BinaryExpr("*", Var("i"), Literal(2)),), F32),
                        Accum("acc", "xv", ElementwiseImpl("add"), F32, ("i",), None)),
                       False, None, True)
    tile = Tile((Axis("a0", Dim(threads)),), (loop, Write("out", (t,), ("acc",), F32)), None)
    args = [_arg("x", "f32", [2 * n], seed=0, dist=["uniform", 0.0, 1.0]),
            _arg("out", "f32", [threads], output=True)]
    spec = _spec("stage_strided", "every other element", 0, 0, "k_stage_strided", tile, args,
                 ["x"], ["out"], {}, 256)
    assert "bar.warp.sync" not in to_ptx(Graph.from_dict(spec.graph), spec.meta)

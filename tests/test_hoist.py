"""Work a loop repeats across one thread axis, done once and shared (``ptxgen.hoist``).

The oracle runs each attention IR as written and as rewritten; the outputs must agree bit for bit
(the oracle keeps shared memory per block, like the GPU). Small loops built here check the cases
the rewrite must leave alone. On the GPU the rewritten build must equal the build without it, bit
for bit, on all 11 attention IRs.
"""

from __future__ import annotations

import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
from conftest import reference_inputs

from oracle.interp import Interpreter
from ptxgen.compiler import kernel_for_meta, to_ptx
from ptxgen.congruence import merge_equal
from ptxgen.hoist import share_invariant
from ptxgen.ir import (Accum, Assign, Axis, BinaryExpr, Dim, ElementwiseImpl, Graph, Let, Load,
                       Loop, Smem, StridedLoop, Sync, Tile, Var, Write, dt)
from ptxgen.jam import jam
from ptxgen.suite import SUITE

SHIPPED = Path(__file__).parent / "golden" / "shipped"
F32 = dt("f32")
ATTENTION = sorted(n for n in SUITE if n.startswith("a0"))
SMALL = ("a00_small", "a02_rect", "a03_noscale", "a05_heads")  # quick in the oracle


def shipped(name: str) -> tuple[dict, dict]:
    d = SHIPPED / name
    return (json.loads(next(d.glob("*.ir.json")).read_text()),
            json.loads((d / "meta.json").read_text()))


def rewritten(graph: dict, meta: dict):
    """(the kernel as the compiler sees it before the rewrite, after it)."""
    op, launch = kernel_for_meta(Graph.from_dict(graph), meta)
    tile = replace(op.body, body=merge_equal(jam(op.body.body)))
    return replace(op, body=tile), replace(op, body=share_invariant(tile, launch["block"][0]))


@pytest.mark.parametrize("key", ["a01_attention", "a03_noscale", *SMALL])
def test_attention_rewrite_is_bit_equal_in_the_oracle(key: str) -> None:
    graph, meta = shipped(key) if key in ("a01_attention", "a03_noscale") else \
        (SUITE[key]().spec.graph, SUITE[key]().spec.meta)
    before, after = rewritten(graph, meta)
    assert after.body is not before.body
    ins = reference_inputs(meta)
    want = Interpreter(graph, meta, ins, op=before).run()
    got = Interpreter(graph, meta, ins, op=after).run()
    for k in want:
        assert np.array_equal(want[k].view(np.uint8), got[k].view(np.uint8)), k


def test_shipped_a01_shape_of_the_rewrite() -> None:
    """a01's scores are computed once per row group and key: each thread takes every 16th key
    from its own ``a5_u``, its 4 rows' scaled scores go to a 32 x 64 shared array, a barrier,
    then the key loop reads them back and keeps the rest of its statements."""
    graph, meta = shipped("a01_attention")
    before, after = rewritten(graph, meta)
    body = after.body.body
    smem = [s for s in body if isinstance(s, Smem)]
    assert [(s.extents, s.dtype) for s in smem] == [((32, 64), "float")]
    i = next(n for n, s in enumerate(body) if isinstance(s, StridedLoop))
    head, sync, loop = body[i], body[i + 1], body[i + 2]
    assert head.start == Var("a5_u") and head.step == 16 and isinstance(sync, Sync)
    assert sum(isinstance(s, Loop) for s in head.body) == 1  # the jammed dot products
    writes = [s for s in head.body if isinstance(s, Write)]
    loads = [s for s in loop.body if isinstance(s, Load) and s.input == smem[0].name]
    assert len(writes) == len(loads) == 4
    old_loop = next(s for s in before.body.body if isinstance(s, Loop))
    kept = [s for s in old_loop.body if not isinstance(s, Loop) and s not in head.body]
    assert list(loop.body[4:]) == kept


def test_no_other_ir_changes() -> None:
    """Only the attention nests repeat work across a thread axis."""
    for key in sorted(SUITE):
        if key in ATTENTION:
            continue
        spec = SUITE[key]().spec
        for op in Graph.from_dict(spec.graph).kernel_ops():
            launch = next(k for k in spec.meta["kernels"] if k["entry"] == op.name)
            tile = replace(op.body, body=merge_equal(jam(op.body.body)))
            assert share_invariant(tile, launch["block"][0]) is tile, key
    for d in sorted(SHIPPED.iterdir()):
        if d.name in ("a01_attention", "a03_noscale"):
            continue
        before, after = rewritten(*shipped(d.name))
        assert after.body is before.body, d.name


def test_flags_turn_it_off() -> None:
    graph, meta = shipped("a01_attention")
    g = Graph.from_dict(graph)
    assert "bar.sync" in to_ptx(g, meta)
    for flag in ("no_unroll", "no_fusion", "no_cse"):
        assert "bar.sync" not in to_ptx(g, meta, **{flag: True})
    assert "bar.sync" not in to_ptx(g, meta, templates=False)


# --- loops the rewrite must leave alone -------------------------------------------------------

A2 = Axis("d", Dim(8))


def tile_of(loop_body, prefix=(), block=32, blocks=2, axes=(("r", 4), ("x", 8))) -> Tile:
    key = Loop(Axis("k", Dim(16)), tuple(loop_body), True)
    return Tile(tuple(Axis(n, Dim(e)) for n, e in (("blk", blocks), *axes)),
                (*prefix, key, Write("o", (Var("r"),), ("acc",), F32)), block)


def dot(index) -> Loop:
    return Loop(A2, (Load(("qv",), "q", index, F32), Load(("kv",), "kt", (Var("d"), Var("k")), F32),
                     Assign("p", ElementwiseImpl("multiply"), ("qv", "kv"), F32),
                     Accum("s", "p", ElementwiseImpl("add"), F32, ("d",), None)))


def fold(value: str = "s") -> Accum:
    return Accum("acc", value, ElementwiseImpl("add"), F32, ("k",), None)


def test_leading_work_per_row_is_shared() -> None:
    t = tile_of([dot((Var("r"), Var("d"))), fold()])
    assert share_invariant(t, 32) is not t


def test_work_that_uses_every_thread_axis_stays() -> None:
    t = tile_of([dot((BinaryExpr("+", Var("r"), Var("x")), Var("d"))), fold()])
    assert share_invariant(t, 32) is t


def test_work_reading_the_loop_state_stays() -> None:
    body = [Loop(A2, (Load(("qv",), "q", (Var("r"), Var("d")), F32),
                      Assign("p", ElementwiseImpl("multiply"), ("qv", "acc"), F32),
                      Accum("s", "p", ElementwiseImpl("add"), F32, ("d",), None))), fold()]
    t = tile_of(body)
    assert share_invariant(t, 32) is t


def test_axis_reached_through_a_name_before_the_loop_stays() -> None:
    """The dot product's row comes from a Let over ``x``: it differs along x after all."""
    prefix = [Let("row", BinaryExpr("+", Var("r"), Var("x")), dt("i32"))]
    t = tile_of([dot((Var("row"), Var("d"))), fold()], prefix=prefix)
    assert share_invariant(t, 32) is t


def test_partial_blocks_stay() -> None:
    """96 threads in blocks of 64: the last block is partial, and a barrier needs them all."""
    t = tile_of([dot((Var("r"), Var("d"))), fold()], block=64, blocks=3)
    assert share_invariant(t, 64) is t


# --- GPU ------------------------------------------------------------------------------------------


@pytest.mark.gpu
@pytest.mark.parametrize("key", ["a01_attention", "a03_noscale", *ATTENTION])
def test_rewrite_bit_equal_on_the_gpu(cuda, key: str) -> None:
    """The default build (rewritten) against the same kernel without templates or the rewrite,
    bit for bit; the canaries past the output must survive."""
    from conftest import gpu_run

    graph, meta = shipped(key) if key in ("a01_attention", "a03_noscale") else \
        (SUITE[key]().spec.graph, SUITE[key]().spec.meta)
    g = Graph.from_dict(graph)
    ptx = to_ptx(g, meta)
    assert "bar.sync" in ptx
    ins = reference_inputs(meta)
    out = meta["graph_outputs"][0]
    got = gpu_run(graph, meta, ins, guard=64, ptx=ptx)[out]
    want = gpu_run(graph, meta, ins, guard=64, ptx=to_ptx(g, meta, templates=False))[out]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))

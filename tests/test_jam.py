"""Loop jamming (``ptxgen.jam``): which sibling loops merge, and that the shipped attention
nests' per-row inner products become one loop per key."""

from __future__ import annotations

from conftest import shipped

from ptxgen.compiler import kernel_for_meta, to_ptx
from ptxgen.ir import Accum, Assign, Axis, Dim, ElementwiseImpl, Graph, Literal, Load, Loop, Var, Write
from ptxgen.jam import can_jam, jam

A = Axis("d", Dim(8))


def _dot(row: str, extra: tuple = ()) -> Loop:
    """acc_<row> += q[row, d] * kt[d, 0] over d."""
    body = (Load((f"q_{row}",), "q", (Literal(int(row[-1])), Var("d"))),
            Load((f"k_{row}",), "kt", (Var("d"), Literal(0))),
            Assign(f"p_{row}", ElementwiseImpl("multiply"), (f"q_{row}", f"k_{row}")),
            Accum(f"acc_{row}", f"p_{row}", ElementwiseImpl("add"), None, ("d",)), *extra)
    return Loop(A, body)


def test_independent_rows_jam_into_one_loop() -> None:
    out = jam((_dot("r0"), _dot("r1"), _dot("r2")))
    assert len(out) == 1 and isinstance(out[0], Loop) and len(out[0].body) == 12


def test_a_loop_that_reads_another_loops_result_stays_apart() -> None:
    reader = Loop(A, (Load(("x",), "q", (Literal(0), Var("d"))),
                      Assign("y", ElementwiseImpl("add"), ("x", "acc_r0")),
                      Accum("acc_y", "y", ElementwiseImpl("add"), None, ("d",))))
    assert not can_jam(_dot("r0"), reader)
    assert len(jam((_dot("r0"), reader))) == 2


def test_loops_with_memory_writes_or_other_axes_stay_apart() -> None:
    writes = _dot("r1", (Write("out", (Var("d"),), ("acc_r1",), None, False),))
    assert not can_jam(_dot("r0"), writes)
    other = Loop(Axis("e", Dim(8)), _dot("r1").body)
    assert not can_jam(_dot("r0"), other)


def _key_loop_children(name: str) -> list[str]:
    from dataclasses import replace

    graph, meta = shipped(name)
    op, _ = kernel_for_meta(Graph.from_dict(graph), meta)
    op = replace(op, body=replace(op.body, body=jam(op.body.body)))
    key = next(st for st in op.body.body if isinstance(st, Loop))
    return [type(st).__name__ for st in key.body]


def test_shipped_attention_rows_jam() -> None:
    """a01 computes four rows' scores per key and a03 six: one loop each after jamming. With
    unrolling off the jammed loop is still a runtime loop, one body per trip: a01's module has
    two loops, the key loop and the row loop inside it (five before jamming)."""
    assert _key_loop_children("a01_attention").count("Loop") == 1
    assert _key_loop_children("a03_noscale").count("Loop") == 1
    graph, meta = shipped("a01_attention")
    rolled = to_ptx(Graph.from_dict(graph), meta, no_unroll=True)
    assert rolled.count("bra $L_loop_") == 2 and rolled.count("fma.rn.f32") >= 4

"""Merging accumulators that hold equal values on every trip (``ptxgen.congruence``).

The positive cases run the oracle on each attention IR before and after the pass and require
the outputs bit for bit equal. The negative cases are small loops built here, where a merge would
change a value, and check that the pass leaves them alone.
"""

from __future__ import annotations

import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
from conftest import reference_inputs

from oracle.interp import Interpreter
from ptxgen.compiler import to_ptx
from ptxgen.congruence import merge_equal
from ptxgen.ir import (Accum, Assign, Axis, Dim, ElementwiseImpl, Graph, Let, Literal, Load, Loop,
                       Var, Write, dt, walk)
from ptxgen.jam import jam
from ptxgen.suite import SUITE

SHIPPED = Path(__file__).parent / "golden" / "shipped"
F32 = dt("f32")


def shipped(name: str) -> tuple[dict, dict]:
    d = SHIPPED / name
    return json.loads(next(d.glob("*.ir.json")).read_text()), json.loads((d / "meta.json").read_text())


def oracle_both(graph: dict, meta: dict) -> tuple[dict, dict, tuple, tuple]:
    """The oracle's outputs on the jammed body and on the merged one, and the two bodies."""
    ins = reference_inputs(meta)
    before = Interpreter(graph, meta, ins)
    body = jam(before.op.body.body)
    before.op = replace(before.op, body=replace(before.op.body, body=body))
    merged = merge_equal(body)
    after = Interpreter(graph, meta, ins)
    after.op = replace(after.op, body=replace(after.op.body, body=merged))
    return before.run(), after.run(), body, merged


def accums(body) -> list[str]:
    return [s.name for s in walk(body) if isinstance(s, Accum)]


@pytest.mark.parametrize("name", ["a01_attention", "a03_noscale"])
def test_shipped_attention_merges_bit_equal(name: str) -> None:
    """Each query row's running max and sum of exponentials were carried once per output column.
    After the pass, one copy per row remains, the output sums all stay, and the oracle's result
    is unchanged bit for bit."""
    graph, meta = shipped(name)
    want, got, body, merged = oracle_both(graph, meta)
    for k in want:
        assert np.array_equal(want[k].view(np.uint8), got[k].view(np.uint8)), k
    before, after = accums(body), accums(merged)
    maxes = [n for n in before if n.startswith("acc1__")]
    sums = [n for n in before if n.startswith("acc3__")]
    outs = [n for n in before if n.startswith("acc5__")]
    assert maxes and sums and outs
    rows = {n.split("__c")[1].split("_")[0] for n in maxes}
    assert len([n for n in after if n.startswith("acc1__")]) == len(rows)
    assert len([n for n in after if n.startswith("acc3__")]) == len(rows)
    assert [n for n in after if n.startswith("acc5__")] == outs


@pytest.mark.parametrize("name", sorted(n for n in SUITE if n.startswith("a0")))
def test_suite_attention_merges_bit_equal(name: str) -> None:
    case = SUITE[name]()
    want, got, body, merged = oracle_both(case.spec.graph, case.spec.meta)
    assert len(accums(merged)) < len(accums(body))
    for k in want:
        assert np.array_equal(want[k].view(np.uint8), got[k].view(np.uint8)), k


def test_rolled_a01_one_exponential_per_row_and_column() -> None:
    """With unrolling off, a key step of the shipped a01 computes two exponentials per query row
    (the rescale of the old state and the new key's weight) for its 4 rows: 8, not 16. Under
    ``--no_cse`` the pass is off and all 16 stay."""
    graph, meta = shipped("a01_attention")
    g = Graph.from_dict(graph)
    assert to_ptx(g, meta, no_unroll=True).count("ex2.approx") == 8
    assert to_ptx(g, meta, no_unroll=True, no_cse=True).count("ex2.approx") == 16


def test_nothing_else_in_the_suite_changes() -> None:
    """Only the attention nests carry equal accumulators: every other case's body is returned
    as it was."""
    for name in sorted(SUITE):
        if name.startswith("a0"):
            continue
        case = SUITE[name]()
        graph = Graph.from_dict(case.spec.graph)
        for op in graph.kernel_ops():
            body = jam(op.body.body)
            assert merge_equal(body) == tuple(body), name


# --- small loops where a merge would be wrong ------------------------------------------------

A = Axis("a", Dim(8))


def load(name: str, buf: str = "x") -> Load:
    return Load((name,), buf, (Var("a"),), F32)


def acc(name: str, value: str, op: str = "add", base: str | None = None) -> Accum:
    return Accum(name, value, ElementwiseImpl(op), F32, ("a",), base)


def mul(name: str, *args: str) -> Assign:
    return Assign(name, ElementwiseImpl("multiply"), args, F32)


def out(*values: str) -> Write:
    return Write("y", (Literal(0),), values)


def test_equal_accumulators_merge_and_later_reads_follow() -> None:
    body = (Loop(A, (load("v"), acc("s1", "v"), acc("s2", "v"))), out("s1", "s2"))
    got = merge_equal(body)
    assert accums(got) == ["s1"]
    assert got[1].values == ("s1", "s1")


def test_different_values_do_not_merge() -> None:
    body = (Loop(A, (load("v"), load("w", "z"), acc("s1", "v"), acc("s2", "w"))), out("s1", "s2"))
    assert merge_equal(body) == body


def test_different_ops_do_not_merge() -> None:
    body = (Loop(A, (load("v"), acc("s1", "v"), acc("s2", "v", "multiply"))), out("s1", "s2"))
    assert merge_equal(body) == body


def test_unseeded_loop_does_not_merge() -> None:
    """Without seeding, each accumulator starts wherever an enclosing loop left it."""
    inner = Loop(A, (load("v"), acc("s1", "v"), acc("s2", "v")), seed=False)
    body = (Loop(Axis("b", Dim(2)), (inner,)), out("s1", "s2"))
    assert accums(merge_equal(body)) == ["s1", "s2"]


def test_update_that_diverges_splits_the_class() -> None:
    """s1 and s2 start equal, but s2 also adds s1's old value: its update differs, so both stay.
    t1 and t2 then fold s1 and s2 respectively, so they differ too."""
    body = (Loop(A, (load("v"), mul("p", "s1", "v"), acc("s1", "v"), acc("s2", "p"),
                     acc("t1", "s1"), acc("t2", "s2"))), out("t1", "t2"))
    assert accums(merge_equal(body)) == ["s1", "s2", "t1", "t2"]


def test_read_between_the_updates_keeps_the_class() -> None:
    """``q`` reads s2 after s1's update and before s2's own, where the two differ by one
    update, and nothing earlier computes the same value: s2 must stay."""
    body = (Loop(A, (load("v"), acc("s1", "v"), mul("q", "s2", "v"), acc("s2", "v"),
                     acc("t", "q"))), out("s1", "s2", "t"))
    assert accums(merge_equal(body)) == ["s1", "s2", "t"]


def test_read_between_the_updates_of_a_repeated_value_merges() -> None:
    """As above, but ``q2`` repeats ``q1``, which read s1 before its update: q2 is dropped, and
    the class merges."""
    body = (Loop(A, (load("v"), mul("q1", "s1", "v"), acc("s1", "v"), mul("q2", "s2", "v"),
                     acc("s2", "v"), acc("t", "q2"))), out("s1", "s2", "t"))
    got = merge_equal(body)
    assert accums(got) == ["s1", "t"]
    assert [s for s in walk(got) if isinstance(s, Accum) and s.name == "t"][0].value == "q1"


def test_loads_of_a_written_buffer_are_not_repeats() -> None:
    body = (Loop(A, (Load(("v1",), "y", (Var("a"),), F32), out("v1"),
                     Load(("v2",), "y", (Var("a"),), F32), acc("s1", "v1"), acc("s2", "v2"))),
            out("s1", "s2"))
    assert merge_equal(body) == body


def test_name_written_twice_is_not_merged() -> None:
    body = (Let("c", Literal(1.0, "float"), F32),
            Loop(A, (load("v"), acc("s1", "v"), acc("s2", "v"))),
            Loop(A, (load("v"), acc("s2", "v"))), out("s1", "s2"))
    assert accums(merge_equal(body)) == ["s1", "s2", "s2"]

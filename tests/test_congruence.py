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


# the two largest attention cases take tens of seconds in the oracle; they are the same nest as
# the shipped a01 at other sizes, so for them only the merge itself is checked here (the GPU
# suite checks their results against the oracle under every flag set)
LARGE = ("a01_256", "a06_long_kv")


@pytest.mark.parametrize("name", sorted(n for n in SUITE if n.startswith("a0")))
def test_suite_attention_merges_bit_equal(name: str) -> None:
    case = SUITE[name]()
    if name in LARGE:
        for op in Graph.from_dict(case.spec.graph).kernel_ops():
            body = jam(op.body.body)
            assert len(accums(merge_equal(body))) < len(accums(body))
        return
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


# --- random loops ----------------------------------------------------------------------------

FUZZ_THREADS, FUZZ_TRIPS = 64, 6


def random_nest(seed: int):
    """A Tile of 64 threads, each running a seeded loop of 6 trips: three loads, then a random
    mix of assignments, accumulations (add, maximum, minimum, multiply; some with a base) and
    repeats of earlier ones under new names, reading loaded values, temporaries and accumulator
    states before and after their updates. After the loop every accumulator is written out (a
    loop body's temporaries are not visible after it)."""
    import random

    from ptxgen.ir import Tile
    from ptxgen.problems import _arg, _spec, add, mul

    rng = random.Random(seed)
    a0, k = Var("a0"), Var("k")
    loop: list = [Load(("xv",), "x", (add(mul(a0, Literal(FUZZ_TRIPS)), k),), F32),
                  Load(("yv",), "y", (add(mul(a0, Literal(FUZZ_TRIPS)), k),), F32),
                  Load(("wv",), "w", (k,), F32)]
    values, accs, temps = ["xv", "yv", "wv"], [], []
    for n in range(rng.randint(8, 18)):
        roll = rng.random()
        if roll < 0.3 and (temps or accs):
            old = rng.choice([s for s in loop if isinstance(s, Assign | Accum)])
            if isinstance(old, Assign):  # a repeat of an earlier assignment
                loop.append(replace(old, name=f"t{n}"))
                temps.append(f"t{n}")
            else:  # a twin of an earlier accumulator
                loop.append(replace(old, name=f"s{n}"))
                accs.append(f"s{n}")
        elif roll < 0.65:
            op = rng.choice(["add", "multiply", "maximum", "subtract", "minimum"])
            args = (rng.choice(values + temps + accs), rng.choice(values + temps + accs))
            loop.append(Assign(f"t{n}", ElementwiseImpl(op), args, F32))
            temps.append(f"t{n}")
        else:
            op = rng.choice(["add", "add", "maximum", "minimum", "multiply"])
            base = rng.choice(values + temps) if op == "add" and rng.random() < 0.3 else None
            loop.append(Accum(f"s{n}", rng.choice(values + temps), ElementwiseImpl(op), F32,
                              ("k",), base))
            accs.append(f"s{n}")
    if not accs:
        loop.append(Accum("s_end", "xv", ElementwiseImpl("add"), F32, ("k",), None))
        accs.append("s_end")
    outs = accs
    body = (Loop(Axis("k", Dim(FUZZ_TRIPS)), tuple(loop)),
            *(Write("out", (add(mul(a0, Literal(len(outs))), Literal(i)),), (name,), F32)
              for i, name in enumerate(outs)))
    tile = Tile((Axis("a0", Dim(FUZZ_THREADS)),), body, None)
    dist = ["uniform", -1.0, 1.0]
    n = FUZZ_THREADS * FUZZ_TRIPS
    args = [_arg("x", "f32", [n], seed=0, dist=dist), _arg("y", "f32", [n], seed=1, dist=dist),
            _arg("w", "f32", [FUZZ_TRIPS], seed=2, dist=dist),
            _arg("out", "f32", [FUZZ_THREADS * len(outs)], output=True)]
    return _spec(f"fuzz{seed}", "random loop", 0, 0, f"k_fuzz{seed}", tile, args,
                 ["x", "y", "w"], ["out"], {}, FUZZ_THREADS)


def test_random_loops_merge_bit_equal() -> None:
    """On 80 random loops the oracle's output is the same bit for bit after the pass, and the
    pass merges something in most of them."""
    merged_any = 0
    for seed in range(80):
        spec = random_nest(seed)
        want, got, body, merged = oracle_both(spec.graph, spec.meta)
        assert np.array_equal(want["out"].view(np.uint8), got["out"].view(np.uint8)), seed
        merged_any += merged != tuple(body)
    assert merged_any >= 40, merged_any


@pytest.mark.gpu
@pytest.mark.parametrize("flag", ["default", "no_unroll"])
def test_random_loops_on_the_gpu(cuda, flag: str) -> None:
    """24 random loops through the whole compiler (merge, lowering, ptxas) on the GPU, each
    against the oracle's run of the original IR, bit for bit: the arithmetic is IEEE-rn adds,
    multiplies (fused into fmas as the oracle models), maxima and minima."""
    from conftest import gpu_run, oracle_run

    for seed in range(24):
        spec = random_nest(seed)
        ins = reference_inputs(spec.meta)
        flags = {} if flag == "default" else {flag: True}
        got = gpu_run(spec.graph, spec.meta, ins, guard=16, **flags)["out"]
        want = oracle_run(spec.graph, spec.meta, ins)["out"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), seed

"""Equal accumulators merged: a loop's accumulators that provably hold the same value on every
trip become one, and the statements that then repeat an earlier one in the same trip go.

Emmy writes a fused softmax-then-matmul nest with one online-softmax state per output element.
The shipped a01 gives each thread 4 query rows and 2 output columns, and for each (row, column)
a running max, a running sum of exponentials and a running output sum. The max and the sum of
exponentials depend on the row only, so every row carries two copies of both, updated by the
same arithmetic from the same values. A common-subexpression pass over straight-line PTX cannot
see that: each copy is a loop-carried register, and its value on one trip depends on its value
on the trip before. So the copies stay, fully unrolled or not: per key step a01 computed 16
exponentials where 8 give the same results.

Method: optimistic value numbering, as in Alpern, Wegman and Zadeck ("Detecting equality of
variables in programs", POPL 1988), over one loop body at a time:

1. Assume that the loop's accumulators of the same op and type hold equal values at the start of
   a trip (a seeding loop starts every one of them at its op's identity).
2. Number every statement of the body in order by its operation and the numbers of its operands.
   An accumulator's state before its update has the number of its class, and after it the number
   of its update. Loads take a number from the input and the index, for inputs the kernel never
   writes. Anything else (nested loops, writes, barriers, shuffles) gives each name it writes a
   number of its own.
3. Split every class whose members' updates got different numbers, and number again, until no
   class splits. What is left holds on every trip by induction: equal at the start of the first
   trip, and equal updates from equal states.

Then, within the body:

* a plain statement (load, assignment, ``Let``, select) whose numbers all equal an earlier plain
  statement's is dropped, and its names are read from the earlier statement's names;
* each class of accumulators keeps the member updated first. The others' updates are dropped,
  and their names are read from the kept member, unless a remaining statement reads a dropped
  member between the kept member's update and its own, where the two differ by one update.
  Such a class stays as it was.

Each statement that is kept performs the same operation on the same values as before, and the
lowering fuses and rounds it the same way (a fusion depends only on the product's definition).
So the results are the same bit for bit. A name is merged or read in place of another only when
exactly one statement of the kernel writes it. The pass is off under ``--no_cse``.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from dataclasses import replace
from typing import Any

from .ir import (Accum, Assign, BinaryExpr, CastExpr, Cond, CpAsyncCopy, FuncCallExpr, Let,
                 Literal, Load, Loop, Select, Smem, Stmt, StridedLoop, TernaryExpr, TreeHalve,
                 Var, WarpShuffle, Write, walk)

_PLAIN = (Load, Assign, Let, Select)


def merge_equal(body: Sequence[Stmt]) -> tuple[Stmt, ...]:
    """A kernel body (the Tile's statements) with every loop's equal accumulators merged and the
    repeated statements dropped; ``body`` itself when nothing merges."""
    stmts = tuple(body)
    writes: dict[str, int] = {}
    for st in walk(stmts):
        for name in _written_here(st):
            writes[name] = writes.get(name, 0) + 1
    ctx = _Context(writes, _mutable(stmts))
    new = ctx.rewrite(stmts)
    if not ctx.renames:
        return stmts
    final = {name: ctx.resolve(name) for name in ctx.renames}
    out = tuple(_rename(st, final) for st in new)
    gone = set(final)
    if any(gone & set(st.deps()) for st in walk(out)):  # a field the renaming missed
        return stmts
    return out


def _written_here(st: Stmt) -> tuple[str, ...]:
    """The names statement ``st`` itself (not its nested bodies) writes."""
    return tuple(st.defines())


def _mutable(stmts: Sequence[Stmt]) -> set[str]:
    """Buffers the kernel writes: loads from them are never numbered alike."""
    out: set[str] = set()
    for st in walk(stmts):
        if isinstance(st, Write):
            out.add(st.output)
        elif isinstance(st, Smem):
            out.add(st.name)
        elif isinstance(st, CpAsyncCopy):
            out.add(st.smem)
        elif isinstance(st, TreeHalve):
            out.update(st.bufs)
    return out


def _all_reads(st: Stmt) -> Iterator[str]:
    yield from st.deps()
    for inner in st.nested():
        for s in walk(inner):
            yield from s.deps()


def _all_writes(st: Stmt) -> Iterator[str]:
    yield from _written_here(st)
    for inner in st.nested():
        for s in walk(inner):
            yield from _written_here(s)


class _Context:
    def __init__(self, writes: dict[str, int], mutable: set[str]):
        self.writes = writes
        self.mutable = mutable
        self.renames: dict[str, str] = {}

    def resolve(self, name: str) -> str:
        while name in self.renames:
            name = self.renames[name]
        return name

    def rewrite(self, stmts: Sequence[Stmt]) -> tuple[Stmt, ...]:
        out = []
        for st in stmts:
            if isinstance(st, Loop | StridedLoop):
                st = self.merge_loop(replace(st, body=self.rewrite(st.body)))
            elif isinstance(st, Cond):
                st = replace(st, body=self.rewrite(st.body),
                             else_body=self.rewrite(st.else_body))
            out.append(st)
        return tuple(out)

    # --- one loop -------------------------------------------------------------------------
    def merge_loop(self, loop: Loop | StridedLoop) -> Loop | StridedLoop:
        body = loop.body
        updates: dict[str, list[int]] = {}
        for i, st in enumerate(body):
            if isinstance(st, Accum):
                updates.setdefault(st.name, []).append(i)
        at = {n: p[0] for n, p in updates.items() if len(p) == 1 and self.writes.get(n) == 1}
        for st in body:  # an accumulator a nested body touches is left alone
            for inner in st.nested():
                for s in walk(inner):
                    for n in (*s.deps(), *_written_here(s)):
                        at.pop(n, None)
        first_write: dict[str, int] = {}
        for i, st in enumerate(body):
            for n in _all_writes(st):
                first_write.setdefault(n, i)
        early = {n for i, st in enumerate(body) for n in _all_reads(st)
                 if n in first_write and i <= first_write[n]}  # read before this trip writes it

        def start_key(n: str) -> Any:
            s = body[at[n]]
            if not loop.seed or s.op.identity is None:
                return ("own", n)  # its start is not known to equal another's
            return (s.op.name, None if s.dtype is None else s.dtype.name)

        keys = {n: start_key(n) for n in at}
        ids: dict[Any, int] = {}
        cls = {n: ids.setdefault(k, len(ids)) for n, k in keys.items()}
        while True:
            numbers, ends = self._number(body, cls, first_write)
            ids = {}
            new = {n: ids.setdefault((cls[n], ends[n]), len(ids)) for n in at}
            if len(set(new.values())) == len(set(cls.values())):
                break
            cls = new

        # repeated plain statements
        drop: set[int] = set()
        first: dict[int, str] = {}
        for i, st in enumerate(body):
            if not isinstance(st, _PLAIN):
                continue
            names = st.defines()
            nums = numbers[i]
            single = all(self.writes.get(n) == 1 for n in names)
            if single and all(n not in early for n in names) and all(v in first for v in nums):
                for n, v in zip(names, nums):
                    self.renames[n] = first[v]
                drop.add(i)
                continue
            if single:
                for n, v in zip(names, nums):
                    first.setdefault(v, n)

        # classes of accumulators
        members: dict[int, list[str]] = {}
        for n in sorted(at, key=at.get):
            members.setdefault(cls[n], []).append(n)
        for group in members.values():
            keep, others = group[0], group[1:]
            if not others:
                continue
            safe = all(m not in set(body[i].deps()) for m in others
                       for i in range(at[keep] + 1, at[m]) if i not in drop)
            if not safe:
                continue
            for m in others:
                self.renames[m] = keep
                drop.add(at[m])
        if not drop:
            return loop
        return replace(loop, body=tuple(st for i, st in enumerate(body) if i not in drop))

    def _number(self, body: Sequence[Stmt], cls: dict[str, int], first_write: dict[str, int]
                ) -> tuple[dict[int, tuple[int, ...]], dict[str, int]]:
        """Numbers of each plain statement's names (by body index), and each merge candidate's
        number at the end of the trip, with the candidates' start states numbered by ``cls``."""
        table: dict[Any, int] = {}

        def num(key: Any) -> int:
            return table.setdefault(key, len(table))

        cur: dict[str, int] = {n: num(("start", c)) for n, c in cls.items()}

        def name(n: str) -> int:
            n = self.resolve(n)
            if n in cur:
                return cur[n]
            if n in first_write:
                return num(("carried", n))
            return num(("outside", n))

        def expr(e: Any) -> int:
            if isinstance(e, Var):
                return name(e.name)
            if isinstance(e, Literal):
                return num(("lit", repr(e.value), e.dtype))
            if isinstance(e, BinaryExpr):
                return num(("bin", e.op, expr(e.left), expr(e.right)))
            if isinstance(e, TernaryExpr):
                return num(("sel", expr(e.cond), expr(e.if_true), expr(e.if_false)))
            if isinstance(e, FuncCallExpr):
                return num(("call", e.name, tuple(expr(a) for a in e.args)))
            if isinstance(e, CastExpr):
                return num(("cast", e.dtype, expr(e.expr)))
            return num(("opaque", id(e)))

        def dtype(d: Any) -> str | None:
            return None if d is None else d.name

        numbers: dict[int, tuple[int, ...]] = {}
        for i, st in enumerate(body):
            if isinstance(st, Assign):
                v = (num(("op", st.op.name, dtype(st.dtype), tuple(name(a) for a in st.args))),)
            elif isinstance(st, Let):
                v = (num(("let", expr(st.value), dtype(st.dtype))),)
            elif isinstance(st, Select):
                v = (num(("select", expr(st.cond), expr(st.if_true), expr(st.if_false))),)
            elif isinstance(st, Load):
                if st.input in self.mutable:
                    v = tuple(num(("written", i, j)) for j in range(len(st.names)))
                else:
                    index = tuple(expr(e) for e in st.index)
                    v = tuple(num(("load", st.input, index, dtype(st.dtype), len(st.names), j))
                              for j in range(len(st.names)))
            elif isinstance(st, Accum) and st.name in cls:
                base = name(st.base) if st.base else cur[st.name]
                cur[st.name] = num(("acc", st.op.name, dtype(st.dtype), base, name(st.value)))
                continue
            else:
                for n in _all_writes(st):
                    cur[n] = num(("own", i, n))
                continue
            numbers[i] = v
            for n, x in zip(st.defines(), v):
                cur[n] = x
        return numbers, {n: cur[n] for n in cls}


# --- renaming reads ------------------------------------------------------------------------


def _rename_expr(e: Any, r: dict[str, str]) -> Any:
    if isinstance(e, Var):
        return Var(r[e.name]) if e.name in r else e
    if isinstance(e, BinaryExpr):
        return replace(e, left=_rename_expr(e.left, r), right=_rename_expr(e.right, r))
    if isinstance(e, TernaryExpr):
        return replace(e, cond=_rename_expr(e.cond, r), if_true=_rename_expr(e.if_true, r),
                       if_false=_rename_expr(e.if_false, r))
    if isinstance(e, FuncCallExpr):
        return replace(e, args=tuple(_rename_expr(a, r) for a in e.args))
    if isinstance(e, CastExpr):
        return replace(e, expr=_rename_expr(e.expr, r))
    if isinstance(e, tuple):
        return tuple(_rename_expr(x, r) for x in e)
    return e


def _rename(st: Stmt, r: dict[str, str]) -> Stmt:
    """``st`` reading ``r[n]`` wherever it read ``n`` (nested bodies included)."""
    def n(x: str) -> str:
        return r.get(x, x)

    def body(b: Sequence[Stmt]) -> tuple[Stmt, ...]:
        return tuple(_rename(s, r) for s in b)

    if isinstance(st, Assign):
        return replace(st, args=tuple(n(a) for a in st.args))
    if isinstance(st, Accum):
        return replace(st, value=n(st.value), base=None if st.base is None else n(st.base))
    if isinstance(st, Load):
        return replace(st, index=_rename_expr(st.index, r))
    if isinstance(st, Write):
        return replace(st, index=_rename_expr(st.index, r), values=tuple(n(v) for v in st.values))
    if isinstance(st, Let):
        return replace(st, value=_rename_expr(st.value, r))
    if isinstance(st, Select):
        return replace(st, cond=_rename_expr(st.cond, r), if_true=_rename_expr(st.if_true, r),
                       if_false=_rename_expr(st.if_false, r))
    if isinstance(st, Cond):
        return replace(st, cond=_rename_expr(st.cond, r), body=body(st.body),
                       else_body=body(st.else_body))
    if isinstance(st, Loop):
        return replace(st, body=body(st.body))
    if isinstance(st, StridedLoop):
        return replace(st, start=_rename_expr(st.start, r), step=_rename_expr(st.step, r),
                       end=_rename_expr(st.end, r), body=body(st.body))
    if isinstance(st, CpAsyncCopy):
        return replace(st, smem_index=_rename_expr(st.smem_index, r),
                       src_index=_rename_expr(st.src_index, r),
                       lane_index=_rename_expr(st.lane_index, r))
    if isinstance(st, WarpShuffle):
        return replace(st, combine_states=tuple(_rename(a, r) for a in st.combine_states))
    if isinstance(st, TreeHalve):
        inner = st.inner if st.inner is None else (n(st.inner[0]), st.inner[1])
        return replace(st, combine_states=tuple(_rename(a, r) for a in st.combine_states),
                       tid_var=n(st.tid_var), inner=inner)
    return st

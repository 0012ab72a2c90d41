"""Work a loop repeats in threads that differ along one axis only, done once and shared.

Emmy's attention nest (the shipped ``a01_attention``: 4 CTAs of 128 threads, ``a0_u`` 8 x ``a5_u``
16) gives each thread 4 query rows and 2 output columns. Per key it computes the 4 rows' scores,
each a 64-term dot product, then runs the online softmax of its rows and columns. The scores
depend on the row and the key only, so the 16 threads along ``a5_u`` that share a row group
compute the same 4 x 64 dot products: 16 times the work, which is most of the kernel (per key a
thread runs 64 x 9 instructions of dot products against about 70 of softmax).

``share_invariant`` rewrites such a loop. It finds an axis X among the block's thread axes that
the loop's leading work does not use, and splits the loop in two:

* first, each thread computes that work for every E-th trip, starting at its own coordinate
  along X (E = X's extent). The statements are the loop's own, unchanged. It writes the values
  the rest of the loop reads into a shared-memory array, indexed by the thread's other
  coordinates and the trip;
* a barrier;
* then the loop runs as before, minus that work, reading those values back from shared memory.

The leading work (``P1``) is the loop's nested plain loops (loads, products and accumulations
only, seeding their own accumulators) that use no thread axis X, together with the assignments
computed from their results alone. None of it may read a value the rest of the loop computes or
the loop's own accumulators, so computing it earlier, in another thread along X, gives the same
values bit for bit, and a round trip through shared memory is exact. Every other statement keeps
its operands and its order.

On the shipped a01 each thread then computes 4 rows x 4 keys of scores in place of 4 rows x 64
keys. The rewrite applies to whole blocks only (the barrier needs every thread), to f32 values,
and where the kernel's shared buffers, the new array included, stay under the static limit
(``lower.STATIC_SMEM_CAP``), so no launch needs dynamic shared memory for it. It is a
template-level change, so a compiler flag turns it off.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from dataclasses import replace

from .ir import (Accum, Assign, BinaryExpr, Literal, Load, Loop, Smem, Stmt, StridedLoop, Sync,
                 Tile, Var, Write, dt, walk)
from .lower import STATIC_SMEM_CAP, pack_shared

F32 = dt("f32")
_PLAIN = (Load, Assign, Accum)


def share_invariant(tile: Tile, block: int) -> Tile:
    """``tile`` with each top-level loop rewritten as the module docstring describes, where
    it applies; ``tile`` itself when none does."""
    if not tile.is_static_grid or tile.aux_threads or tile.n_elements % block:
        return tile
    threads = _thread_axes(tile, block)
    if not threads:
        return tile
    body = list(tile.body)
    # the kernel's shared buffers stay static arrays, so a launcher that passes only meta.json's
    # dynamic shared memory still runs it
    _, used = pack_shared(list({s.name: s for s in walk(body) if isinstance(s, Smem)}.values()))
    out: list[Stmt] = []
    changed = False
    for j, st in enumerate(body):
        split = None
        if isinstance(st, Loop) and st.axis.extent.is_static:
            split = _split(st, threads, body[:j], f"_shared{j}", STATIC_SMEM_CAP - used - 16)
        if split is None:
            out.append(st)
            continue
        decl, first, loop, nbytes = split
        used += nbytes
        out[:0] = [decl]
        out += [first, Sync(), loop]
        changed = True
    return replace(tile, body=tuple(out)) if changed else tile


def _thread_axes(tile: Tile, block: int) -> list[tuple[str, int]]:
    """The Tile's innermost axes whose extents multiply to exactly ``block``: the coordinates
    that tell the threads of one block apart (the rest number the blocks)."""
    out: list[tuple[str, int]] = []
    n = 1
    for ax in reversed(tile.axes):
        if n == block:
            break
        n *= ax.extent.as_static()
        out.insert(0, (ax.name, ax.extent.as_static()))
    return out if n == block else []


def _names_in(e: object) -> set[str]:
    if isinstance(e, Var):
        return {e.name}
    if isinstance(e, tuple):
        return set().union(*(_names_in(x) for x in e)) if e else set()
    deps = getattr(e, "deps", None)
    return set(deps()) if callable(deps) and not isinstance(e, Stmt) else set()


def _reads(st: Stmt) -> set[str]:
    """Names ``st`` reads from outside itself (its nested bodies' own definitions excluded)."""
    inner = set()
    reads = set(st.deps())
    for body in st.nested():
        for s in walk(body):
            reads |= set(s.deps())
            inner |= set(s.defines())
    if isinstance(st, Loop | StridedLoop):
        inner.add(st.axis.name)
    return reads - inner


def _index_names(st: Stmt) -> set[str]:
    """Every name an index expression in ``st`` (nested bodies included) uses."""
    out: set[str] = set()
    for s in walk([st]):
        if isinstance(s, Load | Write):
            out |= _names_in(tuple(s.index))
        if isinstance(s, StridedLoop):
            out |= _names_in((s.start, s.step, s.end))
    return out


def _plain_loop(st: Stmt) -> bool:
    return (isinstance(st, Loop) and st.seed and st.axis.extent.is_static and
            all(isinstance(s, _PLAIN) for s in st.body))


def _split(loop: Loop, threads: list[tuple[str, int]], prefix: Sequence[Stmt], name: str,
           room: int) -> tuple[Smem, StridedLoop, Loop, int] | None:
    body = list(loop.body)
    axis = loop.axis.name
    state = {s.name for s in body if isinstance(s, Accum)}
    body_defs = set()  # every name the loop body writes, at any depth
    for st in walk(body):
        body_defs |= set(st.defines())
    first: list[int] = []
    defined: list[str] = []  # by P1, in order
    for i, st in enumerate(body):
        # P1 reads only names from before the loop, the loop's axis, and earlier P1 results
        reads = _reads(st)
        ok = not (reads & (state | (body_defs - set(defined))))
        if ok and _plain_loop(st):
            first.append(i)
            defined += [s.name for s in st.body if isinstance(s, Accum) and s.name not in defined]
        elif (ok and isinstance(st, Assign) and reads & set(defined) and
              st.dtype is not None and st.dtype.name == "f32"):
            first.append(i)
            defined.append(st.name)
    if not any(isinstance(body[i], Loop) for i in first):
        return None
    p1 = [body[i] for i in first]
    rest = [st for i, st in enumerate(body) if i not in first]
    crossing = [n for n in defined if any(n in _reads(st) for st in rest)]
    if not crossing:
        return None
    for st in p1:  # every crossing value is f32
        for s in walk([st]):
            if isinstance(s, Accum | Assign) and s.name in crossing and \
                    s.dtype is not None and s.dtype.name != "f32":
                return None
    # the thread axes P1 depends on: named in its indices, or through a name defined before the
    # loop from one
    depends: dict[str, set[str]] = {}
    for st in prefix:
        for s in walk([st]):
            for d in s.defines():
                depends[d] = _reads(s) | _index_names(s)
    used = set().union(*(_reads(st) | _index_names(st) for st in p1))
    todo = list(used)
    while todo:
        for m in depends.get(todo.pop(), ()):
            if m not in used:
                used.add(m)
                todo.append(m)
    free = [(n, e) for n, e in threads if n not in used and e > 1]
    if not free:
        return None
    x, extent = max(free, key=lambda t: t[1])
    others = [(n, e) for n, e in threads if n != x]
    rows = math.prod(e for _, e in others) * len(crossing)
    trips = loop.axis.extent.as_static()
    nbytes = rows * trips * 4
    if nbytes > room:
        return None
    # the thread's coordinates other than X, as one index
    w: object = Literal(0)
    stride = 1
    for n, e in reversed(others):
        term = Var(n) if stride == 1 else BinaryExpr("*", Var(n), Literal(stride))
        w = term if isinstance(w, Literal) else BinaryExpr("+", term, w)
        stride *= e

    def at(i: int) -> tuple[object, Var]:
        row = BinaryExpr("+", BinaryExpr("*", w, Literal(len(crossing))), Literal(i))
        return row, Var(axis)

    stores = [Write(name, at(i), (v,), F32) for i, v in enumerate(crossing)]
    loads = [Load((v,), name, at(i), F32) for i, v in enumerate(crossing)]
    decl = Smem(name, (rows, trips), "float", 16)
    head = StridedLoop(replace(loop.axis), Var(x), extent, tuple(p1 + stores), loop.unroll,
                       None, True)
    return decl, head, replace(loop, body=tuple(loads + rest)), nbytes

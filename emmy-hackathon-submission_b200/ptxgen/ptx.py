"""The PTX kernel builder: instructions as objects, virtual registers, scoped value reuse, loop
invariant hoisting, dead-code removal, load/store vectorization and sm_100a rendering.

Instructions are kept as ``Ins`` objects rather than text until ``render``, so two passes can run
over the finished body:

* ``vectorize`` merges scalar loads and stores of one address register whose byte offsets are
  consecutive into 64- and 128-bit accesses (``ld.global.nc.v4.f32``, 16-bit values packed into
  ``.b32`` words), wherever the builder can prove the alignment: every address register carries
  the power of two its value is a multiple of (``align``), from the index algebra's divisibility
  facts and the rule that every kernel buffer starts 16-byte aligned.
* ``drop_dead`` removes side-effect-free results nothing reads (a multiply fused into an fma, a
  load whose value is never used).

Control flow is structured (``region``/``loop``/``skip_if``), so a stack of scopes tells which
cached results dominate the current point. ``pure`` reuses a dominating identical result (unless
CSE is off); inside a runtime loop it moves arithmetic whose inputs predate the loop in front of it.
``forget`` drops cached results that read a register about to be written in place.
"""

from __future__ import annotations

import math
import re
from collections import Counter
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any

from .dtypes import REG_PREFIXES, move_type, reg_class, size

Range = tuple[int, int]
_REG = re.compile(r"%(?:rd|fd|[phrf])\d+")

PTX_VERSION = "8.7"
TARGET = "sm_100a"
SM_COUNT = 148  # B200: SMs one wave of CTAs spreads over
BUFFER_ALIGN = 16  # every kernel buffer pointer is at least this aligned (cudaMalloc gives 256)


@dataclass(eq=False)
class Mem:
    """The structured operand of a load, store or reduction: ``[addr+off]`` over ``regs``."""

    kind: str  # "ld" | "st" | "red"
    space: str  # "global.nc" | "global" | "shared"
    typ: str  # PTX memory type of one element
    addr: str
    off: int
    regs: tuple[str, ...]
    hint: str = ""  # cache qualifier placed after the space, e.g. ".L1::no_allocate"


@dataclass(eq=False)
class Ins:
    """One PTX statement. ``text`` (labels, template lines) renders verbatim."""

    op: str = ""
    dst: tuple[str, ...] = ()
    src: tuple[str, ...] = ()
    pred: str | None = None
    pure: bool = False
    mem: Mem | None = None
    text: str | None = None
    barrier: bool = False  # orders memory: nothing moves across it

    def render(self) -> str:
        if self.text is not None:
            return self.text
        guard = f"@{self.pred} " if self.pred else ""
        if self.mem is not None:
            m = self.mem
            at = f"[{m.addr}+{m.off}]" if m.off else f"[{m.addr}]"
            vec = "" if len(m.regs) == 1 else f".v{len(m.regs)}"
            regs = m.regs[0] if len(m.regs) == 1 else "{" + ", ".join(m.regs) + "}"
            if m.kind == "ld":
                return f"\t{guard}ld.{m.space}{m.hint}{vec}.{m.typ} {regs}, {at};"
            if m.kind == "st":
                return f"\t{guard}st.{m.space}{m.hint}{vec}.{m.typ} {at}, {regs};"
            return f"\t{guard}red.{m.space}.add{vec}.{m.typ} {at}, {regs};"
        ops = ", ".join((*self.dst, *self.src))
        return f"\t{guard}{self.op} {ops};" if ops else f"\t{guard}{self.op};"

    def reads(self) -> Iterator[str]:
        for s in self.src:
            yield from _REG.findall(s)
        if self.pred:
            yield from _REG.findall(self.pred)
        if self.mem is not None:
            yield self.mem.addr
            if self.mem.kind != "ld":
                yield from self.mem.regs
        if self.text is not None and self.mem is None and not self.src and not self.dst:
            yield from _REG.findall(self.text)  # a verbatim line reads what it names

    def writes(self) -> tuple[str, ...]:
        if self.mem is not None and self.mem.kind == "ld":
            return self.mem.regs
        return self.dst


@dataclass
class _LoopMark:
    at: int  # body index in front of the loop, where hoisted instructions go
    born: int  # registers numbered from here on belong to the loop
    home: int  # the scope that keeps hoisted results
    counter: str | None = None  # the loop's counter register, when it steps by a constant
    step: int = 0  # what the latch adds to the counter each trip
    # 64-bit induction pointers: key -> (register, alignment), and what the latch adds to each
    ivs: dict = field(default_factory=dict)
    incs: list = field(default_factory=list)


class Kernel:
    def __init__(self, name: str, params: list[str], max_threads: int, *,
                 no_fusion: bool = False, no_cse: bool = False):
        self.name, self.params, self.max_threads = name, params, max_threads
        self.no_fusion, self.no_cse = no_fusion, no_cse
        self.body: list[Ins] = []
        self.shared_decls: list[str] = []
        self.module_decls: list[str] = []
        self.header_notes: list[str] = []  # "// @ptxgen ..." lines the launcher reads
        self.ranges: dict[str, Range] = {}
        self.mult: dict[str, int] = {}  # u32 register -> a known divisor of its value
        self.align: dict[str, int] = {}  # address register -> power-of-two byte alignment
        self.variables: set[str] = set()
        self.divmods: dict[str, tuple[str, str, int]] = {}
        self.param_align: dict[str, int] = {}  # extra .param alignment (none by default)
        self.extern_shared: tuple[str, int] | None = None
        self.reqntid: int | None = None
        self.min_ctas: int | None = None
        self.pipes: list = []  # runtime loops whose loads the pipeline pass issues ahead
        self.stages: list = []  # counted loops whose warp rows the staging pass fetches wide
        # induction pointer -> (counter coefficient, element bytes, other index terms)
        self.iv_meta: dict[str, tuple[int, int, tuple]] = {}
        self.markers: list[Ins] = []  # placeholder lines the render drops
        self._counts: dict[str, int] = {}
        self._labels = 0
        self._scopes: list[dict[tuple[str, ...], str]] = [{}]
        self._defs: dict[str, tuple[str, ...]] = {}
        self._readers: dict[str, list[tuple[str, ...]]] = {}
        self._born: dict[str, int] = {}
        self._loops: list[_LoopMark] = []
        self._uniq = 0

    # --- registers, labels, raw emission ----------------------------------------------
    def reg(self, typ: str, rng: Range | None = None, mult: int | None = None) -> str:
        prefix = reg_class(typ)[0]
        n = self._counts.get(prefix, 0)
        self._counts[prefix] = n + 1
        r = f"{prefix}{n}"
        self._born[r] = len(self._born)
        if rng is not None:
            self.ranges[r] = rng
        if mult is not None and mult > 1:
            self.mult[r] = mult
        return r

    def variable(self, typ: str, init: str) -> str:
        """A fresh register that is written in place later, starting at ``init``."""
        r = self.reg(typ)
        self.variables.add(r)
        self.emit(f"mov.{move_type(typ)}", (r,), (init,))
        return r

    def label(self, hint: str) -> str:
        self._labels += 1
        return f"$L_{hint}_{self._labels}"

    def place(self, label: str) -> None:
        self.body.append(Ins(text=f"{label}:", barrier=True))

    def emit(self, op: str, dst: tuple[str, ...] = (), src: tuple[str, ...] = (),
             pred: str | None = None, barrier: bool = False) -> Ins:
        ins = Ins(op, tuple(dst), tuple(src), pred, barrier=barrier)
        self.body.append(ins)
        return ins

    def raw(self, line: str, barrier: bool = True) -> None:
        """A verbatim line (template code); it orders memory like a barrier."""
        self.body.append(Ins(text=line if line.startswith(("\t", "$", "//")) else f"\t{line}",
                             barrier=barrier))

    def mem(self, kind: str, space: str, typ: str, addr: str, off: int, regs: tuple[str, ...],
            pred: str | None = None, hint: str = "") -> Ins:
        ins = Ins(pred=pred, mem=Mem(kind, space, typ, addr, off, tuple(regs), hint))
        # A load of memory nothing writes during the kernel has no side effect.
        ins.pure = kind == "ld" and space in ("global.nc",) and pred is None
        self.body.append(ins)
        return ins

    # --- value reuse ------------------------------------------------------------------
    def _cached(self, key: tuple[str, ...]) -> str | None:
        for scope in reversed(self._scopes):
            if key in scope:
                return scope[key]
        return None

    def _remember(self, key: tuple[str, ...], out: str, home: int = -1) -> None:
        self._scopes[home][key] = out
        self._defs[out] = key
        for part in key:
            for src in _REG.findall(part):
                self._readers.setdefault(src, []).append(key)

    def pure(self, op: str, typ: str, *srcs: str, rng: Range | None = None,
             mult: int | None = None) -> str:
        """``op out, *srcs`` for a side-effect-free op, or an identical dominating earlier result
        (never with CSE off). Arithmetic inside a runtime loop whose sources all predate the
        loop is placed in front of it."""
        key: tuple[str, ...] = (op, *srcs)
        if self.no_cse:
            self._uniq += 1
            key = (*key, f"#{self._uniq}")
        if (out := self._cached(key)) is not None:
            return out
        out = self.reg(typ, rng, mult)
        ins = Ins(op, (out,), tuple(srcs), pure=True)
        loop = self._hoist_target(op, srcs)
        if loop is None:
            self.body.append(ins)
            self._remember(key, out)
        else:
            self.body.insert(loop.at, ins)
            loop.at += 1
            self._born[out] = loop.born - 1
            self._remember(key, out, loop.home)
        return out

    def cached_load(self, space: str, typ: str, addr: str, off: int, hint: str = "") -> str:
        """A scalar load of read-only memory, reused like a pure result."""
        key: tuple[str, ...] = (f"ld.{space}.{typ}", f"[{addr}+{off}]")
        if self.no_cse:
            self._uniq += 1
            key = (*key, f"#{self._uniq}")
        if (out := self._cached(key)) is not None:
            return out
        out = self.reg(typ)
        self.mem("ld", space, typ, addr, off, (out,), hint=hint)
        self._remember(key, out)
        return out

    def _hoist_target(self, op: str, srcs: tuple[str, ...]) -> _LoopMark | None:
        if not self._loops or op.startswith(("ld.", "mov.u32 %", "activemask")):
            return None
        loop = self._loops[-1]
        regs = [r for s in srcs for r in _REG.findall(s)]
        if any(r in self.variables or self._born[r] >= loop.born for r in regs):
            return None
        if any(s.startswith("%") and not _REG.fullmatch(s) for s in srcs):
            return None  # special registers (%tid.x, ...) stay where they are
        return loop

    def definition(self, reg: str) -> tuple[str, ...] | None:
        """The key of cached result ``reg`` while it is still reusable at this point."""
        key = self._defs.get(reg)
        if key is None or self._cached(key) != reg:
            return None
        return key

    def forget(self, reg: str) -> None:
        """``reg`` is being written in place: no cached result that read it stays reusable."""
        for key in self._readers.pop(reg, []):
            for scope in self._scopes:
                if (out := scope.pop(key, None)) is not None:
                    self._defs.pop(out, None)

    @contextmanager
    def region(self) -> Iterator[None]:
        """A block dominated by the current one that does not dominate what follows."""
        self._scopes.append({})
        try:
            yield
        finally:
            for out in self._scopes.pop().values():
                self._defs.pop(out, None)

    @contextmanager
    def loop(self, entered: bool, counter: str | None = None, step: int = 0
             ) -> Iterator[_LoopMark]:
        """The body of a runtime loop. ``entered``: every thread runs at least one trip, so code
        in front of the loop dominates what follows it and hoisted results stay reusable.
        ``counter``/``step``: the counter register and its constant step, which lets addresses
        become induction pointers (``induction``); the caller adds each ``incs`` entry to its
        pointer at the latch."""
        home = len(self._scopes) - 1 if entered else len(self._scopes)
        mark = _LoopMark(len(self.body), len(self._born), home, counter, step)
        self._loops.append(mark)
        try:
            with self.region():
                yield mark
        finally:
            self._loops.pop()

    def induction(self, ptr: str, var: Any, esz: int, align: int) -> str | None:
        """A 64-bit pointer register holding ``ptr + var * esz`` on every trip of the innermost
        runtime loop, for ``var`` (an index ``Aff``) = ``coef * counter + sum(c_r * r)`` with
        ``coef`` and every ``c_r`` positive and every ``r`` older than the loop or an enclosing
        loop's counter. It is set in front of the loop, where the counter holds its start, by
        the same u32 arithmetic and ``mul.wide`` the per-trip address would use, and the latch
        adds ``coef * step * esz`` to it. None when ``var`` is not of that form (or with CSE
        off, where every address is computed again)."""
        if self.no_cse or not self._loops:
            return None
        loop = self._loops[-1]
        if loop.counter is None or loop.step <= 0 or var.const:
            return None
        coef = var.terms.get(loop.counter, 0)
        rest = {r: c for r, c in var.terms.items() if r != loop.counter}
        outer = {m.counter for m in self._loops[:-1] if m.counter is not None}
        if coef <= 0 or any(c <= 0 for c in rest.values()):
            return None
        if any(r not in outer and (r in self.variables or self._born[r] >= loop.born)
               for r in rest):
            return None
        key = (ptr, coef, esz, tuple(sorted(rest.items())))
        if key in loop.ivs:
            return loop.ivs[key]
        t = self.reg("u32")
        pre = [Ins("mul.lo.u32", (t,), (loop.counter, str(coef)))]
        for r, c in sorted(rest.items()):
            t2 = self.reg("u32")
            pre.append(Ins("mad.lo.u32", (t2,), (r, str(c), t)))
            t = t2
        w, p = self.reg("u64"), self.reg("u64")
        pre += [Ins("mul.wide.u32", (w,), (t, str(esz))), Ins("add.s64", (p,), (ptr, w))]
        self.body[loop.at:loop.at] = pre
        loop.at += len(pre)
        self.variables.add(p)
        self.align[p] = align
        loop.ivs[key] = p
        loop.incs.append((p, coef * loop.step * esz))
        self.iv_meta[p] = (coef, esz, tuple(sorted(rest.items())))
        return p

    @contextmanager
    def skip_if(self, pred: str) -> Iterator[None]:
        """A block skipped where ``pred`` holds (``pred`` may be negated, ``!%p1``)."""
        skip = self.label("skip")
        self.emit("bra", src=(skip,), pred=pred, barrier=True)
        with self.region():
            yield
        self.place(skip)

    # --- passes -----------------------------------------------------------------------
    def drop_dead(self) -> None:
        """Remove side-effect-free instructions whose results nothing reads, to a fixpoint."""
        while True:
            reads = Counter(r for ins in self.body for r in ins.reads())
            live = []
            for ins in self.body:
                outs = ins.writes()
                if ins.pure and outs and not any(reads[r] for r in outs):
                    continue
                live.append(ins)
            if len(live) == len(self.body):
                return
            self.body = live

    def vectorize(self) -> None:
        """Merge scalar loads/stores at consecutive offsets of one address register into
        aligned 64/128-bit accesses."""
        self.body = _Vectorizer(self).run(self.body)

    # --- rendering --------------------------------------------------------------------
    def render(self) -> str:
        from .slp import SLP

        from .pipeline import pipeline_loads
        from .stage import stage_loads

        self.drop_dead()
        self.vectorize()
        self.drop_dead()
        pipeline_loads(self, self.pipes)
        stage_loads(self, self.stages)
        drop = {id(m) for m in self.markers}
        self.body = [ins for ins in self.body if id(ins) not in drop]
        if not self.no_cse:  # pairing reuses values across copies, as CSE does
            self.body = SLP(self).run(self.body)
            self.drop_dead()
        params = ",\n".join(f"\t.param .u64 {self.name}_param_{p}" for p in self.params)
        decls = []
        classes = {reg_class(t) for t in ("pred", "b16", "b32", "b64", "f32", "f64")}
        for prefix, typ in sorted(classes, key=lambda c: REG_PREFIXES.index(c[0])):
            if prefix in self._counts:
                decls.append(f"\t.reg .{typ} {prefix}<{self._counts[prefix]}>;")
        perf = f".maxntid {self.max_threads}, 1, 1"
        if self.reqntid:
            perf = f".reqntid {self.reqntid}, 1, 1"
        if self.min_ctas:
            perf += f"\n.minnctapersm {self.min_ctas}"
        lines = [
            "//\n// Generated by ptxgen (B200 backend)\n//",
            *self.header_notes,
            "",
            f".version {PTX_VERSION}\n.target {TARGET}\n.address_size 64\n",
            *self.module_decls,
            f".visible .entry {self.name}(\n{params}\n)\n{perf}\n{{",
            *decls,
            *self.shared_decls,
            "",
            *(ins.render() for ins in self.body),
            "\tret;\n}\n",
        ]
        return "\n".join(lines)


def pow2_part(n: int) -> int:
    """The largest power of two dividing ``n`` (a large value for 0)."""
    return 1 << 30 if n == 0 else n & -n


class _Vectorizer:
    """Finds groups of scalar accesses ``[addr+off]`` in straight-line code and merges each
    aligned run of 2 or 4 (8 for 16-bit values, through .b32 words) into one access."""

    def __init__(self, k: Kernel):
        self.k = k

    def run(self, body: list[Ins]) -> list[Ins]:
        out: list[Ins] = []
        seg: list[Ins] = []
        for ins in body:
            if ins.barrier or (ins.op.startswith(("bra", "bar", "membar", "fence", "cp.async",
                                                   "mbarrier", "tcgen05", "exit", "ret"))):
                out += self._segment(seg)
                seg = []
                out.append(ins)
            else:
                seg.append(ins)
        out += self._segment(seg)
        return out

    def _segment(self, seg: list[Ins]) -> list[Ins]:
        if len(seg) < 2:
            return seg
        # bf16 registers that are a plain rounding of an f32 register, for cvt.rn.bf16x2.f32
        self.bf16_sources = {ins.dst[0]: ins.src[0] for ins in seg
                             if ins.op == "cvt.rn.bf16.f32" and len(ins.dst) == 1}
        seg = self._loads(seg)
        seg = self._stores(seg)
        return seg

    def _width_ok(self, addr: str, off: int, nbytes: int) -> bool:
        return (self.k.align.get(addr, 1) % nbytes == 0) and off % nbytes == 0

    def _plan(self, items: list[tuple[int, int]], esize: int, addr: str) -> list[list[int]]:
        """Chunks (lists of item indices) of consecutive offsets, each an aligned vector."""
        by_off = {}
        for idx, (off, _) in enumerate(items):
            by_off.setdefault(off, idx)
        offs = sorted(by_off)
        chunks, used = [], set()
        widths = (8, 4, 2) if esize == 2 else (4, 2)
        for off in offs:
            if by_off[off] in used:
                continue
            for w in widths:
                if w * esize > 16:
                    continue
                run = [off + i * esize for i in range(w)]
                if all(o in by_off and by_off[o] not in used for o in run) and \
                        self._width_ok(addr, off, w * esize):
                    chunk = [by_off[o] for o in run]
                    chunks.append(chunk)
                    used.update(chunk)
                    break
        return chunks

    def _loads(self, seg: list[Ins]) -> list[Ins]:
        """Read-only global loads merge anywhere in the segment. Shared loads merge within a
        stretch that no shared store, reduction or opaque line splits (segments already end at
        every barrier, ``cp.async`` and fence), so a merged load, issued at its first member's
        place, reads what each member would have read."""
        groups: dict[tuple[str, str, str, str, int], list[int]] = {}
        epoch = 0
        for i, ins in enumerate(seg):
            m = ins.mem
            if (m is not None and m.kind != "ld" and m.space == "shared") or \
                    (ins.text is not None and not ins.pure):
                epoch += 1
            if m is None or m.kind != "ld" or len(m.regs) != 1 or ins.pred or m.typ == "u8":
                continue
            if m.space not in ("global.nc", "shared"):
                continue  # loads of global memory the kernel writes keep their order
            groups.setdefault((m.space, m.typ, m.addr, m.hint,
                               epoch if m.space == "shared" else 0), []).append(i)
        replace: dict[int, list[Ins]] = {}
        drop: set[int] = set()
        for (space, typ, addr, hint, _), idxs in groups.items():
            if len(idxs) < 2:
                continue
            esize = size(typ)
            items = [(seg[i].mem.off, i) for i in idxs]  # type: ignore[union-attr]
            for chunk in self._plan(items, esize, addr):
                members = [idxs[c] for c in chunk]
                first = min(members)
                regs = tuple(seg[i].mem.regs[0] for i in members)  # type: ignore[union-attr]
                off = seg[members[0]].mem.off  # type: ignore[union-attr]
                new = self._vector_load(space, typ, addr, off, regs, hint)
                replace.setdefault(first, []).extend(new)
                drop.update(members)
        if not replace:
            return seg
        out = []
        for i, ins in enumerate(seg):
            if i in replace:
                out.extend(replace[i])
            if i not in drop:
                out.append(ins)
        return out

    def _vector_load(self, space: str, typ: str, addr: str, off: int, regs: tuple[str, ...],
                     hint: str) -> list[Ins]:
        k = self.k
        if size(typ) == 2 and len(regs) >= 2:
            words = tuple(k.reg("b32") for _ in range(len(regs) // 2))
            ins = [Ins(mem=Mem("ld", space, "b32", addr, off, words, hint), pure=True)]
            for j, w in enumerate(words):
                ins.append(Ins(text=f"\tmov.b32 {{{regs[2 * j]}, {regs[2 * j + 1]}}}, {w};",
                               pure=True))
                ins[-1].dst = (regs[2 * j], regs[2 * j + 1])
                ins[-1].src = (w,)
            return ins
        return [Ins(mem=Mem("ld", space, typ, addr, off, regs, hint), pure=True)]

    def _stores(self, seg: list[Ins]) -> list[Ins]:
        groups: dict[tuple[str, str, str, str], list[int]] = {}
        for i, ins in enumerate(seg):
            m = ins.mem
            if m is None or m.kind not in ("st", "red") or len(m.regs) != 1 or ins.pred:
                continue
            if m.typ == "u8" or (m.kind == "red" and m.typ != "f32"):
                continue
            groups.setdefault((m.kind + "|" + m.space, m.typ, m.addr, m.hint), []).append(i)
        replace: dict[int, list[Ins]] = {}
        drop: set[int] = set()
        for (kind_space, typ, addr, hint), idxs in groups.items():
            if len(idxs) < 2:
                continue
            kind, space = kind_space.split("|")
            esize = size(typ)
            items = [(seg[i].mem.off, i) for i in idxs]  # type: ignore[union-attr]
            for chunk in self._plan(items, esize, addr):
                members = [idxs[c] for c in chunk]
                last = max(members)
                if not self._store_can_sink(seg, members, last, space):
                    continue
                regs = tuple(seg[i].mem.regs[0] for i in members)  # type: ignore[union-attr]
                off = seg[members[0]].mem.off  # type: ignore[union-attr]
                replace.setdefault(last, []).extend(
                    self._vector_store(kind, space, typ, addr, off, regs, hint))
                drop.update(members)
        if not replace:
            return seg
        out = []
        for i, ins in enumerate(seg):
            if i not in drop:
                out.append(ins)
            if i in replace:
                out.extend(replace[i])
        return out

    @staticmethod
    def _store_can_sink(seg: list[Ins], members: list[int], last: int, space: str) -> bool:
        """Stores move down to ``last``: nothing between may read that memory, and no register
        a moved store writes out may be rewritten after that store's own position."""
        member_set = set(members)
        first = min(members)
        for j in range(first, last):
            if j in member_set:
                continue
            ins = seg[j]
            m = ins.mem
            if m is not None and m.kind == "ld" and m.space == space:
                return False
            if ins.text is not None and ins.mem is None and ins.dst == ():
                return False
            written = set(ins.writes())
            if written and any(p < j and seg[p].mem.regs[0] in written  # type: ignore[union-attr]
                               for p in members):
                return False
        return True

    def _vector_store(self, kind: str, space: str, typ: str, addr: str, off: int,
                      regs: tuple[str, ...], hint: str) -> list[Ins]:
        k = self.k
        if size(typ) == 2 and len(regs) >= 2 and kind == "st":
            out, words = [], []
            for j in range(len(regs) // 2):
                w = k.reg("b32")
                words.append(w)
                lo, hi = self.bf16_sources.get(regs[2 * j]), self.bf16_sources.get(regs[2 * j + 1])
                if lo is not None and hi is not None:
                    # two f32 -> bf16 roundings packed by one instruction (upper half first)
                    ins = Ins("cvt.rn.bf16x2.f32", (w,), (hi, lo), pure=True)
                else:
                    ins = Ins(text=f"\tmov.b32 {w}, {{{regs[2 * j]}, {regs[2 * j + 1]}}};")
                    ins.dst, ins.src = (w,), (regs[2 * j], regs[2 * j + 1])
                out.append(ins)
            out.append(Ins(mem=Mem(kind, space, "b32", addr, off, tuple(words), hint)))
            return out
        return [Ins(mem=Mem(kind, space, typ, addr, off, regs, hint))]


def gcd_all(*xs: int) -> int:
    g = 0
    for x in xs:
        g = math.gcd(g, x)
    return g

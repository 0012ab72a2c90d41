"""Pairing of scalar f32 arithmetic into sm_100's packed ``f32x2`` instructions.

sm_100 issues ``add/sub/mul/fma.rn.f32x2`` on 64-bit register pairs: two IEEE round-to-nearest
f32 operations per instruction, each lane rounding exactly as the scalar instruction would. An
unrolled pointwise body is many copies of one instruction chain, and a kernel such as the bf16
gelu chain is bound by how many instructions the SM can issue, so pairing the copies halves its
arithmetic instructions without changing a single bit of the results.

The pass works on one straight-line segment at a time:

1. **Seeds** are register pairs that are consumed together: the two f32 sources of a
   ``cvt.rn.bf16x2.f32`` and the neighbouring registers of a vector store of f32. An add or
   sub that reads a multiply's result is never packed: ptxas may contract a packed multiply
   and add into an fma (the packed forms' mandatory ``.rn`` does not forbid it the way the
   scalar forms' explicit ``.rn`` does), which would break the results' bit-reproducibility.
2. **Trees** grow bottom-up from a seed: two results defined by pure instructions of one
   packable opcode, neither depending on the other and neither already paired, become a pair
   node, and their operands in the same position are paired recursively. An operand shared by
   both lanes becomes a broadcast ``{x, x}``; anything else becomes a pack leaf. A tree of fewer
   than two pair nodes is not worth its pack and unpack moves and is dropped.
3. **Scheduling.** The segment's dependence graph is contracted (each pair one node) and listed
   again in topological order, earliest original position first. Instructions with side effects
   keep their relative order, and an in-place register write stays between the reads around it.
   A pair's result is unpacked right after it when another instruction still reads a lane.
"""

from __future__ import annotations

import heapq
import re
import struct

from .ptx import Ins

PACKABLE = {"add.rn.f32": "add.rn.f32x2", "sub.rn.f32": "sub.rn.f32x2",
            "mul.rn.f32": "mul.rn.f32x2", "fma.rn.f32": "fma.rn.f32x2"}
_REG = re.compile(r"%(?:rd|fd|[phrf])\d+")
_F32_IMM = re.compile(r"^0f([0-9A-Fa-f]{8})$")
MIN_TREE = 2


def _is_reg(s: str) -> bool:
    return bool(_REG.fullmatch(s))


class _Pair:
    __slots__ = ("a", "b", "ops", "out", "opc")

    def __init__(self, a: Ins, b: Ins):
        self.a, self.b = a, b
        self.opc = PACKABLE[a.op]
        self.ops: list[tuple[str, object]] = []  # ("pair", _Pair) | ("bcast", x) | ("leaf", (x, y))
        self.out = ""


class SLP:
    def __init__(self, kernel: object):
        self.k = kernel

    def run(self, body: list[Ins]) -> list[Ins]:
        from collections import Counter

        # reads of every register anywhere in the kernel: a lane read by anything but its
        # parent pair must be unpacked, even when the reader sits in a later segment
        self.global_reads = Counter(r for ins in body for r in ins.reads())
        self.products = {r for ins in body if ins.op == "mul.rn.f32" for r in ins.writes()}
        out: list[Ins] = []
        seg: list[Ins] = []
        for ins in body:
            if ins.barrier or ins.op.startswith(("bra", "bar", "membar", "fence", "cp.async",
                                                 "mbarrier", "tcgen05", "exit", "ret")) or (
                    ins.text is not None and ins.mem is None and not ins.dst):
                out += self._segment(seg)
                seg = []
                out.append(ins)
            else:
                seg.append(ins)
        out += self._segment(seg)
        return out

    # --- one segment ------------------------------------------------------------------
    def _segment(self, seg: list[Ins]) -> list[Ins]:
        if len(seg) < 4 or not any(i.op in PACKABLE for i in seg):
            return seg
        self.seg = seg
        self.pos = {id(i): n for n, i in enumerate(seg)}
        self.defs: dict[str, Ins] = {}
        for ins in seg:
            for r in ins.writes():
                if _is_reg(r):
                    self.defs[r] = ins
        self.users: dict[str, list[Ins]] = {}
        for ins in seg:
            for r in set(ins.reads()):
                self.users.setdefault(r, []).append(ins)
        self.variables = self.k.variables  # type: ignore[attr-defined]
        self.paired: dict[int, _Pair] = {}
        self.seen_scalar: set[int] = set()
        self._preds_cache: dict[int, set[int]] = {}
        roots: list[_Pair] = []
        for lo, hi in self._seeds():
            trial: dict[int, _Pair] = {}
            root = self._build(lo, hi, trial)
            if root is None:
                continue
            if len({id(p) for p in trial.values()}) < MIN_TREE:
                continue
            self.paired.update(trial)
            roots.append(root)
        if not self.paired:
            return seg
        sched = self._schedule()
        if sched is None:
            return seg
        return sched

    def _seeds(self) -> list[tuple[str, str]]:
        out = []
        for ins in self.seg:
            if ins.op == "cvt.rn.bf16x2.f32" and len(ins.src) == 2:
                hi, lo = ins.src
                out.append((lo, hi))
            m = ins.mem
            if m is not None and m.kind in ("st", "red") and m.typ == "f32" and len(m.regs) >= 2:
                for j in range(0, len(m.regs) - 1, 2):
                    out.append((m.regs[j], m.regs[j + 1]))
        return out

    def _packable(self, a: Ins | None, b: Ins | None) -> bool:
        return (a is not None and b is not None and a is not b and a.op in PACKABLE and
                a.op == b.op and a.pure and b.pure and not a.pred and not b.pred and
                len(a.src) == len(b.src) and len(a.dst) == 1 and len(b.dst) == 1 and
                a.dst[0] not in self.variables and b.dst[0] not in self.variables and
                not self._contractible(a) and not self._contractible(b))

    def _contractible(self, ins: Ins) -> bool:
        """An add or sub of a product. Its scalar ``.rn`` form keeps ptxas from fusing the two
        into an fma, but the packed forms' rounding modifier is mandatory and does not: a packed
        ``mul`` + ``add`` pair came out fused on a B200. So such an add or sub stays scalar, and
        the only fma contractions left are the lowering's own."""
        return ins.op in ("add.rn.f32", "sub.rn.f32") and any(
            r in self.products for r in ins.src)

    def _preds(self, ins: Ins) -> set[int]:
        """Ids of the segment instructions ``ins`` depends on through registers."""
        key = id(ins)
        if key in self._preds_cache:
            return self._preds_cache[key]
        acc: set[int] = set()
        stack = [ins]
        while stack:
            cur = stack.pop()
            for r in cur.reads():
                d = self.defs.get(r)
                if d is not None and id(d) not in acc and self.pos[id(d)] < self.pos[id(cur)]:
                    acc.add(id(d))
                    stack.append(d)
        self._preds_cache[key] = acc
        return acc

    def _isomorphic(self, a: Ins | None, b: Ins | None) -> bool:
        """Two pure single-result instructions of one opcode with no packed form (ex2, rcp,
        abs, ...): they stay scalar, but pairing continues through their operands."""
        return (a is not None and b is not None and a is not b and a.op == b.op and a.op and
                a.op not in PACKABLE and a.pure and b.pure and a.mem is None and
                b.mem is None and a.text is None and b.text is None and not a.pred and
                not b.pred and len(a.src) == len(b.src) and len(a.dst) == 1 and
                len(b.dst) == 1)

    def _build(self, x: str, y: str, trial: dict[int, _Pair]) -> _Pair | None:
        a, b = self.defs.get(x), self.defs.get(y)
        if self._isomorphic(a, b) and id(a) not in self.seen_scalar:
            assert a is not None and b is not None
            self.seen_scalar.add(id(a))
            if id(a) not in self._preds(b) and id(b) not in self._preds(a):
                for sa, sb in zip(a.src, b.src, strict=True):
                    if sa != sb and _is_reg(sa) and _is_reg(sb):
                        self._build(sa, sb, trial)
            return None
        if not self._packable(a, b):
            return None
        assert a is not None and b is not None
        for i in (a, b):
            if id(i) in self.paired or id(i) in trial:
                prev = self.paired.get(id(i)) or trial.get(id(i))
                if prev is not None and prev.a is a and prev.b is b:
                    return prev
                return None
        if id(a) in self._preds(b) or id(b) in self._preds(a):
            return None
        node = _Pair(a, b)
        trial[id(a)] = trial[id(b)] = node
        for sa, sb in zip(a.src, b.src, strict=True):
            if sa == sb:
                node.ops.append(("bcast", sa))
                continue
            child = self._build(sa, sb, trial) if _is_reg(sa) and _is_reg(sb) else None
            node.ops.append(("pair", child) if child is not None else ("leaf", (sa, sb)))
        return node

    # --- contraction and list scheduling -------------------------------------------------
    def _schedule(self) -> list[Ins] | None:
        seg = self.seg
        nodes: list[object] = []  # Ins or _Pair
        node_of: dict[int, int] = {}
        for ins in seg:
            p = self.paired.get(id(ins))
            if p is None:
                node_of[id(ins)] = len(nodes)
                nodes.append(ins)
            elif id(p) not in node_of:
                node_of[id(p)] = len(nodes)
                nodes.append(p)
                node_of[id(p.a)] = node_of[id(p.b)] = node_of[id(p)]
            else:
                node_of[id(ins)] = node_of[id(p)]
        n = len(nodes)
        edges: list[set[int]] = [set() for _ in range(n)]
        indeg = [0] * n

        def add_edge(u: int, v: int) -> None:
            if u != v and v not in edges[u]:
                edges[u].add(v)
                indeg[v] += 1

        last_side: int | None = None
        last_write: dict[str, int] = {}
        reads_since: dict[str, list[int]] = {}
        for ins in seg:
            v = node_of[id(ins)]
            for r in ins.reads():
                d = self.defs.get(r)
                if d is not None and self.pos[id(d)] < self.pos[id(ins)]:
                    add_edge(node_of[id(d)], v)
                if r in self.variables:
                    if r in last_write:
                        add_edge(last_write[r], v)
                    reads_since.setdefault(r, []).append(v)
            if not ins.pure:
                if last_side is not None:
                    add_edge(last_side, v)
                last_side = v
            for r in ins.writes():
                if r in self.variables:
                    for u in reads_since.pop(r, []):
                        add_edge(u, v)
                    if r in last_write:
                        add_edge(last_write[r], v)
                    last_write[r] = v
        prio = [min(self.pos[id(x.a)], self.pos[id(x.b)]) if isinstance(x, _Pair) else
                self.pos[id(x)] for x in nodes]
        for i, x in enumerate(nodes):
            if isinstance(x, _Pair):
                prio[i] = max(self.pos[id(x.a)], self.pos[id(x.b)])
        heap = [(prio[i], i) for i in range(n) if indeg[i] == 0]
        heapq.heapify(heap)
        order: list[int] = []
        while heap:
            _, u = heapq.heappop(heap)
            order.append(u)
            for v in edges[u]:
                indeg[v] -= 1
                if indeg[v] == 0:
                    heapq.heappush(heap, (prio[v], v))
        if len(order) != n:
            return None  # the contraction made a cycle: keep the segment as it was
        out: list[Ins] = []
        bcast: dict[str, str] = {}
        for u in order:
            x = nodes[u]
            if isinstance(x, _Pair):
                out += self._emit_pair(x, bcast)
            else:
                out.append(x)
        return out

    def _pack_regs(self, lo: str, hi: str, out: list[Ins]) -> str:
        k = self.k
        w = k.reg("b64")  # type: ignore[attr-defined]
        srcs = []
        for s in (lo, hi):
            if _is_reg(s):
                srcs.append(s)
            else:
                t = k.reg("f32")  # type: ignore[attr-defined]
                out.append(Ins("mov.f32", (t,), (s,), pure=True))
                srcs.append(t)
        ins = Ins(text=f"\tmov.b64 {w}, {{{srcs[0]}, {srcs[1]}}};", pure=True)
        ins.dst, ins.src = (w,), tuple(srcs)
        out.append(ins)
        return w

    def _emit_pair(self, p: _Pair, bcast: dict[str, str]) -> list[Ins]:
        out: list[Ins] = []
        k = self.k
        srcs = []
        for kind, val in p.ops:
            if kind == "pair":
                srcs.append(val.out)  # type: ignore[union-attr]
            elif kind == "bcast":
                x = str(val)
                if x not in bcast:
                    m = _F32_IMM.match(x)
                    if m:
                        w = k.reg("b64")  # type: ignore[attr-defined]
                        out.append(Ins("mov.b64", (w,), (f"0x{m.group(1) * 2}",), pure=True))
                        bcast[x] = w
                    else:
                        bcast[x] = self._pack_regs(x, x, out)
                srcs.append(bcast[x])
            else:
                lo, hi = val  # type: ignore[misc]
                srcs.append(self._pack_regs(lo, hi, out))
        p.out = k.reg("b64")  # type: ignore[attr-defined]
        out.append(Ins(p.opc, (p.out,), tuple(srcs), pure=True))
        # unpack when a lane is still read by anything but the pairs consuming this one
        lanes = (p.a.dst[0], p.b.dst[0])
        consumed = sum(1 for q in {id(v): v for v in self.paired.values()}.values()
                       for kind, val in q.ops if kind == "pair" and val is p)
        if any(self.global_reads[r] > consumed for r in lanes):
            ins = Ins(text=f"\tmov.b64 {{{lanes[0]}, {lanes[1]}}}, {p.out};", pure=True)
            ins.dst, ins.src = lanes, (p.out,)
            out.append(ins)
        return out


def f32_bits_imm(value: float) -> str:
    return f"0f{struct.unpack('<I', struct.pack('<f', value))[0]:08X}"

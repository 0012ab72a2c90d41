"""Rows a warp reads one 4-byte element a lane at a time, fetched 8 bytes a lane through shared
memory.

Emmy writes a grid-stride reduction (config 4's sum, the shipped r02) with one element per thread
per stride. A trip of its counted loop issues 16 scalar loads a thread, and for each of them a
warp reads one contiguous 128-byte row. On a B200 a stream of 4-byte loads reads 2^30 f32 at
6.1-6.2 TB/s, where 8- and 16-byte loads of the same addresses reach 7.0 (702 against 614 us).
The IR's order of additions fixes which thread adds which element, so a wider load has to hand
each lane its own element back:

* the lanes load the trip's rows 8 bytes each: load q brings row 2q to lanes 0-15 and row 2q+1
  to lanes 16-31;
* each lane stores its 8 bytes to a warp-private shared area (row r at r * 128 bytes), and the
  warp syncs (``bar.warp.sync``);
* each of the trip's original loads becomes a 4-byte shared load of the lane's own element of its
  row, in place, so the additions run as before;
* the warp syncs again at the end of the trip, before the next trip's stores.

The warp reads exactly the addresses its lanes read before, and every lane gets the same values
in the same order, so results are the same bit for bit.

The lowering records a counted loop (``Stage``) only where every thread of the block runs every
trip together (no partial block, no enclosing condition), with the induction pointers through
which a warp's lanes read consecutive 4-byte elements from a 32-element-aligned start. The pass
takes the pointer with the most plain ``ld.global.nc`` 4-byte loads in the trip, when they are an
even number from ``MIN_ROWS`` to ``MAX_ROWS``, at offsets ``o + j * S`` (``S`` and ``o`` multiples
of 8), in a body without branches, and when the block's shared memory stays static.
"""

from __future__ import annotations

from dataclasses import dataclass

MIN_ROWS = 4
# at most this many rows a trip: the areas of the 2048 threads an SM can hold then take
# MAX_ROWS * 8 KiB (128 KiB), whatever the block size, so residency is unchanged
MAX_ROWS = 16
STATIC_LIMIT = 48 << 10  # a block's static shared memory
ROW = 128  # bytes of one warp row: 32 lanes x 4 bytes


@dataclass(eq=False)
class Stage:
    """A counted loop as the lowering left it: the marker where its preheader ends, its top
    label, its latch branch, and the lane-contiguous induction pointers with their per-trip
    steps in bytes."""

    pre: object
    top: object
    latch: object
    rows: dict[str, int]


def _static_smem(k) -> int:
    import re

    return sum(int(m.group(1)) for d in k.shared_decls for m in [re.search(r"\[(\d+)\]", d)]
               if m)


def stage_loads(k, stages: list[Stage]) -> None:
    """Rewrite each recorded loop of kernel ``k`` in place (see the module docstring)."""
    from .ptx import Ins, Mem

    for n, st in enumerate(stages):
        body = k.body
        try:
            pre, top, latch = (next(i for i, ins in enumerate(body) if ins is want)
                               for want in (st.pre, st.top, st.latch))
        except StopIteration:  # a pass removed the loop
            continue
        if not pre < top < latch:
            continue
        inner = body[top + 1:latch]
        if any(ins.op.startswith("bra") or ins.barrier or
               (ins.text is not None and ins.text.strip()) for ins in inner):
            continue  # not one straight-line trip
        best: list[int] = []
        for ptr in st.rows:
            loads = [i for i in range(top + 1, latch)
                     if (m := body[i].mem) is not None and m.kind == "ld" and
                     m.space == "global.nc" and not m.hint and m.addr == ptr and
                     len(m.regs) == 1 and m.typ in ("f32", "b32", "u32", "s32") and
                     not body[i].pred]
            if len(loads) > len(best):
                best = loads
        rows = len(best)
        if rows < MIN_ROWS or rows > MAX_ROWS or rows % 2:
            continue
        ptr = body[best[0]].mem.addr
        offs = sorted(body[i].mem.off for i in best)
        stride = offs[1] - offs[0]
        if (stride <= 0 or stride % 8 or offs[0] % 8 or stride >= 1 << 31 or
                offs != [offs[0] + j * stride for j in range(rows)]):
            continue
        warps = k.max_threads // 32
        size = rows * ROW * warps
        if _static_smem(k) + size > STATIC_LIMIT:
            continue
        sym = f"{k.name}_rows{n}"
        k.shared_decls.append(f"\t.shared .align 16 .b8 {sym}[{size}];")

        def r(typ: str) -> str:
            return k.reg(typ)

        tid, lane, warp, base = r("u32"), r("u32"), r("u32"), r("u32")
        put, get = r("u32"), r("u32")
        t1, t2, t3 = r("u32"), r("u32"), r("u32")
        d64, q = r("u64"), r("u64")
        # the lane's first 8 bytes: the warp's row 0 (this pointer less lane * 4 bytes), plus
        # row 1 for lanes 16-31, plus 8 bytes per lane within the row
        prologue = [
            Ins("mov.u32", (tid,), ("%tid.x",)),
            Ins("and.b32", (lane,), (tid, "31")),
            Ins("shr.u32", (warp,), (tid, "5")),
            Ins("mov.u32", (base,), (sym,)),
            Ins("mad.lo.u32", (base,), (warp, str(rows * ROW), base)),
            Ins("mad.lo.u32", (put,), (lane, "8", base)),
            Ins("mad.lo.u32", (get,), (lane, "4", base)),
            Ins("and.b32", (t1,), (lane, "15")),
            Ins("shl.b32", (t1,), (t1, "3")),
            Ins("shl.b32", (t2,), (lane, "2")),
            Ins("sub.s32", (t1,), (t1, t2)),
            Ins("shr.u32", (t3,), (lane, "4")),
            Ins("mad.lo.s32", (t1,), (t3, str(stride), t1)),
            Ins("cvt.s64.s32", (d64,), (t1,)),
            Ins("add.s64", (q,), (ptr, d64)),
        ]
        k.variables.add(q)
        wide = [(r("f32"), r("f32")) for _ in range(rows // 2)]
        head = [Ins(mem=Mem("ld", "global.nc", "f32", q, offs[0] + 2 * j * stride, pair))
                for j, pair in enumerate(wide)]
        head += [Ins(mem=Mem("st", "shared", "f32", put, j * 2 * ROW, pair))
                 for j, pair in enumerate(wide)]
        head.append(Ins("bar.warp.sync", src=("-1",), barrier=True))
        row_of = {i: (body[i].mem.off - offs[0]) // stride for i in best}
        tail = [Ins("bar.warp.sync", src=("-1",), barrier=True),
                Ins("add.s64", (q,), (q, str(st.rows[ptr])))]
        out = body[:pre] + prologue + body[pre:top + 1] + head
        for i in range(top + 1, len(body)):
            ins = body[i]
            if i in row_of:
                m = ins.mem
                out.append(Ins(mem=Mem("ld", "shared", m.typ, get, row_of[i] * ROW, m.regs)))
                continue
            if i == latch:
                out += tail
            out.append(ins)
        k.body = out

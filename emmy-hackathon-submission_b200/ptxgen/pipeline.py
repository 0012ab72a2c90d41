"""Asynchronous copies ahead of a single-wave runtime loop's read-only loads.

A runtime loop (one body per trip: unrolling is off, or the threads' trip counts differ) in a
kernel that runs in one wave has few warps per SM, and each trip's arithmetic waits on that
trip's own load: the loop runs at one memory latency per trip (the shipped ``r02_big_sum`` with
``--no_loop_unroll``: 128 threads, 512 trips of a load and an add each). A warp issues in
order, and any instruction that reads a register with a load still in flight stops it. So a
ring of registers cannot hold later trips' values without a copy of the body per ring slot,
which is unrolling. The copies go through shared memory instead: ``cp.async`` writes no
register, so a thread can have several trips' loads in flight while its arithmetic runs.

For each qualifying load, every thread owns one column of a ring of ``DEPTH`` slots in shared
memory (slot-major across the block's threads, so a warp's accesses to a slot are contiguous):

* in front of the loop, copies of trips 0 .. DEPTH-2 (trip j only where it exists), one
  commit group per trip;
* at the top of trip t: ``cp.async.wait_group DEPTH-2`` (trip t's group, the oldest, has
  landed), a copy of trip t + DEPTH - 1 into the slot trip t - 1 used (whose value that trip
  has already consumed: a warp issues in order, and its consumer waited for it), predicated on
  that trip existing, and one commit;
* the load itself becomes an ``ld.shared`` of the same width from trip t's slot, issued right
  after the wait (ahead of the refill and the slot arithmetic, which then cover its latency)
  unless an instruction before it in the body touches its registers;
* after the loop, ``cp.async.wait_all``.

The loop keeps one body per trip, with the same arithmetic in the same order on the same values.
A load qualifies when it reads ``global.nc`` memory (the kernel never writes it, so reading it
early reads the same value) of 4, 8 or 16 bytes (the sizes ``cp.async`` copies) through one of
the loop's 64-bit induction pointers (its address on every trip is the pointer plus a fixed
offset, and the latch adds a fixed delta), and runs on every trip: it sits in the body's first
straight-line stretch, unpredicated. Trip ``t + j``'s address is the pointer at trip ``t`` plus
``j`` deltas, and it is read only where trip ``t + j`` runs, so no address is touched that the
loop itself would not touch. Only short bodies (``MAX_BODY`` instructions) are rewritten, since a
long body already gives its loads a trip's worth of other work. A kernel that issues
``cp.async`` itself is left alone: its commit groups would share the thread's group count.
Each thread reads only the slots it wrote itself, after its own ``wait_group``, so no barrier
is needed.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field

from .dtypes import size

DEPTH = 8  # ring slots; trips in flight = DEPTH - 1 (the shipped r02: 8 and 16 ran alike)
MAX_BODY = 32  # instructions between a loop's top and its latch
MAX_RING_BYTES = 16 << 10  # shared memory all of a kernel's rings may take
STATIC_SMEM = 48 << 10  # a kernel's static shared memory limit
COPY_SIZES = (4, 8, 16)


@dataclass(eq=False)
class Pipe:
    """A runtime loop as the lowering left it: the instruction in front of which its preheader
    ends (``pre``), its top label, its latch branch, the counter with its constant step and the
    operand it is compared with, the latch's pointer deltas, and the L1 prefetch code the
    lowering put at its top (which the copies replace)."""

    pre: object
    top: object
    latch: object
    counter: str
    step: int
    end: str
    deltas: dict[str, int]
    prefetch: list = field(default_factory=list)


def _static_smem(k) -> int:
    return sum(int(m.group(1)) for d in k.shared_decls for m in [re.search(r"\[(\d+)\]", d)]
               if m)


def pipeline_loads(k, pipes: list[Pipe]) -> None:
    """Rewrite each recorded loop of kernel ``k`` in place (see the module docstring)."""
    from .ptx import Ins, Mem

    if not pipes or any(ins.op.startswith("cp.async") or
                        (ins.text is not None and "cp.async" in ins.text) for ins in k.body):
        return
    budget = min(MAX_RING_BYTES, STATIC_SMEM - _static_smem(k) - 1024)
    for n_ring, pipe in enumerate(pipes):
        body = k.body
        try:
            pre, top, latch = (next(n for n, ins in enumerate(body) if ins is want)
                               for want in (pipe.pre, pipe.top, pipe.latch))
        except StopIteration:  # a pass removed the loop
            continue
        if not pre < top < latch or latch - top > MAX_BODY:
            continue
        loads = []
        for n in range(top + 1, latch):
            ins = body[n]
            if ins.op.startswith("bra") or (ins.text is not None and ins.text.endswith(":")):
                break  # past the first straight-line stretch
            m = ins.mem
            if (m is None or m.kind != "ld" or m.space != "global.nc" or ins.pred or
                    m.addr not in pipe.deltas or
                    len(m.regs) * size(m.typ) not in COPY_SIZES):
                continue
            loads.append(n)
        if not loads:
            continue
        width = {n: len(body[n].mem.regs) * size(body[n].mem.typ) for n in loads}
        slot = k.max_threads * sum(width.values())  # bytes of one slot, all rings' columns
        if DEPTH * slot > budget:
            continue
        budget -= DEPTH * slot
        sym = f"{k.name}_ring{n_ring}"
        k.shared_decls.append(f"\t.shared .align 16 .b8 {sym}[{DEPTH * slot}];")

        def exists(j: int, code: list) -> str | None:
            """Predicate: trip (current + j) runs (the latch's own test); None for j = 0."""
            if j == 0:
                return None
            t, e = k.reg("u32"), k.reg("pred")
            code += [Ins("add.u32", (t,), (pipe.counter, str(j * pipe.step))),
                     Ins("setp.lt.s32", (e,), (t, pipe.end))]
            return e

        # this thread's column of each ring: ring base + the columns before it + tid * width
        tid, base = k.reg("u32"), k.reg("u32")
        prologue = [Ins("mov.u32", (tid,), ("%tid.x",)), Ins("mov.u32", (base,), (sym,))]
        column, at = {}, 0
        for n in loads:
            c = k.reg("u32")
            prologue.append(Ins("mad.lo.u32", (c,), (tid, str(width[n]), base)))
            if at:
                prologue.append(Ins("add.u32", (c,), (c, str(at))))
            column[n] = c
            at += k.max_threads * width[n]

        def copy(n: int, dst: str, dst_off: int, trips: int, pred: str | None) -> Ins:
            m = body[n].mem
            src = f"[{m.addr}+{m.off + trips * pipe.deltas[m.addr]}]"
            return Ins(text=f"\t{'@' + pred + ' ' if pred else ''}cp.async.ca.shared.global "
                            f"[{dst}+{dst_off}], {src}, {width[n]};")

        for j in range(DEPTH - 1):
            e = exists(j, prologue)
            prologue += [copy(n, column[n], j * slot, j, e) for n in loads]
            prologue.append(Ins(text="\tcp.async.commit_group;"))
        cur, prev = k.reg("u32"), k.reg("u32")
        prologue += [Ins("mov.u32", (cur,), ("0",)),
                     Ins("mov.u32", (prev,), (str((DEPTH - 1) * slot),))]
        k.variables.update((cur, prev))

        head = [Ins(text=f"\tcp.async.wait_group {DEPTH - 2};")]
        now, hoisted = {}, set()
        for n in loads:
            m = body[n].mem
            now[n] = k.reg("u32")
            head.append(Ins("add.u32", (now[n],), (column[n], cur)))
            regs = set(m.regs)
            if not any(regs & (set(body[j].reads()) | set(body[j].writes()))
                       for j in range(top + 1, n)):
                head.append(Ins(mem=Mem("ld", "shared", m.typ, now[n], 0, m.regs)))
                hoisted.add(n)
        e = exists(DEPTH - 1, head)
        for n in loads:
            old = k.reg("u32")
            head += [Ins("add.u32", (old,), (column[n], prev)), copy(n, old, 0, DEPTH - 1, e)]
        wrap = k.reg("pred")
        head += [Ins(text="\tcp.async.commit_group;"),
                 Ins("mov.u32", (prev,), (cur,)),
                 Ins("add.u32", (cur,), (cur, str(slot))),
                 Ins("setp.eq.u32", (wrap,), (cur, str(DEPTH * slot))),
                 Ins("mov.u32", (cur,), ("0",), pred=wrap)]
        covered = {body[n].mem.addr for n in loads}
        prefetched = {ins.mem.addr if ins.mem else None for ins in pipe.prefetch}
        prefetched |= {re.search(r"\[(%\w+)", s).group(1) for ins in pipe.prefetch
                       for s in ins.src if s.startswith("[")}
        drop = ({id(ins) for ins in pipe.prefetch}
                if prefetched - {None} <= covered else set())
        out = body[:pre] + prologue + body[pre:top + 1] + head
        for n in range(top + 1, len(body)):
            ins = body[n]
            if id(ins) in drop:
                continue
            if n in hoisted:
                continue
            if n in now:
                m = ins.mem
                out.append(Ins(mem=Mem("ld", "shared", m.typ, now[n], 0, m.regs)))
                continue
            out.append(ins)
            if ins is pipe.latch:
                out.append(Ins(text="\tcp.async.wait_all;"))
        k.body = out

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
* in front of the loop, once trip 0's group has landed, an ``ld.shared`` of its slot into a
  set of registers of the load's width (the read-ahead registers);
* at the top of trip t: the load's registers take the read-ahead registers' values (read one
  trip earlier, so the moves find them landed); ``cp.async.wait_group DEPTH-3`` (trip t + 1's
  group has landed); the read-ahead registers read trip t + 1's slot; a copy of trip
  t + DEPTH - 1 goes into the slot of trip t - 1 (read two trips before, its value long
  consumed), predicated on that trip existing; one commit;
* the load itself is gone from the body (a load qualifies only if nothing before it in the body
  touches its registers);
* after the loop, ``cp.async.wait_all``.

A slot's value is read into registers a whole trip before the trip that uses it, so the
shared-memory latency is hidden too: the shipped r02 with unrolling off took 17.4 us reading
each slot in its own trip and 15.95 us reading it a trip ahead.

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

from .dtypes import move_type, size

DEPTH = 8  # ring slots; trips in flight = DEPTH - 1 (the shipped r02: 8 and 16 ran alike)
MAX_BODY = 32  # instructions between a loop's top and its latch
MAX_RING_BYTES = 16 << 10  # shared memory all of a kernel's rings may take
STATIC_SMEM = 48 << 10  # a kernel's static shared memory limit
COPY_SIZES = (4, 8, 16)
_TYPE = {"%f": "f32", "%fd": "f64", "%r": "b32", "%rd": "b64", "%h": "b16"}


def _type_of(reg: str) -> str:
    return _TYPE[reg.rstrip("0123456789")]


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
            if any(set(m.regs) & (set(body[j].reads()) | set(body[j].writes()))
                   for j in range(top + 1, n)):
                continue  # its value cannot move to the top of the body
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
        # trip 0's values, read ahead once its group has landed
        ahead = {n: tuple(k.reg(_type_of(r)) for r in body[n].mem.regs) for n in loads}
        prologue.append(Ins(text=f"\tcp.async.wait_group {DEPTH - 2};"))
        prologue += [Ins(mem=Mem("ld", "shared", body[n].mem.typ, column[n], 0, ahead[n]))
                     for n in loads]
        nxt, prev = k.reg("u32"), k.reg("u32")  # slot offsets of trips t + 1 and t - 1
        prologue += [Ins("mov.u32", (nxt,), (str(slot),)),
                     Ins("mov.u32", (prev,), (str((DEPTH - 1) * slot),))]
        k.variables.update((nxt, prev))

        head = [Ins(f"mov.{move_type(_type_of(r))}", (r,), (a,))
                for n in loads for r, a in zip(body[n].mem.regs, ahead[n])]
        head.append(Ins(text=f"\tcp.async.wait_group {DEPTH - 3};"))
        for n in loads:
            at = k.reg("u32")
            head += [Ins("add.u32", (at,), (column[n], nxt)),
                     Ins(mem=Mem("ld", "shared", body[n].mem.typ, at, 0, ahead[n]))]
        e = exists(DEPTH - 1, head)
        for n in loads:
            old = k.reg("u32")
            head += [Ins("add.u32", (old,), (column[n], prev)), copy(n, old, 0, DEPTH - 1, e)]
        head.append(Ins(text="\tcp.async.commit_group;"))
        for r in (nxt, prev):
            wrap = k.reg("pred")
            head += [Ins("add.u32", (r,), (r, str(slot))),
                     Ins("setp.eq.u32", (wrap,), (r, str(DEPTH * slot))),
                     Ins("mov.u32", (r,), ("0",), pred=wrap)]
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
            if n in ahead:
                continue
            out.append(ins)
            if ins is pipe.latch:
                out.append(Ins(text="\tcp.async.wait_all;"))
        k.body = out

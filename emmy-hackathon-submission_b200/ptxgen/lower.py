"""Kernel IR -> PTX for sm_100a: the generic lowering, one ``emit_<Node>`` per statement kind.

Names map to values: an index is an ``Aff`` (see ``index``), data is a ``Val`` (see ``ops``), and a
predicate the ranges decide is a Python ``bool``. Semantics follow the reference lowering
(reference ``ptxgen/compiler.py``); the code generation is sm_100a's:

* every float add/sub/mul rounds with an explicit ``.rn`` and the only fma contractions are the
  ones ``ops.fma_operands`` makes, so results are reproducible bit for bit;
* global accesses are scalar here and merged into 64/128-bit ones by ``Kernel.vectorize``, using
  the divisibility facts of the index algebra to prove alignment;
* a 32-lane ``WarpShuffle`` whose combine is an f32 max/min (or an integer add) is one
  ``redux.sync`` instruction (sm_100a has the f32 form); other shuffles are a ``shfl.sync.bfly``
  ladder;
* a ``TreeHalve`` of at most 32 slots is read once from shared memory by every warp and finished
  with a shuffle ladder plus a broadcast of lane 0, which computes exactly the halving tree's
  value without a barrier per level;
* loops unroll by a static cost model (``_cost``): fully when all trips fit ``UNROLL_BUDGET``
  instructions, else with as many copies per trip as fit ``BODY_BUDGET`` (at most
  ``MAX_COPIES``; ``NESTED_COPIES`` for a loop around loops).
"""

from __future__ import annotations

import math
from typing import Any
from collections.abc import Iterator, Mapping, Sequence
from contextlib import AbstractContextManager, contextmanager, nullcontext
from dataclasses import dataclass

from . import fastmath, index, ops
from .dtypes import is_int, literal, mem_type, move_type, reg_type, size, smem_dtype
from .index import Aff
from .ir import (Accum, Assign, BinaryExpr, CastExpr, Cond, CpAsyncCommit, CpAsyncCopy,
                 CpAsyncWait, Expr, FuncCallExpr, Init, KernelOp, Let, Literal, Load, Loop,
                 Select, Smem, Stmt, StridedLoop, Sync, TernaryExpr, Tile, TreeHalve, Var,
                 WarpShuffle, Write, walk)
from .ops import Val
from .pipeline import Pipe
from .stage import MAX_ROWS as STAGE_ROWS
from .stage import Stage
from .ptx import BUFFER_ALIGN, SM_COUNT, Ins, Kernel, pow2_part

UNROLL_BUDGET = 6144  # instructions a loop may fully unroll to
BODY_BUDGET = 768  # instructions the copies in one trip of a partly unrolled loop may hold
MAX_COPIES = 16
NESTED_COPIES = 2
STATIC_SMEM_CAP = 48 * 1024  # past this, shared buffers live in one dynamic pool
MAX_IMM_OFFSET = 1 << 30  # larger constant byte offsets are added into the address register
PREFETCH_TRIPS = 16  # how many trips ahead a single-wave runtime loop prefetches its loads
BARRIERS = (Sync, WarpShuffle, TreeHalve, CpAsyncWait)
F32_SYMBOL = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide"}

Value = Aff | Val | bool


@dataclass(frozen=True)
class Buffer:
    """A kernel parameter's buffer, as meta.json describes it."""

    shape: tuple[int, ...]
    dtype: str
    is_output: bool


@dataclass(frozen=True)
class GlobalBuf:
    shape: tuple[int, ...]
    dtype: str
    ptr: str  # u64 register holding the buffer's global address
    writable: bool


@dataclass(frozen=True)
class SharedBuf:
    shape: tuple[int, ...]
    dtype: str
    base: str  # u32 register holding the shared address of the symbol
    offset: int  # byte offset of the buffer from it
    align: int


Memory = GlobalBuf | SharedBuf


def pack_shared(decls: Sequence[Smem]) -> tuple[dict[str, int], int]:
    """Byte offsets of the shared buffers packed in declaration order, each aligned to
    max(16, its alignment, its element size), and the total."""
    offsets, end = {}, 0
    for s in decls:
        esz = size(smem_dtype(s.dtype))
        align = max(16, int(s.align or 0), esz)
        end = -(-end // align) * align
        offsets[s.name] = end
        end += math.prod(int(e) for e in s.extents) * esz
    return offsets, end


class Lowering:
    def __init__(self, op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str],
                 block: int, *, no_unroll: bool = False, no_fusion: bool = False,
                 no_cse: bool = False, exchange: str | None = None):
        if not 1 <= block <= 1024:
            raise ValueError(f"block of {block} threads")
        self.op, self.block, self.buffers = op, block, dict(buffers)
        # an f32 output whose blocks' atomic adds this kernel then sums across ranks itself
        self.exchange = exchange
        if exchange is not None:
            buf = self.buffers.get(exchange)
            if buf is None or buf.dtype != "f32" or math.prod(buf.shape) != 1:
                raise ValueError(f"exchange: {exchange!r} is not a one-element f32 buffer")
        self.k = Kernel(op.name, list(arg_order), block, no_fusion=no_fusion, no_cse=no_cse)
        self.no_unroll = no_unroll
        self.env: dict[str, Value] = {}
        self.mem: dict[str, Memory] = {}
        self.loop_depth = 0
        self._converged = False  # every thread of the block is running this code together
        self._order = {id(st): i for i, st in enumerate(walk([op.body]))}
        self._stmts = list(walk([op.body]))

    # --- walking ----------------------------------------------------------------------
    def run(self) -> Kernel:
        """The whole kernel: parameter pointers, thread registers, shared buffers, then the
        body's statements in order."""
        self._bind_parameters()
        k = self.k
        self.tid = k.pure("mov.u32", "u32", "%tid.x", rng=(0, self.block - 1))
        self.ctaid = k.pure("mov.u32", "u32", "%ctaid.x")
        if self._uses_lanes():
            last = self.block - 1
            lane = k.pure("and.b32", "u32", self.tid, "31", rng=(0, min(31, last)))
            warp = k.pure("shr.u32", "u32", self.tid, "5", rng=(0, last >> 5))
            self.env["lane"], self.env["warp"] = Aff.of(lane), Aff.of(warp)
        self.mem.update(self._declare_shared(list(self.op.smem_buffers.values())))
        self.body([self.op.body])
        return k

    def _bind_parameters(self) -> None:
        """Each parameter's global pointer, in ``arg_order`` (the entry's .param list)."""
        k = self.k
        missing = [name for name in k.params if name not in self.buffers]
        if missing:
            raise ValueError(f"parameter {missing[0]!r} has no buffer")
        for name in k.params:
            buf = self.buffers[name]
            param = k.reg("u64")
            k.emit("ld.param.u64", (param,), (f"[{k.name}_param_{name}]",))
            ptr = k.pure("cvta.to.global.u64", "u64", param)
            k.align[ptr] = BUFFER_ALIGN
            self.mem[name] = GlobalBuf(tuple(buf.shape), buf.dtype, ptr, buf.is_output)

    def _uses_lanes(self) -> bool:
        """Whether the body needs the lane and warp registers: it reduces across lanes, or an
        expression names ``lane`` or ``warp``."""
        if any(isinstance(st, WarpShuffle | TreeHalve) for st in self._stmts):
            return True
        return any(isinstance(e, Var) and e.name in ("lane", "warp")
                   for st in self._stmts for e in _expressions_of(st))

    def body(self, stmts: Sequence[Stmt]) -> None:
        for st in stmts:
            method = _HANDLERS.get(type(st))
            if method is None:
                raise NotImplementedError(f"no PTX lowering for Kernel IR node {type(st).__name__}")
            getattr(self, method)(st)

    @contextmanager
    def _block(self) -> Iterator[None]:
        """A lexical scope: a name first bound inside it is unbound when it ends, while a new
        value given to a name bound outside it stays."""
        outer = frozenset(self.env)
        try:
            yield
        finally:
            for name in [n for n in self.env if n not in outer]:
                self.env.pop(name)

    def _where(self, p: str | bool) -> AbstractContextManager[None]:
        """A block that runs only where predicate ``p`` holds (always when ``p`` is True)."""
        if p is True:
            return nullcontext()
        return self.k.skip_if(f"!{p}")

    # --- names ------------------------------------------------------------------------
    # ``env`` maps each Kernel IR name to its value. A *variable* is a register that is written
    # in place (an accumulator, a loop-carried state, a reduction's state); every other data
    # register is written once. A name bound to data never shares a variable's register, or it
    # would see the variable's later writes.

    def _lookup(self, name: str) -> Value:
        try:
            return self.env[name]
        except KeyError:
            raise KeyError(f"{name!r} is used before it is defined") from None

    def _data(self, name: str) -> Val:
        return self._as_val(self._lookup(name))

    def _snapshot(self, v: Val) -> Val:
        """A write-once copy of a variable's current value."""
        typ = reg_type(v.dtype)
        copy = self.k.reg(typ)
        self.k.emit(f"mov.{move_type(typ)}", (copy,), (v.reg,))
        return Val(copy, v.dtype)

    def _define(self, name: str, v: Val) -> None:
        """Bind ``name`` to ``v`` (a snapshot, when ``v`` is a variable)."""
        self.env[name] = self._snapshot(v) if v.reg in self.k.variables else v

    def _init(self, name: str, identity: float | None, dtype: str) -> None:
        """Bind ``name`` to a new variable of ``dtype`` that starts at ``identity``."""
        if identity is None:
            raise ValueError(f"{name!r} has no identity to start from")
        typ = reg_type(dtype)
        self.env[name] = Val(self.k.variable(typ, literal(identity, typ)), dtype)

    def _variable(self, name: str, dtype: str | None = None) -> Val:
        """``name``'s value as a variable (of ``dtype``, when given) that can be written in
        place; a write-once value is moved into a new variable, which ``name`` then names."""
        current = self._data(name)
        if dtype is not None and dtype != current.dtype:
            current = ops.convert(self.k, current, dtype)
        if current.reg in self.k.variables:
            return current
        var = Val(self.k.variable(reg_type(current.dtype), current.reg), current.dtype)
        self.env[name] = var
        return var

    def _write(self, name: str, v: Val) -> None:
        """Write ``v`` into variable ``name`` in place (converted to the variable's dtype)."""
        var = self._variable(name)
        self._move_into(var, ops.convert(self.k, v, var.dtype).reg)

    def _move_into(self, var: Val, src: str) -> None:
        if src == var.reg:
            return
        self.k.emit(f"mov.{move_type(reg_type(var.dtype))}", (var.reg,), (src,))
        self.k.forget(var.reg)  # results computed from its old value are stale now

    # --- launch -----------------------------------------------------------------------
    def emit_Tile(self, t: Tile) -> None:
        """The grid: one thread per Tile cell, cell ``ctaid * block + tid``; the axes decoded
        from it; the tail guard only when the last block is partial."""
        k = self.k
        cells = self._check_grid(t)
        blocks = -(-cells // self.block)
        k.ranges[self.ctaid] = (0, blocks - 1)
        k.header_notes.append(f"// @ptxgen launch grid={blocks} block={self.block}")
        if blocks <= SM_COUNT:
            # One wave: no SM ever holds a second CTA, so ptxas may spend the whole register file
            # on one. Left to its occupancy heuristic, a long unrolled block can come out at 32
            # registers and kilobytes of spills.
            k.min_ctas = 1
        cell = Aff.combine((Aff.of(self.ctaid), self.block), (Aff.of(self.tid), 1))
        beyond = index.compare(k, ">=", cell, Aff.k(cells))
        if beyond is True:
            return
        guarded = beyond is not False
        if guarded and any(isinstance(st, BARRIERS) for st in walk(t.body)):
            raise NotImplementedError("Tile: a partial last block around a barrier")
        with (k.skip_if(beyond) if guarded else nullcontext()), self._block():
            self.env.update(self._decode(t, cell, _raster_pair(t)))
            # every thread of a block runs the Tile body together (no tail guard), until a
            # condition splits them; the staging pass needs whole warps
            self._converged = not guarded
            self.body(t.body)
            self._converged = False
        if self.exchange is not None:  # every thread reaches it, past the tail guard
            from .templates.exchange import emit_epilogue

            # whichever thread added the block's share, it happens before thread 0's release
            k.emit("bar.sync", src=("0",), barrier=True)
            emit_epilogue(k, self.tid, self.mem[self.exchange].ptr)

    def _check_grid(self, t: Tile) -> int:
        """The Tile's cell count, after the checks this lowering needs of its grid."""
        if not t.is_static_grid or t.aux_threads:
            raise NotImplementedError("Tile: only static grids without an aux thread band")
        if t.n_elements > 2**31 - 1:
            raise NotImplementedError("Tile: more than 2^31 - 1 cells")
        if t.block_threads is not None and t.block_threads != self.block:
            raise ValueError(f"Tile block_threads {t.block_threads} != launch block {self.block}")
        return t.n_elements

    def emit_Sync(self, s: Sync) -> None:
        if s.warp:
            if s.barrier_id:
                raise ValueError("Sync(warp=True) cannot carry a named barrier_id")
            self.k.emit("bar.warp.sync", src=("-1",), barrier=True)
            return
        if s.count is None:
            if s.barrier_id:
                raise ValueError(f"Sync(barrier_id={s.barrier_id}) requires count")
            operands: tuple[str, ...] = ("0",)
        else:
            operands = (str(s.barrier_id), str(s.count))
        self.k.emit("bar.sync", src=operands, barrier=True)

    def _decode(self, t: Tile, cell: Aff, raster: tuple[int, int, int] | None
                ) -> dict[str, Aff]:
        """Each Tile axis as an index of the cell number, in Emmy's block order: row-major
        (axis i is ``cell / stride_i % extent_i``; the outermost axis needs no ``%``), except a
        raster pair, which ``_grouped`` decodes."""
        k = self.k
        extents = [int(e) for e in t.extents]
        strides = [math.prod(extents[i + 1:]) for i in range(len(extents))]
        paired = set(raster[:2]) if raster is not None else set()
        out: dict[str, Aff] = {}
        for i, axis in enumerate(t.axes):
            if i in paired:
                continue
            if extents[i] == 1:
                out[axis.name] = Aff()
                continue
            value = index.div(k, cell, strides[i])
            out[axis.name] = value if i == 0 else index.mod(k, value, extents[i])
        if raster is not None:
            grouped, other, group = raster
            inner = max(grouped, other)
            pair_cell = index.div(k, cell, strides[inner])
            if min(grouped, other) > 0:  # axes outside the pair: keep the pair's own part
                pair_cell = index.mod(k, pair_cell, extents[grouped] * extents[other])
            a, b = self._grouped(pair_cell, extents[grouped], extents[other], group)
            out[t.axes[grouped].name], out[t.axes[other].name] = a, b
        return out

    def _grouped(self, c: Aff, ea: int, eb: int, g: int) -> tuple[Aff, Aff]:
        """The grouped decode of a raster pair's cell ``c``: the grouped axis (extent ``ea``)
        advances in groups of ``g``; within a group the cells run down the group first, then
        across the other axis (extent ``eb``). A ragged last group is ``ea mod g`` wide."""
        k = self.k
        if eb == 1:
            return c, Aff()
        span = g * eb  # cells of one whole group
        group_no = index.div(k, c, span)
        within = index.mod(k, c, span)
        width: Aff = Aff.k(g)
        if ea % g:
            width = index.minimum(k, Aff.k(ea) - group_no * g, width)
        a = group_no * g + index.mod(k, within, width)
        return a, index.div(k, within, width)

    # --- memory -----------------------------------------------------------------------
    def emit_Smem(self, s: Smem) -> None:
        pass  # declared up front, so an Smem inside a loop is still one buffer

    def _address(self, mem: Memory, flat: Aff, dtype: str) -> tuple[str, int, str]:
        """(address register, byte offset, state space) of element ``flat``."""
        k, esz = self.k, size(mem_type(dtype))
        if abs(flat.const * esz) > MAX_IMM_OFFSET:  # the constant joins the index register
            var, flat = flat, Aff()
        else:
            var = flat.var_part()
        if isinstance(mem, GlobalBuf):
            addr, align = mem.ptr, BUFFER_ALIGN
            if not var.is_const:
                g = math.gcd(var.var_mult(k.mult), var.const)
                align = min(BUFFER_ALIGN, pow2_part(g * esz))
                # in a runtime loop: a 64-bit pointer the latch steps, not index math per trip
                iv = k.induction(mem.ptr, var, esz, align)
                if iv is not None:
                    addr = iv
                else:
                    wide = k.pure("mul.wide.u32", "u64", index.reg_of(k, var), str(esz))
                    addr = k.pure("add.s64", "u64", mem.ptr, wide)
            k.align[addr] = max(k.align.get(addr, 1), align)
            return addr, flat.const * esz, "global" if mem.writable else "global.nc"
        addr, align = mem.base, mem.align
        if not var.is_const:
            g = math.gcd(var.var_mult(k.mult), var.const)
            addr = k.pure("mad.lo.u32", "u32", index.reg_of(k, var), str(esz), mem.base)
            align = min(mem.align, pow2_part(g * esz))
        k.align[addr] = max(k.align.get(addr, 1), align)
        return addr, mem.offset + flat.const * esz, "shared"

    def _load(self, mem: Memory, flat: Aff, dtype: str, n: int = 1) -> list[Val]:
        addr, off, space = self._address(mem, flat, dtype)
        typ, rtyp, esz = mem_type(dtype), reg_type(dtype), size(mem_type(dtype))
        out = []
        for j in range(n):
            if space == "global.nc":
                r = self.k.cached_load(space, typ, addr, off + j * esz)
                if rtyp != typ and typ not in ("b16",):
                    r = self._retype(r, typ, rtyp)
            else:
                r = self.k.reg(rtyp if typ != "u8" else "u16")
                self.k.mem("ld", space, typ, addr, off + j * esz, (r,))
            out.append(Val(r, dtype))
        return out

    def _retype(self, r: str, typ: str, rtyp: str) -> str:
        return r  # registers of one width share a class; no move is needed

    def _store(self, mem: Memory, flat: Aff, values: Sequence[Val]) -> None:
        addr, off, space = self._address(mem, flat, mem.dtype)
        typ, esz = mem_type(mem.dtype), size(mem_type(mem.dtype))
        for j, v in enumerate(values):
            r = ops.convert(self.k, v, mem.dtype).reg
            self.k.mem("st", space, typ, addr, off + j * esz, (r,))

    def _element(self, name: str, exprs: Sequence[Expr]) -> tuple[Memory, Aff]:
        """Buffer ``name`` and the flat element offset its index expressions select."""
        mem = self.mem[name]
        return mem, _row_major(name, mem.shape, [self._int(e) for e in exprs])

    def emit_Load(self, s: Load) -> None:
        mem, flat = self._element(s.input, s.index)
        dtype = mem.dtype if s.dtype is None else s.dtype.name
        values = self._load(mem, flat, dtype, len(s.names))
        self.env.update(zip(s.names, values, strict=True))

    def emit_Write(self, s: Write) -> None:
        if s.swizzle != "NONE":
            raise NotImplementedError(f"Write: swizzle {s.swizzle}")
        mem, flat = self._element(s.output, s.index)
        values = [self._data(v) for v in s.values]
        if s.atomic:
            self._add_into(mem, flat, values)
        else:
            self._store(mem, flat, values)

    def _add_into(self, mem: Memory, flat: Aff, values: Sequence[Val]) -> None:
        """``red.global.add`` of each value into consecutive elements from ``flat`` (the
        split-K finalize: blocks add their partials into a zeroed output)."""
        if isinstance(mem, SharedBuf):
            raise NotImplementedError("Write: atomic to shared memory")
        form = _RED_ADD.get(mem.dtype)
        if form is None:
            raise NotImplementedError(f"Write: atomic add of {mem.dtype}")
        k = self.k
        addr, off, _ = self._address(mem, flat, mem.dtype)
        step = size(mem_type(mem.dtype))
        for j, v in enumerate(values):
            k.mem("red", "global", form, addr, off + j * step,
                  (ops.convert(k, v, mem.dtype).reg,))

    def emit_CpAsyncCopy(self, s: CpAsyncCopy) -> None:
        """One asynchronous copy of ``nbytes`` (4, 8 or 16) from global to shared memory; a
        ``lane_index`` offsets the shared destination per lane. 16-byte copies bypass L1."""
        if s.swizzle != "NONE":
            raise NotImplementedError(f"CpAsyncCopy: swizzle {s.swizzle}")
        if s.nbytes not in (4, 8, 16):
            raise ValueError(f"CpAsyncCopy: nbytes {s.nbytes} is not 4, 8 or 16")
        dst_index: tuple[Expr, ...] = tuple(s.smem_index)
        if s.lane_index is not None:
            dst_index = tuple(BinaryExpr("+", at, lane)
                              for at, lane in zip(dst_index, s.lane_index, strict=True))
        operands = []
        for name, exprs in ((s.smem, dst_index), (s.src, s.src_index)):
            mem, flat = self._element(name, exprs)
            addr, off, _ = self._address(mem, flat, mem.dtype)
            operands.append(f"[{addr}+{off}]")
        level = "cg" if s.nbytes == 16 else "ca"
        self.k.raw(f"cp.async.{level}.shared.global {operands[0]}, {operands[1]}, {s.nbytes};")

    def emit_CpAsyncCommit(self, _s: CpAsyncCommit) -> None:
        self.k.raw("cp.async.commit_group;")

    def emit_CpAsyncWait(self, s: CpAsyncWait) -> None:
        self.k.raw(f"cp.async.wait_group {s.group};")

    def _declare_shared(self, decls: list[Smem]) -> dict[str, SharedBuf]:
        """Every Smem buffer of the kernel, declared once up front in declaration order: each a
        static ``.shared`` array, or, when together they pass ``STATIC_SMEM_CAP``, an offset
        into one dynamic pool the launcher sizes (``// @ptxgen dynamic_smem=``)."""
        k = self.k
        offsets, total = pack_shared(decls)
        pooled = total > STATIC_SMEM_CAP
        if pooled:
            pool_align = max([16, *(int(d.align or 0) for d in decls)])
            k.module_decls.append(f".extern .shared .align {pool_align} .b8 smem_pool[];\n")
            k.header_notes.append(f"// @ptxgen dynamic_smem={total}")
        out: dict[str, SharedBuf] = {}
        for d in decls:
            out[d.name] = self._shared_buffer(d, offsets[d.name] if pooled else None)
        return out

    def _shared_buffer(self, d: Smem, pool_offset: int | None) -> SharedBuf:
        dtype = smem_dtype(d.dtype)
        if dtype not in _SHARED_DTYPES:
            raise NotImplementedError(f"Smem: dtype {d.dtype}")
        if d.name in self.buffers:
            raise ValueError(f"Smem {d.name!r}: name already declared")
        k = self.k
        shape = tuple(int(e) for e in d.extents)
        esz = size(mem_type(dtype))
        if pool_offset is not None:
            base = k.pure("mov.u32", "u32", "smem_pool", mult=16)
            return SharedBuf(shape, dtype, base, pool_offset, 16)
        align = max(16, int(d.align or 0), esz)
        symbol = f"smem_{d.name}"
        k.shared_decls.append(
            f"\t.shared .align {align} .b8 {symbol}[{math.prod(shape) * esz}];")
        base = k.pure("mov.u32", "u32", symbol)
        k.align[base] = align
        return SharedBuf(shape, dtype, base, 0, align)

    # --- data -------------------------------------------------------------------------
    def emit_Assign(self, s: Assign) -> None:
        args = [self._data(a) for a in s.args]
        dtype = None if s.dtype is None else s.dtype.name
        self._define(s.name, ops.assign(self.k, s.op.name, dtype, args))

    def emit_Let(self, s: Let) -> None:
        """An untyped Let binds whatever its expression is (an index stays an index); a typed
        one binds data of its dtype."""
        if s.dtype is None:
            value = self.expr(s.value)
        else:
            value = self._value(s.value, s.dtype.name)
        if isinstance(value, Val):
            self._define(s.name, value)
        else:
            self.env[s.name] = value

    def emit_Init(self, s: Init) -> None:
        self._init(s.name, s.identity, s.dtype.name)

    def emit_Select(self, s: Select) -> None:
        choice = TernaryExpr(s.cond, s.if_true, s.if_false)
        self._define(s.name, self._value(choice, "f32"))

    def emit_Accum(self, s: Accum) -> None:
        """``acc = base op value`` in place (``base`` is the accumulator itself unless the
        statement names one, as an online-softmax rescale does)."""
        op = ops.canonical(s.op.name)
        dtype = "f32" if s.dtype is None else s.dtype.name
        if op not in ops.ACCUM:
            raise NotImplementedError(f"Accum: op {s.op.name} is not a binary op")
        if s.name not in self.env:  # no seeding loop: start from the identity here
            self._init(s.name, s.op.identity, dtype)
        k = self.k
        acc = self._variable(s.name, dtype).reg
        value = ops.convert(k, self._data(s.value), dtype).reg
        base = acc
        if s.base is not None:
            base = ops.convert(k, self._data(s.base), dtype).reg
        self._fold_into(acc, op, reg_type(dtype), base, value)
        k.forget(acc)

    def _fold_into(self, acc: str, op: str, typ: str, base: str, value: str) -> None:
        """One instruction (or an f32 detour) writing ``base op value`` into ``acc``: an add of
        a reusable product fuses into an fma; bf16, and f16 division, have no native form and
        compute in f32, rounded back once."""
        k = self.k
        if op == "add":
            fused = ops.fma_operands(k, typ, value, base)
            if fused is not None:
                k.emit(f"fma.rn.{typ}", (acc,), fused)
                return
        if typ == "bf16" or (typ == "f16" and op == "divide"):
            wide = [Val(ops.cvt(k, r, typ, "f32"), "f32") for r in (base, value)]
            k.emit(f"cvt.rn.{typ}.f32", (acc,), (ops.apply(k, op, wide, "f32").reg,))
            return
        float_form, int_form = ops.ACCUM[op]
        mnemonic = float_form if typ in ("f32", "f64", "f16") else int_form
        k.emit(f"{ops.arith(k, mnemonic)}.{typ}", (acc,), (base, value))

    # --- reduce -----------------------------------------------------------------------
    def _combine(self, program: Sequence[Assign], states: Sequence[str]) -> None:
        for a in program:
            dtype = a.dtype.name if a.dtype is not None else None
            v = ops.assign(self.k, a.op.name, dtype, [self._data(x) for x in a.args])
            (self._write if a.name in states else self._define)(a.name, v)

    def _redux_form(self, s: WarpShuffle) -> str | None:
        """The ``redux.sync`` op computing this 32-lane shuffle exactly, if there is one."""
        if s.length != 32 or len(s.state) != 1 or len(s.combine_states) != 1:
            return None
        a = s.combine_states[0]
        st, sb, dtype = s.state[0], s.state_b[0], s.dtype.name
        if a.name != st or set(a.args) != {st, sb} or len(a.args) != 2:
            return None
        if a.dtype is not None and a.dtype.name != dtype:
            return None
        name = ops.canonical(a.op.name)
        if dtype == "f32" and name in ("maximum", "minimum"):
            return f"redux.sync.{'max' if name == 'maximum' else 'min'}.f32"
        if dtype in ("i32", "u32") and name in ("add", "maximum", "minimum"):
            op = {"add": "add", "maximum": "max", "minimum": "min"}[name]
            return f"redux.sync.{op}.{'s32' if dtype == 'i32' else 'u32'}"
        return None

    def emit_WarpShuffle(self, s: WarpShuffle) -> None:
        """A butterfly across ``length`` lanes of each state variable, combined by the Assign
        program at every stride (one ``redux.sync`` where that is exact)."""
        problem = _shuffle_problem(s)
        if problem is not None:
            raise problem
        dtype = s.dtype.name
        states = [self._variable(st, dtype) for st in s.state]
        mask = self._active_mask()
        form = self._redux_form(s)
        if form is None:
            self._ladder(s.state, s.state_b, s.combine_states, s.length, dtype, mask)
            return
        reduced = self.k.reg(reg_type(dtype))
        self.k.emit(form, (reduced,), (self._data(s.state[0]).reg, mask))
        self._write(s.state[0], Val(reduced, states[0].dtype))

    def _active_mask(self) -> str:
        mask = self.k.reg("u32")
        self.k.emit("activemask.b32", (mask,))
        return mask

    def _ladder(self, state: Sequence[str], state_b: Sequence[str], program: Sequence[Assign],
                length: int, dtype: str, mask: str) -> None:
        step = length // 2
        while step:
            for st, sb in zip(state, state_b, strict=True):
                other = ops.shfl(self.k, self._data(st).reg, reg_type(dtype), "bfly", step, 31,
                                 mask)
                self.env[sb] = Val(other, dtype)
            self._combine(program, state)
            step //= 2

    def _touched_after(self, s: Stmt, bufs: Sequence[str]) -> bool:
        """Whether any statement after ``s`` (or ``s`` inside a loop) uses one of ``bufs``."""
        if self.loop_depth:
            return True
        pos = self._order[id(s)]
        names = set(bufs)
        for st in self._stmts[pos + 1:]:
            used = set()
            if isinstance(st, Load):
                used.add(st.input)
            elif isinstance(st, Write):
                used.add(st.output)
            elif isinstance(st, CpAsyncCopy):
                used |= {st.smem, st.src}
            elif isinstance(st, TreeHalve):
                used |= set(st.bufs)
            if used & names:
                return True
        return False

    def emit_TreeHalve(self, s: TreeHalve) -> None:
        """The halving tree over shared slots: at each level slot t folds in slot t + half,
        until slot 0 holds the result, which every thread takes. Segmented (``inner``): slot t
        is buf[t * scale + inner]. Up to 32 unsegmented shared slots are reduced by a shuffle
        ladder over one read of the slots instead (``_tree_by_shuffle``), with the same
        result."""
        problem = _tree_problem(s)
        if problem is not None:
            raise problem
        trees = [(self.mem[buf], st, sb)
                 for buf, st, sb in zip(s.bufs, s.state, s.state_b, strict=True)]
        for mem, st, _ in trees:
            self._variable(st, mem.dtype)
        tid = self._int(Var(s.tid_var))
        by_shuffle = s.length <= 32 and s.inner is None and all(
            isinstance(mem, SharedBuf) for mem, _, _ in trees)
        if not by_shuffle:
            self._tree_by_halving(s, trees, tid)
            return
        self._tree_by_shuffle(s, trees)
        if self._touched_after(s, s.bufs):
            self.emit_Sync(Sync(barrier_id=s.barrier_id, count=s.barrier_count))

    def _tree_by_shuffle(self, s: TreeHalve, trees: list[tuple[Memory, str, str]]) -> None:
        """Every warp reads the ``length`` slots into its lanes and runs the butterfly ladder
        with strides length/2 .. 1: lane 0 then holds exactly the halving tree's value (each
        level combines the same pairs in the same order), which lane 0 broadcasts."""
        k = self.k
        lane = self._lookup("lane")
        assert isinstance(lane, Aff)
        slot = lane if s.length == 32 else index.mod(k, lane, s.length)
        for mem, st, _ in trees:
            self._write(st, self._load(mem, slot, mem.dtype)[0])
        mask = k.reg("u32")
        k.emit("activemask.b32", (mask,))
        dtype = trees[0][0].dtype
        if any(m.dtype != dtype for m, _, _ in trees):
            raise NotImplementedError("TreeHalve: buffers of different dtypes")
        self._ladder(s.state, s.state_b, s.combine_states, s.length, dtype, mask)
        for _, st, _ in trees:
            v = self._data(st)
            top = ops.shfl(k, v.reg, reg_type(v.dtype), "idx", 0, 31, mask)
            self._write(st, Val(top, v.dtype))

    def _tree_by_halving(self, s: TreeHalve, trees: list[tuple[Memory, str, str]], t: Aff) -> None:
        """Level by level, halves ``length/2 .. 1``: thread t < half combines slot t with slot
        t + half and stores the result in slot t; a barrier closes each level. Then every
        thread reads the root slot."""
        k = self.k
        if s.inner is None:
            scale, root = 1, Aff()
        else:
            scale, root = s.inner[1], self._int(Var(s.inner[0]))
        level_done = Sync(barrier_id=s.barrier_id, count=s.barrier_count)
        half = s.length // 2
        while half:
            mine = t * scale + root
            active = index.compare(k, "<", t, Aff.k(half))
            with self._where(active), self._block():
                for mem, st, sb in trees:
                    self._write(st, self._load(mem, mine, mem.dtype)[0])
                    self.env[sb] = self._load(mem, mine + half * scale, mem.dtype)[0]
                self._combine(s.combine_states, s.state)
                for mem, st, _ in trees:
                    self._store(mem, mine, [self._data(st)])
            self.emit_Sync(level_done)
            half //= 2
        for mem, st, _ in trees:
            self._write(st, self._load(mem, root, mem.dtype)[0])

    # --- control ----------------------------------------------------------------------
    def emit_Cond(self, s: Cond) -> None:
        """``if``: a decided condition keeps one branch only; an ``if`` without ``else`` is a
        predicated region; otherwise two regions joined by branches."""
        p = self._pred(s.cond)
        if isinstance(p, bool):
            with self._block():
                self.body(s.body if p else s.else_body)
            return
        converged, self._converged = self._converged, False
        if not s.else_body:
            with self._where(p), self._block():
                self.body(s.body)
        else:
            self._if_else(p, s.body, s.else_body)
        self._converged = converged

    def _if_else(self, p: str, then: Sequence[Stmt], otherwise: Sequence[Stmt]) -> None:
        k = self.k
        to_else, to_end = k.label("else"), k.label("endif")
        k.emit("bra", src=(to_else,), pred=f"!{p}", barrier=True)
        for label, stmts, leave in ((None, then, to_end), (to_else, otherwise, None)):
            if label is not None:
                k.place(label)
            with k.region(), self._block():
                self.body(stmts)
                if leave is not None:
                    k.emit("bra.uni", src=(leave,), barrier=True)
        k.place(to_end)

    def emit_Loop(self, s: Loop | StridedLoop) -> None:
        """for (axis = start; axis < end; axis += step) body. Seeds the Accums of its own body,
        then picks a shape: a runtime loop (one copy per trip) when threads run trip counts
        more than one apart, a barrier meets differing counts, or unrolling is off; otherwise
        a full unroll when it fits ``UNROLL_BUDGET``, else a counted loop of ``f`` copies per
        trip followed by the leftover trips as copies (guarded where some thread stops)."""
        start, step, end = self._loop_range(s)
        self._seed_accumulators(s)
        stmts = list(walk(s.body))
        written = self._carried(stmts)
        trips = None if self.no_unroll else self._trips(start, step, end, stmts)
        self.loop_depth += 1
        try:
            if trips is None:
                self._runtime_loop(s, start, step, end, written)
            else:
                self._static_loop(s, start, step.const, end, trips, stmts, written)
        finally:
            self.loop_depth -= 1

    def _loop_range(self, s: Loop | StridedLoop) -> tuple[Aff, Aff, Aff]:
        """(start, step, end) of the loop's axis; a Loop runs 0, 1, ... up to its extent, a
        StridedLoop from its own start by its own step up to its end (default: the extent)."""
        end: Aff | None = None
        if isinstance(s, StridedLoop):
            step = self._int(s.step) if isinstance(s.step, Expr) else Aff.k(int(s.step))
            start = self._int(s.start)
            if s.end is not None:
                end = self._int(s.end)
        else:
            if getattr(s, "carries", None):
                raise NotImplementedError("Loop: carried state")
            start, step = Aff(), Aff.k(1)
        if end is None:
            extent = s.axis.extent
            if not extent.is_static:
                raise NotImplementedError(f"loop over {s.axis.name}: symbolic extent")
            end = Aff.k(extent.as_static())
        return start, step, end

    def _seed_accumulators(self, s: Loop | StridedLoop) -> None:
        """A seeding loop starts each accumulator its body folds into at the op's identity;
        otherwise an enclosing loop must have seeded it."""
        firsts: dict[str, Accum] = {}
        for st in s.body:
            if isinstance(st, Accum):
                firsts.setdefault(st.name, st)
        for name, acc in firsts.items():
            if s.seed:
                self._init(name, acc.op.identity, "f32" if acc.dtype is None else acc.dtype.name)
            elif name not in self.env:
                raise ValueError(f"Accum {name!r}: seed=False but no enclosing seed")

    def _carried(self, stmts: Sequence[Stmt]) -> list[str]:
        """The variables of the names the loop body writes in place (live across every trip);
        no result computed from them before the loop may be reused inside it."""
        names = {n for st in stmts for n in _state_written(st)} & set(self.env)
        regs = [self._variable(n).reg for n in sorted(names)]
        for reg in regs:
            self.k.forget(reg)
        return regs

    def _static_loop(self, s: Loop | StridedLoop, start: Aff, n: int, end: Aff,
                     trips: tuple[int, int], stmts: Sequence[Stmt], written: list[str]) -> None:
        """A loop whose trip counts the facts bound (``lo`` every thread runs, ``hi`` some):
        fully unrolled, or ``f`` copies per counted trip and the rest unrolled."""
        lo, hi = trips
        f = self._unroll_factor(s, hi, stmts)
        if f is None and lo >= 2 * STAGE_ROWS and self._stageable(s, start, stmts):
            # a counted loop of whole warp rows, which the staging pass fetches wide, where a
            # full unroll would leave scalar loads (config 4's per-rank shares)
            f = STAGE_ROWS
        m = 0 if f is None else lo // f * f  # trips the counted loop runs
        if m:
            self._counted(s, start, n, m, f, written)
        self._unrolled(s, start, n, end, lo, range(m, hi))

    def _unroll_factor(self, s: Loop | StridedLoop, hi: int, stmts: Sequence[Stmt]
                       ) -> int | None:
        """Copies per trip of a counted loop, or None to unroll every trip: when there is at
        most one, or all ``hi`` copies fit ``UNROLL_BUDGET`` estimated instructions (four
        times that for a loop marked unroll). A loop around loops takes ``NESTED_COPIES``,
        others the largest power of two whose copies fit ``BODY_BUDGET``."""
        if hi <= 1:
            return None
        cost = max(1, self._cost(s.body))
        budget = UNROLL_BUDGET * (4 if s.unroll is True else 1)
        if hi * cost <= UNROLL_BUDGET or hi * cost <= budget:
            return None
        if any(isinstance(st, Loop | StridedLoop) for st in stmts):
            f = NESTED_COPIES
        else:
            f = 1 << max(0, (BODY_BUDGET // cost).bit_length() - 1)
        return max(1, min(f, MAX_COPIES, hi))

    emit_StridedLoop = emit_Loop

    def _unrolled(self, s: Loop | StridedLoop, start: Aff, n: int, end: Aff, lo: int,
                  trips: range) -> None:
        """One copy of the body per trip j in ``trips``, the axis at ``start + j*n``. Trips
        below ``lo`` run on every thread; a later copy runs where its axis value is still below
        ``end``, and none after the first copy no thread reaches."""
        k = self.k
        for j in trips:
            at = start + j * n
            runs = True if j < lo else index.compare(k, "<", at, end)
            if runs is False:
                return
            with self._where(runs), self._block():
                self.env[s.axis.name] = at
                self.body(s.body)

    def _loop_head(self, init: Aff, bound: Aff, rng: tuple[int, int] | None,
                   mult: int) -> tuple[str, str, str, str | bool]:
        k = self.k
        i = k.variable("u32", index.operand(k, init))
        if rng is not None:
            k.ranges[i] = rng
        if mult > 1:
            k.mult[i] = mult
        enters = index.compare(k, "<", init, bound)
        top, done = k.label("loop"), k.label("loop_end")
        return i, top, done, enters

    def _iv_counter(self, s: Loop | StridedLoop, i: str) -> str | None:
        """The counter through which this loop's global addresses become 64-bit induction
        pointers (``Kernel.induction``), or None. A pointer takes two registers for the whole
        loop where the index arithmetic it replaces keeps one 32-bit invariant. So only loops
        with no loop inside them and no runtime loop around them get pointers: grid-stride and
        other flat loops. Around inner loops, or inside a loop whose carried state is live
        across them, ptxas answered with spills. The shipped a03 went from 144 to 524
        spilled bytes, and with unrolling off from none to 992; its time grew from 236 to
        304 µs. The shipped a01 with unrolling off ran faster all the same (108 to 76 µs),
        but not by a rule that tells the two apart."""
        if self.k._loops or any(isinstance(st, Loop | StridedLoop) for st in walk(s.body)):
            return None
        return i

    def _counted(self, s: Loop | StridedLoop, start: Aff, n: int, m: int, f: int,
                 written: list[str]) -> None:
        """A bottom-tested loop over the axis itself, from ``start`` while below
        ``start + m*n``, with ``f`` copies of the body (copy j at axis + j*n, so their
        addresses share one base register and differ by immediate offsets)."""
        k = self.k
        srng = start.range(k.ranges)
        rng = (srng[0], srng[1] + (m - f) * n) if srng else None
        mult = math.gcd(math.gcd(start.var_mult(k.mult), start.const), n * f)
        bound = start + m * n
        bound_op = index.operand(k, bound)
        i, top, done, enters = self._loop_head(start, bound, rng, mult)
        if enters is False:
            return
        if enters is not True:
            k.emit("bra", src=(done,), pred=f"!{enters}", barrier=True)
        with k.loop(entered=enters is True, counter=self._iv_counter(s, i), step=n * f) as mark:
            k.place(top)
            top_label = k.body[-1]
            for reg in written:
                k.forget(reg)
            for j in range(f):
                with self._block():
                    self.env[s.axis.name] = Aff.of(i) + j * n
                    self.body(s.body)
        k.ranges.pop(i, None)
        again = k.reg("pred")
        for ptr, delta in mark.incs:
            k.emit("add.s64", (ptr,), (ptr, str(delta)))
        k.emit("add.u32", (i,), (i, str(n * f)))
        k.emit("setp.lt.s32", (again,), (i, bound_op))
        k.emit("bra", src=(top,), pred=again, barrier=True)
        rows = self._warp_rows(start, enters, mark)
        if rows:
            pre = Ins(text="")  # where the preheader ends, for the staging pass
            k.body.insert(mark.at, pre)
            k.markers.append(pre)
            k.stages.append(Stage(pre, top_label, k.body[-1], rows))
        k.place(done)

    def _lane_contiguous(self, start: Aff) -> bool:
        """Whether every thread of the block runs this code together, in a grid of several waves,
        and a loop starting at ``start`` gives a warp's lanes consecutive values from a 32-aligned
        first one: ``tid`` plus block-uniform terms that are multiples of 32. In a grid of one
        wave an SM holds too few warps to cover a staged trip's round of loads, stores and warp
        syncs: the shipped r02 (one block) took 26.7 us staged against 14.3 unrolled."""
        if not self._converged or self.k._loops or self.block % 32 or self.k.min_ctas == 1:
            return False
        if start.terms.get(self.tid) != 1 or start.const % 32:
            return False
        return not any(r != self.tid and (r != self.ctaid or c % 32)
                       for r, c in start.terms.items())

    def _stageable(self, s: Loop | StridedLoop, start: Aff, stmts: Sequence[Stmt]) -> bool:
        """Whether this loop's loads are warp rows the staging pass could fetch wide: loads of
        4-byte global elements at the loop's own axis, from a lane-contiguous start, in a body of
        loads, assignments and accumulations only (and CSE on, for its induction pointers)."""
        if self.k.no_cse or not self._lane_contiguous(start):
            return False
        loads = [st for st in stmts if isinstance(st, Load)]
        if not loads or not all(isinstance(st, Load | Assign | Accum) for st in stmts):
            return False
        for st in loads:
            mem = self.mem.get(st.input)
            if (not isinstance(mem, GlobalBuf) or len(st.index) != 1 or len(st.names) != 1 or
                    st.index[0] != Var(s.axis.name) or size(mem_type(mem.dtype)) != 4):
                return False
        return True

    def _warp_rows(self, start: Aff, enters: Any, mark: Any) -> dict[str, int]:
        """The induction pointers of a counted loop through which each warp reads one contiguous
        row of 4-byte elements per load, with their per-trip steps; empty unless every thread of
        the block runs every trip together. A pointer qualifies when the loop starts at ``tid``
        plus block-uniform terms that keep a warp's first element 32-element aligned, and the
        pointer steps the counter with coefficient 1 over 4-byte elements and nothing else."""
        k = self.k
        if enters is not True or not self._lane_contiguous(start):
            return {}
        return {p: d for p, d in mark.incs if k.iv_meta.get(p) == (1, 4, ())}

    def _runtime_loop(self, s: Loop | StridedLoop, start: Aff, step: Aff, end: Aff,
                      written: list[str]) -> None:
        k = self.k
        srng, erng = start.range(k.ranges), end.range(k.ranges)
        rng = (srng[0], erng[1] - 1) if srng and erng else None
        mult = 1
        if step.is_const:
            mult = math.gcd(math.gcd(start.var_mult(k.mult), start.const), step.const)
        step_op, end_op = index.operand(k, step), index.operand(k, end)
        i, top, done, enters = self._loop_head(start, end, rng, mult)
        if enters is False:
            return
        if enters is not True:
            k.emit("bra", src=(done,), pred=f"!{enters}", barrier=True)
        const_step = step.const if step.is_const else 0
        with k.loop(entered=enters is True, counter=self._iv_counter(s, i),
                    step=const_step) as mark:
            k.place(top)
            top_label = k.body[-1]
            for reg in written:
                k.forget(reg)
            with self._block():
                self.env[s.axis.name] = Aff.of(i)
                self.body(s.body)
        prefetch = self._prefetch_ahead(mark, top_label, i, const_step, end_op)
        pre = Ins(text="")  # where the preheader ends, for the load pipeline pass
        k.body.insert(mark.at, pre)
        k.ranges.pop(i, None)
        again = k.reg("pred")
        for ptr, delta in mark.incs:
            k.emit("add.s64", (ptr,), (ptr, str(delta)))
        k.emit("add.u32", (i,), (i, step_op))
        k.emit("setp.lt.s32", (again,), (i, end_op))
        k.emit("bra", src=(top,), pred=again, barrier=True)
        if k.min_ctas == 1 and const_step > 0 and mark.incs:
            # a single-wave loop's trips wait on their own loads: issue them trips ahead
            k.pipes.append(Pipe(pre, top_label, k.body[-1], i, const_step, end_op,
                                dict(mark.incs), prefetch))
        k.markers.append(pre)
        k.place(done)

    def _prefetch_ahead(self, mark: Any, top_label: Any, i: str, step: int, end_op: str
                        ) -> list[Ins]:
        """In a single-wave kernel a runtime loop's trips wait on their own loads: one body per
        trip, each load feeding that trip's arithmetic, and too few warps per SM to cover the
        latency. So each read-only global load that walks an induction pointer is prefetched
        into L1 ``PREFETCH_TRIPS`` trips ahead, at the top of the body, where the counter then
        stands; the trip's own load then finds its line in L1. The prefetch is predicated on
        that trip existing, so it never reaches past the loop's end. It moves no data into
        registers and changes no result. Returns the inserted code (the load pipeline pass
        removes it where its copies cover the same loads)."""
        k = self.k
        if k.min_ctas != 1 or step <= 0 or not mark.incs:
            return []
        start = next(n for n, ins in enumerate(k.body) if ins is top_label)
        loaded = {ins.mem.addr for ins in k.body[start:]
                  if ins.mem is not None and ins.mem.kind == "ld" and ins.mem.space == "global.nc"}
        streams = [(ptr, delta) for ptr, delta in mark.incs if ptr in loaded]
        if not streams:
            return []
        ahead, exists = k.reg("u32"), k.reg("pred")
        code = [Ins("add.u32", (ahead,), (i, str(PREFETCH_TRIPS * step))),
                Ins("setp.lt.s32", (exists,), (ahead, end_op))]
        code += [Ins("prefetch.global.L1", (), (f"[{ptr}+{PREFETCH_TRIPS * delta}]",), exists)
                 for ptr, delta in streams]
        k.body[start + 1:start + 1] = code
        return code

    def _trips(self, start: Aff, step: Aff, end: Aff, stmts: Sequence[Stmt]
               ) -> tuple[int, int] | None:
        """(trips every thread runs, trips some thread runs) for a constant positive step and
        end, when the two differ by at most one; a body with a barrier needs them equal (every
        thread on every trip). Otherwise None: the loop runs as a runtime loop."""
        first = start.range(self.k.ranges)
        if first is None or not (step.is_const and step.const > 0 and end.is_const):
            return None

        def count(from_value: int) -> int:  # trips from an axis value: ceil((end - v) / step)
            return max(0, -((from_value - end.const) // step.const))

        fewest, most = count(first[1]), count(first[0])
        if most - fewest > 1:
            return None
        if fewest != most and any(isinstance(st, BARRIERS) for st in stmts):
            return None
        return fewest, most

    def _cost(self, body: Sequence[Stmt]) -> int:
        """Estimated PTX instructions of one pass over ``body``."""
        c = 0
        for st in body:
            if isinstance(st, Load):
                c += 1 + len(st.names)
            elif isinstance(st, Write):
                c += 2 + len(st.values)
            elif isinstance(st, Assign):
                c += 6 if ops.canonical(st.op.name) in fastmath.F32_FUNCS else 1
            elif isinstance(st, Cond):
                c += 2 + self._cost(st.body) + self._cost(st.else_body)
            elif isinstance(st, Loop | StridedLoop):
                inner = self._cost(st.body)
                trips = st.axis.extent.as_static() if st.axis.extent.is_static else 8
                if isinstance(st, StridedLoop):
                    step = st.step.value if isinstance(st.step, Literal) else st.step
                    trips = -(-trips // step) if isinstance(step, int) and step > 0 else 8
                c += inner * trips if inner * trips <= UNROLL_BUDGET else inner * NESTED_COPIES
            elif isinstance(st, WarpShuffle):
                c += 3 * len(st.state) * max(1, st.length.bit_length() - 1)
            elif isinstance(st, TreeHalve):
                c += 6 * len(st.state) * max(1, st.length.bit_length() - 1)
            else:
                c += 1
        return c

    # --- expressions ------------------------------------------------------------------
    # An expression evaluates to an index (``Aff``), data (``Val``), or a ``bool`` for a
    # predicate the index facts decide. Each Expr class has its own method (``_EXPR``).

    def expr(self, e: Expr) -> Value:
        method = _EXPR.get(type(e))
        if method is None:
            raise NotImplementedError(f"expression {e!r}")
        return method(self, e)

    def _expr_var(self, e: Var) -> Value:
        return self._lookup(e.name)

    def _expr_literal(self, e: Literal) -> Value:
        if e.dtype == "bool" or isinstance(e.value, bool):
            return bool(e.value)
        if e.dtype == "int" or isinstance(e.value, int):
            return Aff.k(int(e.value))
        return Val(ops.const(self.k, float(e.value), "f32"), "f32")

    def _expr_ternary(self, e: TernaryExpr) -> Value:
        p = self._pred(e.cond)
        if isinstance(p, bool):
            return self.expr(e.if_true if p else e.if_false)
        yes, no = self.expr(e.if_true), self.expr(e.if_false)
        if isinstance(yes, Aff) and isinstance(no, Aff):
            return index.select(self.k, p, yes, no)
        vy, vn = self._as_val(yes), self._as_val(no)
        dtype = vy.dtype if vy.dtype == vn.dtype else "f32"
        ry = ops.convert(self.k, vy, dtype).reg
        rn = ops.convert(self.k, vn, dtype).reg
        return ops.select(self.k, p, ry, rn, dtype)

    def _expr_call(self, e: FuncCallExpr) -> Value:
        args = [self._value(a, "f32") for a in e.args]
        return ops.apply(self.k, e.name, args, "f32")

    def _expr_cast(self, e: CastExpr) -> Value:
        if e.dtype != "float":
            raise NotImplementedError(f"expression {e!r}")
        return self._value(e.expr, "f32")

    def _expr_binary(self, e: BinaryExpr) -> Value:
        if e.op in ("&&", "||"):
            return self._logical(e.op, self._pred(e.left), self._pred(e.right))
        left, right = self.expr(e.left), self.expr(e.right)
        if isinstance(left, Aff) and isinstance(right, Aff):
            return self._index_binary(e, left, right)
        x = ops.convert(self.k, self._as_val(left), "f32")
        y = ops.convert(self.k, self._as_val(right), "f32")
        if e.op in ops.CMP_SYMBOL:
            return Val(self.k.pure(f"setp.{ops.CMP_SYMBOL[e.op]}.f32", "pred", x.reg, y.reg),
                       "bool")
        if e.op not in F32_SYMBOL:
            raise NotImplementedError(f"f32 expression {e!r}")
        return ops.apply(self.k, F32_SYMBOL[e.op], [x, y], "f32")

    def _logical(self, op: str, pa: str | bool, pb: str | bool) -> Value:
        """``pa && pb`` / ``pa || pb``. A decided side either settles the result (false for
        ``&&``, true for ``||``) or leaves the other side as the result."""
        if isinstance(pa, str) and isinstance(pb, str):
            opcode = "and.pred" if op == "&&" else "or.pred"
            return Val(self.k.pure(opcode, "pred", pa, pb), "bool")
        settles = op == "||"
        known, other = (pa, pb) if isinstance(pa, bool) else (pb, pa)
        result = known if known == settles else other
        return result if isinstance(result, bool) else Val(result, "bool")

    def _index_binary(self, e: BinaryExpr, a: Aff, b: Aff) -> Value:
        k = self.k
        if e.op in ops.CMP_SYMBOL:
            p = index.compare(k, e.op, a, b)
            return p if isinstance(p, bool) else Val(p, "bool")
        fold = _INDEX_OPS.get(e.op)
        if fold is None:
            raise NotImplementedError(f"index expression {e!r}")
        return fold(k, a, b)

    def _as_val(self, v: Value) -> Val:
        """Any value as data: an index as an i32 register, a decided bool as a predicate."""
        if isinstance(v, Val):
            return v
        k = self.k
        if isinstance(v, bool):
            word = index.reg_of(k, Aff.k(1 if v else 0))
            return Val(k.pure("setp.ne.u32", "pred", word, "0"), "bool")
        return Val(index.reg_of(k, v), "i32")

    def _value(self, e: Expr, dtype: str) -> Val:
        """Expression ``e`` as data of ``dtype``; a number literal becomes a constant of that
        type directly."""
        numeric = isinstance(e, Literal) and e.dtype != "bool" and not isinstance(e.value, bool)
        if numeric:
            return Val(ops.const(self.k, float(e.value), reg_type(dtype)), dtype)
        return ops.convert(self.k, self._as_val(self.expr(e)), dtype)

    def _int(self, e: Expr) -> Aff:
        """Expression ``e`` as an index. Integer data in a variable is copied out first: the
        index may be used after the variable changes."""
        v = self.expr(e)
        if isinstance(v, Aff):
            return v
        if isinstance(v, bool) or not is_int(v.dtype):
            raise NotImplementedError(f"index expression {e!r} is not an integer")
        k = self.k
        reg = ops.convert(k, v, "i32").reg
        if reg in k.variables:
            snapshot = k.reg("u32")
            k.emit("mov.b32", (snapshot,), (reg,))
            reg = snapshot
        return Aff.of(reg)

    def _pred(self, e: Expr) -> str | bool:
        """Expression ``e`` as a predicate register, or a bool when it is decided here; an index
        is true where it is nonzero."""
        v = self.expr(e)
        if isinstance(v, bool):
            return v
        if isinstance(v, Aff):
            return index.compare(self.k, "!=", v, Aff())
        return ops.convert(self.k, v, "bool").reg

def _expressions_of(st: Stmt) -> Iterator[Expr]:
    """Every expression a statement holds directly (nested statements' bodies excluded), with
    all of their subexpressions."""
    pending: list[object] = [getattr(st, f) for f in getattr(st, "__dataclass_fields__", {})
                             if f not in ("body", "else_body")]
    while pending:
        item = pending.pop()
        if isinstance(item, tuple):
            pending.extend(item)
        elif isinstance(item, Expr):
            yield item
            pending.extend(getattr(item, f) for f in getattr(item, "__dataclass_fields__", {}))


# statement class -> the Lowering method that emits it (``emit_<ClassName>``)
_HANDLERS: dict[type, str] = {
    cls: f"emit_{cls.__name__}" for cls in (
        Accum, Assign, Cond, CpAsyncCommit, CpAsyncCopy, CpAsyncWait, Init, Let, Load, Loop,
        Select, Smem, StridedLoop, Sync, Tile, TreeHalve, WarpShuffle, Write)
    if hasattr(Lowering, f"emit_{cls.__name__}")}


def _raster_pair(t: Tile) -> tuple[int, int, int] | None:
    """(grouped axis, other axis, group size) when the Tile orders a pair of adjacent block
    axes in raster groups, else None. ``raster_orient`` "m" groups the first axis of
    ``raster_axes``, otherwise the second; a group of one, or a grouped axis of extent one,
    leaves plain row-major order."""
    names = [a.name for a in t.axes]
    wanted = t.raster_axes or ()
    if not t.raster_group or not wanted or any(n not in names for n in wanted):
        return None
    first, second = (names.index(n) for n in wanted)
    if second != first + 1:
        return None
    grouped, other = (first, second) if t.raster_orient == "m" else (second, first)
    size = min(t.raster_group, t.extents[grouped])
    if t.extents[grouped] <= 1 or size <= 1:
        return None
    return grouped, other, size


# the red.global.add type of each buffer dtype an atomic Write can add into
_RED_ADD = {"f32": "f32", "f64": "f64", "f16": "noftz.f16", "bf16": "noftz.bf16",
            "i32": "s32", "u32": "u32", "u64": "u64", "i64": "u64"}


def _row_major(buf: str, shape: tuple[int, ...], parts: Sequence[Aff]) -> Aff:
    """The row-major element offset of ``buf[parts]``: a single index is already flat;
    otherwise one index per axis, each scaled by the product of the extents after it."""
    if len(parts) < 2:
        return parts[0] if parts else Aff()
    if len(parts) != len(shape):
        raise NotImplementedError(f"{buf}: {len(parts)}-d index into a {len(shape)}-d buffer")
    scales = [math.prod(shape[i + 1:]) for i in range(len(shape))]
    return Aff.combine(*zip(parts, scales, strict=True))


# index arithmetic of a binary expression over two indices
_INDEX_OPS = {"+": lambda k, a, b: a + b, "-": lambda k, a, b: a - b, "*": index.mul,
              "/": index.div, "//": index.div, "%": index.mod}

# Expr class -> the Lowering method that evaluates it
_EXPR = {Var: Lowering._expr_var, Literal: Lowering._expr_literal,
         BinaryExpr: Lowering._expr_binary, TernaryExpr: Lowering._expr_ternary,
         FuncCallExpr: Lowering._expr_call, CastExpr: Lowering._expr_cast}


def _shuffle_problem(s: WarpShuffle) -> Exception | None:
    """Why this lowering cannot take the shuffle, or None."""
    if getattr(s, "prefix", False):
        return NotImplementedError("WarpShuffle: prefix (shfl.up) form")
    n = s.length
    if n < 2 or n > 32 or n & (n - 1):
        return ValueError(f"WarpShuffle: length {n} is not a power of two in [2, 32]")
    if len(s.state) != len(s.state_b):
        return ValueError("WarpShuffle: state and state_b differ in length")
    return None


_SHARED_DTYPES = frozenset({"f32", "f64", "f16", "bf16", "i32", "u32", "i64", "u64"})


def _state_written(st: Stmt) -> Sequence[str]:
    """Names a statement writes in place: an accumulator, a reduction's state."""
    if isinstance(st, Accum):
        return (st.name,)
    if isinstance(st, WarpShuffle | TreeHalve):
        return tuple(st.state)
    return ()


def _tree_problem(s: TreeHalve) -> Exception | None:
    """Why this lowering cannot take the halving tree, or None."""
    n = s.length
    if n < 2 or n & (n - 1):
        return ValueError(f"TreeHalve: length {n} is not a power of two >= 2")
    if len({len(s.bufs), len(s.state), len(s.state_b)}) != 1:
        return ValueError("TreeHalve: bufs, state and state_b differ in length")
    return None

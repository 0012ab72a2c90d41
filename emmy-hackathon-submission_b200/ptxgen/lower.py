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
from .ptx import BUFFER_ALIGN, SM_COUNT, Kernel, pow2_part

UNROLL_BUDGET = 6144  # instructions a loop may fully unroll to
BODY_BUDGET = 768  # instructions the copies in one trip of a partly unrolled loop may hold
MAX_COPIES = 16
NESTED_COPIES = 2
STATIC_SMEM_CAP = 48 * 1024  # past this, shared buffers live in one dynamic pool
MAX_IMM_OFFSET = 1 << 30  # larger constant byte offsets are added into the address register
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
        self._order = {id(st): i for i, st in enumerate(walk([op.body]))}
        self._stmts = list(walk([op.body]))

    # --- walking ----------------------------------------------------------------------
    def run(self) -> Kernel:
        k = self.k
        for name in k.params:
            if name not in self.buffers:
                raise ValueError(f"parameter {name!r} has no buffer")
            raw = k.reg("u64")
            k.emit("ld.param.u64", (raw,), (f"[{k.name}_param_{name}]",))
            buf = self.buffers[name]
            ptr = k.pure("cvta.to.global.u64", "u64", raw)
            k.align[ptr] = BUFFER_ALIGN
            self.mem[name] = GlobalBuf(tuple(buf.shape), buf.dtype, ptr, buf.is_output)
        self.tid = k.pure("mov.u32", "u32", "%tid.x", rng=(0, self.block - 1))
        self.ctaid = k.pure("mov.u32", "u32", "%ctaid.x")
        if any(isinstance(st, WarpShuffle | TreeHalve) for st in self._stmts) or any(
                isinstance(e, Var) and e.name in ("lane", "warp") for e in self._all_exprs()):
            lane = k.pure("and.b32", "u32", self.tid, "31", rng=(0, min(31, self.block - 1)))
            warp = k.pure("shr.u32", "u32", self.tid, "5", rng=(0, (self.block - 1) >> 5))
            self.env |= {"lane": Aff.of(lane), "warp": Aff.of(warp)}
        self.mem |= self._declare_shared(list(self.op.smem_buffers.values()))
        self.body([self.op.body])
        return k

    def _all_exprs(self) -> Iterator[Expr]:
        def sub(e: object) -> Iterator[Expr]:
            if isinstance(e, Expr):
                yield e
                for f in getattr(e, "__dataclass_fields__", {}):
                    yield from sub(getattr(e, f))
            elif isinstance(e, tuple):
                for x in e:
                    yield from sub(x)

        for st in self._stmts:
            for f in getattr(st, "__dataclass_fields__", {}):
                if f not in ("body", "else_body"):
                    yield from sub(getattr(st, f))

    def body(self, stmts: Sequence[Stmt]) -> None:
        for st in stmts:
            fn = getattr(self, f"emit_{type(st).__name__}", None)
            if fn is None:
                raise NotImplementedError(f"no PTX lowering for Kernel IR node {type(st).__name__}")
            fn(st)

    @contextmanager
    def _block(self) -> Iterator[None]:
        """Names first bound inside end with it (rebinding an outer name persists)."""
        before = set(self.env)
        yield
        for name in set(self.env) - before:
            del self.env[name]

    def _where(self, p: str | bool) -> AbstractContextManager[None]:
        """A block that runs only where predicate ``p`` holds (always when ``p`` is True)."""
        return nullcontext() if p is True else self.k.skip_if(f"!{p}")

    # --- names ------------------------------------------------------------------------
    def _lookup(self, name: str) -> Value:
        if name not in self.env:
            raise KeyError(f"{name!r} is used before it is defined")
        return self.env[name]

    def _data(self, name: str) -> Val:
        return self._as_val(self._lookup(name))

    def _define(self, name: str, v: Val) -> None:
        """Bind ``name`` to ``v``; a name never aliases a variable, so one is copied first."""
        if v.reg in self.k.variables:
            typ = reg_type(v.dtype)
            copy = self.k.reg(typ)
            self.k.emit(f"mov.{move_type(typ)}", (copy,), (v.reg,))
            v = Val(copy, v.dtype)
        self.env[name] = v

    def _init(self, name: str, identity: float | None, dtype: str) -> None:
        if identity is None:
            raise ValueError(f"{name!r} has no identity to start from")
        typ = reg_type(dtype)
        self.env[name] = Val(self.k.variable(typ, literal(identity, typ)), dtype)

    def _variable(self, name: str, dtype: str | None = None) -> Val:
        """Make ``name``'s value a variable (of ``dtype``) so it can be written in place."""
        v = self._data(name)
        if dtype is not None and v.dtype != dtype:
            v = ops.convert(self.k, v, dtype)
        if v.reg not in self.k.variables:
            v = Val(self.k.variable(reg_type(v.dtype), v.reg), v.dtype)
            self.env[name] = v
        return v

    def _write(self, name: str, v: Val) -> None:
        """Write ``v`` into variable ``name`` in place."""
        var = self._variable(name)
        src = ops.convert(self.k, v, var.dtype).reg
        if src != var.reg:
            self.k.emit(f"mov.{move_type(reg_type(var.dtype))}", (var.reg,), (src,))
            self.k.forget(var.reg)

    # --- launch -----------------------------------------------------------------------
    def emit_Tile(self, t: Tile) -> None:
        if not t.is_static_grid or t.aux_threads:
            raise NotImplementedError("Tile: only static grids without an aux thread band")
        n, k = t.n_elements, self.k
        if n > 2**31 - 1:
            raise NotImplementedError("Tile: more than 2^31 - 1 cells")
        if t.block_threads is not None and t.block_threads != self.block:
            raise ValueError(f"Tile block_threads {t.block_threads} != launch block {self.block}")
        blocks = -(-n // self.block)
        k.ranges[self.ctaid] = (0, blocks - 1)
        k.header_notes.append(f"// @ptxgen launch grid={blocks} block={self.block}")
        if blocks <= SM_COUNT:
            # One wave: no SM ever holds a second CTA, so ptxas may spend the whole register file
            # on one. Left to its occupancy heuristic, a long unrolled block can come out at 32
            # registers and kilobytes of spills.
            k.min_ctas = 1
        gid = Aff.of(self.ctaid) * self.block + Aff.of(self.tid)
        past = index.compare(k, ">=", gid, Aff.k(n))
        if past is True:
            return
        if past is not False and any(isinstance(st, BARRIERS) for st in walk(t.body)):
            raise NotImplementedError("Tile: a partial last block around a barrier")
        with k.skip_if(past) if past else nullcontext(), self._block():
            self.env |= self._decode(t, gid, self._raster(t))
            self.body(t.body)
        if self.exchange is not None:  # every thread reaches it, past the tail guard
            from .templates.exchange import emit_epilogue

            # whichever thread added the block's share, it happens before thread 0's release
            k.emit("bar.sync", src=("0",), barrier=True)
            emit_epilogue(k, self.tid, self.mem[self.exchange].ptr)

    def emit_Sync(self, s: Sync) -> None:
        if s.warp:
            if s.barrier_id:
                raise ValueError("Sync(warp=True) cannot carry a named barrier_id")
            self.k.emit("bar.warp.sync", src=("-1",), barrier=True)
        elif s.barrier_id == 0 and s.count is None:
            self.k.emit("bar.sync", src=("0",), barrier=True)
        elif s.count is None:
            raise ValueError(f"Sync(barrier_id={s.barrier_id}) requires count")
        else:
            self.k.emit("bar.sync", src=(str(s.barrier_id), str(s.count)), barrier=True)

    @staticmethod
    def _raster(t: Tile) -> tuple[int, int, int] | None:
        """(grouped axis, other axis, group) when the Tile orders its block axes in groups."""
        names = [a.name for a in t.axes]
        if not (t.raster_group and t.raster_axes and all(n in names for n in t.raster_axes)):
            return None
        mi, ni = (names.index(n) for n in t.raster_axes)
        if ni != mi + 1:
            return None
        gi, oi = (mi, ni) if t.raster_orient == "m" else (ni, mi)
        g = min(t.raster_group, t.extents[gi])
        return (gi, oi, g) if t.extents[gi] > 1 and g > 1 else None

    def _decode(self, t: Tile, gid: Aff, raster: tuple[int, int, int] | None) -> dict[str, Aff]:
        """Each axis from the global id, row-major (the outermost axis takes no %). A raster
        pair, grouped axis a (extent Ea, group G) beside axis b (Eb), is decoded in grouped
        order: a = grp*G + (s % (G*Eb)) % gsz and b = (s % (G*Eb)) / gsz, where gsz is G except
        in a ragged last group (Ea - grp*G)."""
        k = self.k
        extents = list(t.extents)
        strides = [math.prod(extents[i + 1:]) for i in range(len(extents))]
        axes: dict[str, Aff] = {}
        for i, (axis, e) in enumerate(zip(t.axes, extents, strict=True)):
            if raster is not None and i in raster[:2]:
                continue
            v = Aff() if e == 1 else index.div(k, gid, strides[i])
            axes[axis.name] = index.mod(k, v, e) if i and e > 1 else v
        if raster is None:
            return axes
        gi, oi, g = raster
        ea, eb = extents[gi], extents[oi]
        sub = index.div(k, gid, strides[max(gi, oi)])
        if min(gi, oi):
            sub = index.mod(k, sub, ea * eb)
        if eb == 1:
            a, b = sub, Aff()
        else:
            grp, r = index.div(k, sub, g * eb), index.mod(k, sub, g * eb)
            gsz: Aff = Aff.k(g)
            if ea % g:
                gsz = index.minimum(k, Aff.k(ea) - grp * g, gsz)
            a = grp * g + index.mod(k, r, gsz)
            b = index.div(k, r, gsz)
        axes[t.axes[gi].name], axes[t.axes[oi].name] = a, b
        return axes

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

    def emit_Load(self, s: Load) -> None:
        mem = self.mem[s.input]
        dtype = s.dtype.name if s.dtype is not None else mem.dtype
        flat = self._flat(s.input, mem.shape, [self._int(e) for e in s.index])
        vals = self._load(mem, flat, dtype, len(s.names))
        for name, v in zip(s.names, vals, strict=True):
            self.env[name] = v

    def emit_Write(self, s: Write) -> None:
        if s.swizzle != "NONE":
            raise NotImplementedError(f"Write: swizzle {s.swizzle}")
        k, mem = self.k, self.mem[s.output]
        flat = self._flat(s.output, mem.shape, [self._int(e) for e in s.index])
        values = [self._data(v) for v in s.values]
        if not s.atomic:
            self._store(mem, flat, values)
            return
        if isinstance(mem, SharedBuf):
            raise NotImplementedError("Write: atomic to shared memory")
        forms = {"f32": "f32", "f64": "f64", "f16": "noftz.f16", "bf16": "noftz.bf16",
                 "i32": "s32", "u32": "u32", "u64": "u64", "i64": "u64"}
        if mem.dtype not in forms:
            raise NotImplementedError(f"Write: atomic add of {mem.dtype}")
        addr, off, space = self._address(mem, flat, mem.dtype)
        esz = size(mem_type(mem.dtype))
        for j, v in enumerate(values):
            r = ops.convert(k, v, mem.dtype).reg
            k.mem("red", "global", forms[mem.dtype], addr, off + j * esz, (r,))

    def emit_CpAsyncCopy(self, s: CpAsyncCopy) -> None:
        if s.swizzle != "NONE":
            raise NotImplementedError(f"CpAsyncCopy: swizzle {s.swizzle}")
        if s.nbytes not in (4, 8, 16):
            raise ValueError(f"CpAsyncCopy: nbytes {s.nbytes} is not 4, 8 or 16")
        k, dst, src = self.k, self.mem[s.smem], self.mem[s.src]
        idx: tuple[Expr, ...] = s.smem_index
        if s.lane_index is not None:
            idx = tuple(BinaryExpr("+", b, ln) for b, ln in zip(idx, s.lane_index, strict=True))
        flat = self._flat(s.smem, dst.shape, [self._int(e) for e in idx])
        d_addr, d_off, _ = self._address(dst, flat, dst.dtype)
        flat = self._flat(s.src, src.shape, [self._int(e) for e in s.src_index])
        s_addr, s_off, _ = self._address(src, flat, src.dtype)
        cache = "cg" if s.nbytes == 16 else "ca"
        k.raw(f"cp.async.{cache}.shared.global [{d_addr}+{d_off}], [{s_addr}+{s_off}], "
              f"{s.nbytes};")

    def emit_CpAsyncCommit(self, _s: CpAsyncCommit) -> None:
        self.k.raw("cp.async.commit_group;")

    def emit_CpAsyncWait(self, s: CpAsyncWait) -> None:
        self.k.raw(f"cp.async.wait_group {s.group};")

    def _declare_shared(self, decls: list[Smem]) -> dict[str, SharedBuf]:
        """Static ``.shared`` arrays, or offsets into one dynamic pool past the static cap."""
        k = self.k
        offsets, total = pack_shared(decls)
        pool = total > STATIC_SMEM_CAP
        out: dict[str, SharedBuf] = {}
        if pool:
            align = max(16, *(int(s.align or 0) for s in decls))
            k.module_decls.append(f".extern .shared .align {align} .b8 smem_pool[];\n")
            k.header_notes.append(f"// @ptxgen dynamic_smem={total}")
        for s in decls:
            dtype = smem_dtype(s.dtype)
            if dtype not in ("f32", "f64", "f16", "bf16", "i32", "u32", "i64", "u64"):
                raise NotImplementedError(f"Smem: dtype {s.dtype}")
            if s.name in self.buffers:
                raise ValueError(f"Smem {s.name!r}: name already declared")
            shape, esz = tuple(int(e) for e in s.extents), size(mem_type(dtype))
            align = max(16, int(s.align or 0), esz)
            if pool:
                base = k.pure("mov.u32", "u32", "smem_pool", mult=16)
                out[s.name] = SharedBuf(shape, dtype, base, offsets[s.name], 16)
                continue
            sym = f"smem_{s.name}"
            k.shared_decls.append(f"\t.shared .align {align} .b8 {sym}[{math.prod(shape) * esz}];")
            out[s.name] = SharedBuf(shape, dtype, k.pure("mov.u32", "u32", sym), 0, align)
            k.align[out[s.name].base] = align
        return out

    @staticmethod
    def _flat(buf: str, shape: tuple[int, ...], parts: list[Aff]) -> Aff:
        """Row-major element offset of ``buf[parts]``; a single index is already flat."""
        if len(parts) <= 1:
            return parts[0] if parts else Aff()
        if len(parts) != len(shape):
            raise NotImplementedError(f"{buf}: {len(parts)}-d index into a {len(shape)}-d buffer")
        flat, stride = Aff(), 1
        for i, extent in zip(reversed(parts), reversed(shape), strict=True):
            flat, stride = flat + i * stride, stride * extent
        return flat

    # --- data -------------------------------------------------------------------------
    def emit_Assign(self, s: Assign) -> None:
        dtype = s.dtype.name if s.dtype is not None else None
        self._define(s.name, ops.assign(self.k, s.op.name, dtype, [self._data(a) for a in s.args]))

    def emit_Let(self, s: Let) -> None:
        v = self.expr(s.value) if s.dtype is None else self._value(s.value, s.dtype.name)
        if isinstance(v, Val):
            self._define(s.name, v)
        else:
            self.env[s.name] = v

    def emit_Init(self, s: Init) -> None:
        self._init(s.name, s.identity, s.dtype.name)

    def emit_Select(self, s: Select) -> None:
        self._define(s.name, self._value(TernaryExpr(s.cond, s.if_true, s.if_false), "f32"))

    def emit_Accum(self, s: Accum) -> None:
        k, name = self.k, ops.canonical(s.op.name)
        dtype = s.dtype.name if s.dtype is not None else "f32"
        if name not in ops.ACCUM:
            raise NotImplementedError(f"Accum: op {s.op.name} is not a binary op")
        if s.name not in self.env:  # no seeding loop: start from the identity here
            self._init(s.name, s.op.identity, dtype)
        acc = self._variable(s.name, dtype).reg
        value = ops.convert(k, self._data(s.value), dtype).reg
        base = acc if s.base is None else ops.convert(k, self._data(s.base), dtype).reg
        typ = reg_type(dtype)
        if name == "add" and (fma := ops.fma_operands(k, typ, value, base)) is not None:
            k.emit(f"fma.rn.{typ}", (acc,), fma)
        elif typ == "bf16" or (typ == "f16" and name == "divide"):  # no native form: in f32
            f32 = [Val(ops.cvt(k, r, typ, "f32"), "f32") for r in (base, value)]
            k.emit(f"cvt.rn.{typ}.f32", (acc,), (ops.apply(k, name, f32, "f32").reg,))
        else:
            m = ops.ACCUM[name][0 if typ in ("f32", "f64", "f16") else 1]
            k.emit(f"{ops.arith(k, m)}.{typ}", (acc,), (base, value))
        k.forget(acc)

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
        if getattr(s, "prefix", False):
            raise NotImplementedError("WarpShuffle: prefix (shfl.up) form")
        if not 2 <= s.length <= 32 or s.length & (s.length - 1):
            raise ValueError(f"WarpShuffle: length {s.length} is not a power of two in [2, 32]")
        if len(s.state) != len(s.state_b):
            raise ValueError("WarpShuffle: state and state_b differ in length")
        k, dtype = self.k, s.dtype.name
        for st in s.state:
            self._variable(st, dtype)
        mask = k.reg("u32")
        k.emit("activemask.b32", (mask,))
        if (form := self._redux_form(s)) is not None:
            st = s.state[0]
            out = k.reg(reg_type(dtype))
            k.emit(form, (out,), (self._data(st).reg, mask))
            self._write(st, Val(out, dtype))
            return
        self._ladder(s.state, s.state_b, s.combine_states, s.length, dtype, mask)

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
        is buf[t * scale + inner]."""
        if s.length < 2 or s.length & (s.length - 1):
            raise ValueError(f"TreeHalve: length {s.length} is not a power of two >= 2")
        if not len(s.bufs) == len(s.state) == len(s.state_b):
            raise ValueError("TreeHalve: bufs, state and state_b differ in length")
        trees = [(self.mem[b], st, sb) for b, st, sb in zip(s.bufs, s.state, s.state_b,
                                                            strict=True)]
        for mem, st, _ in trees:
            self._variable(st, mem.dtype)
        t = self._int(Var(s.tid_var))
        if s.length <= 32 and s.inner is None and all(isinstance(m, SharedBuf) for m, _, _ in
                                                        trees):
            self._tree_by_shuffle(s, trees)
            if self._touched_after(s, s.bufs):
                self.emit_Sync(Sync(barrier_id=s.barrier_id, count=s.barrier_count))
            return
        self._tree_by_halving(s, trees, t)

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
        k = self.k
        scale, root = (1, Aff()) if s.inner is None else (s.inner[1], self._int(Var(s.inner[0])))
        sync = Sync(barrier_id=s.barrier_id, count=s.barrier_count)
        for half in (s.length >> i for i in range(1, s.length.bit_length())):
            mine, stride = t * scale + root, half * scale
            active = index.compare(k, "<", t, Aff.k(half))
            with self._where(active), self._block():
                for mem, st, sb in trees:
                    self._write(st, self._load(mem, mine, mem.dtype)[0])
                    self.env[sb] = self._load(mem, mine + stride, mem.dtype)[0]
                self._combine(s.combine_states, s.state)
                for mem, st, _ in trees:
                    self._store(mem, mine, [self._data(st)])
            self.emit_Sync(sync)
        for mem, st, _ in trees:
            self._write(st, self._load(mem, root, mem.dtype)[0])

    # --- control ----------------------------------------------------------------------
    def emit_Cond(self, s: Cond) -> None:
        p = self._pred(s.cond)
        if isinstance(p, bool):
            with self._block():
                self.body(s.body if p else s.else_body)
            return
        k = self.k
        if not s.else_body:
            with self._where(p), self._block():
                self.body(s.body)
            return
        other, end = k.label("else"), k.label("endif")
        k.emit("bra", src=(other,), pred=f"!{p}", barrier=True)
        with k.region(), self._block():
            self.body(s.body)
            k.emit("bra.uni", src=(end,), barrier=True)
        k.place(other)
        with k.region(), self._block():
            self.body(s.else_body)
        k.place(end)

    def emit_Loop(self, s: Loop | StridedLoop) -> None:
        """for (axis = start; axis < end; axis += step) body. Seeds the Accums of its own body,
        then picks a shape: a runtime loop (one copy per trip) when threads run trip counts
        more than one apart, a barrier meets differing counts, or unrolling is off; otherwise
        a full unroll when it fits ``UNROLL_BUDGET``, else a counted loop of ``f`` copies per
        trip followed by the leftover trips as copies (guarded where some thread stops)."""
        k = self.k
        if isinstance(s, StridedLoop):
            step = self._int(s.step) if isinstance(s.step, Expr) else Aff.k(int(s.step))
            start = self._int(s.start)
            end = None if s.end is None else self._int(s.end)
        else:
            if getattr(s, "carries", None):
                raise NotImplementedError("Loop: carried state")
            start, step, end = Aff(), Aff.k(1), None
        if end is None:
            if not s.axis.extent.is_static:
                raise NotImplementedError(f"loop over {s.axis.name}: symbolic extent")
            end = Aff.k(s.axis.extent.as_static())

        seen: set[str] = set()
        for st in s.body:
            if not isinstance(st, Accum) or st.name in seen:
                continue
            seen.add(st.name)
            if s.seed:
                self._init(st.name, st.op.identity,
                           st.dtype.name if st.dtype is not None else "f32")
            elif st.name not in self.env:
                raise ValueError(f"Accum {st.name!r}: seed=False but no enclosing seed")

        stmts = list(walk(s.body))
        names = sorted({n for st in stmts for n in self._written(st)} & set(self.env))
        written = [self._variable(n).reg for n in names]
        for reg in written:  # whatever the loop's shape, no product of these survives into it
            k.forget(reg)

        trips = None if self.no_unroll else self._trips(start, step, end, stmts)
        self.loop_depth += 1
        try:
            if trips is None:
                self._runtime_loop(s, start, step, end, written)
                return
            lo, hi = trips
            n = step.const
            if hi <= 1:
                self._unrolled(s, start, n, end, lo, range(hi))
                return
            cost = max(1, self._cost(s.body))
            if hi * cost <= UNROLL_BUDGET or s.unroll is True and hi * cost <= 4 * UNROLL_BUDGET:
                self._unrolled(s, start, n, end, lo, range(hi))
                return
            nested = any(isinstance(st, Loop | StridedLoop) for st in stmts)
            f = NESTED_COPIES if nested else 1 << max(0, (BODY_BUDGET // cost).bit_length() - 1)
            f = max(1, min(f, MAX_COPIES, hi))
            m = lo // f * f
            if m == 0:
                self._unrolled(s, start, n, end, lo, range(hi))
                return
            self._counted(s, start, n, m, f, written)
            self._unrolled(s, start, n, end, lo, range(m, hi))
        finally:
            self.loop_depth -= 1

    emit_StridedLoop = emit_Loop

    def _unrolled(self, s: Loop | StridedLoop, start: Aff, n: int, end: Aff, lo: int,
                  trips: range) -> None:
        """Copy j of the body for each j in ``trips``, the axis at start + j*n; copies from
        ``lo`` on run only where start + j*n < end."""
        k = self.k
        for j in trips:
            p = True if j < lo else index.compare(k, "<", start + j * n, end)
            if p is False:
                break
            with self._where(p), self._block():
                self.env[s.axis.name] = start + j * n
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
        k.place(done)

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
            for reg in written:
                k.forget(reg)
            with self._block():
                self.env[s.axis.name] = Aff.of(i)
                self.body(s.body)
        k.ranges.pop(i, None)
        again = k.reg("pred")
        for ptr, delta in mark.incs:
            k.emit("add.s64", (ptr,), (ptr, str(delta)))
        k.emit("add.u32", (i,), (i, step_op))
        k.emit("setp.lt.s32", (again,), (i, end_op))
        k.emit("bra", src=(top,), pred=again, barrier=True)
        k.place(done)

    def _trips(self, start: Aff, step: Aff, end: Aff, stmts: list[Stmt]
               ) -> tuple[int, int] | None:
        """(trips every thread runs, trips some thread runs) when at most one apart; a barrier
        needs every thread on every trip. Else None."""
        rng = start.range(self.k.ranges)
        if not (step.is_const and step.const > 0 and end.is_const and rng is not None):
            return None
        n = step.const
        lo = max(0, -(-(end.const - rng[1]) // n))
        hi = max(0, -(-(end.const - rng[0]) // n))
        barrier = any(isinstance(st, BARRIERS) for st in stmts)
        if hi - lo > 1 or (barrier and lo != hi):
            return None
        return lo, hi

    @staticmethod
    def _written(st: Stmt) -> Sequence[str]:
        if isinstance(st, Accum):
            return (st.name,)
        if isinstance(st, WarpShuffle | TreeHalve):
            return tuple(st.state)
        return ()

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
    def expr(self, e: Expr) -> Value:
        """An index expression as an Aff, data as a Val, a decided predicate as a bool."""
        k = self.k
        if isinstance(e, Var):
            return self._lookup(e.name)
        if isinstance(e, Literal):
            if e.dtype == "bool" or isinstance(e.value, bool):
                return bool(e.value)
            if e.dtype == "int" or isinstance(e.value, int):
                return Aff.k(int(e.value))
            return Val(ops.const(k, float(e.value), "f32"), "f32")
        if isinstance(e, BinaryExpr):
            return self._binary(e)
        if isinstance(e, TernaryExpr):
            p = self._pred(e.cond)
            if isinstance(p, bool):
                return self.expr(e.if_true if p else e.if_false)
            a, b = self.expr(e.if_true), self.expr(e.if_false)
            if isinstance(a, Aff) and isinstance(b, Aff):
                return index.select(k, p, a, b)
            va, vb = self._as_val(a), self._as_val(b)
            dtype = va.dtype if va.dtype == vb.dtype else "f32"
            x, y = ops.convert(k, va, dtype).reg, ops.convert(k, vb, dtype).reg
            return ops.select(k, p, x, y, dtype)
        if isinstance(e, FuncCallExpr):
            return ops.apply(k, e.name, [self._value(a, "f32") for a in e.args], "f32")
        if isinstance(e, CastExpr) and e.dtype == "float":
            return self._value(e.expr, "f32")
        raise NotImplementedError(f"expression {e!r}")

    def _binary(self, e: BinaryExpr) -> Value:
        k, op = self.k, e.op
        if op in ("&&", "||"):
            pa, pb = self._pred(e.left), self._pred(e.right)
            if isinstance(pa, str) and isinstance(pb, str):
                return Val(k.pure("and.pred" if op == "&&" else "or.pred", "pred", pa, pb),
                           "bool")
            c, other = (pa, pb) if isinstance(pa, bool) else (pb, pa)
            p = other if c == (op == "&&") else c
            return p if isinstance(p, bool) else Val(p, "bool")
        a, b = self.expr(e.left), self.expr(e.right)
        if isinstance(a, Aff) and isinstance(b, Aff):
            if op in ops.CMP_SYMBOL:
                p = index.compare(k, op, a, b)
                return p if isinstance(p, bool) else Val(p, "bool")
            if op == "+":
                return a + b
            if op == "-":
                return a - b
            if op == "*":
                return index.mul(k, a, b)
            if op in ("/", "//"):
                return index.div(k, a, b)
            if op == "%":
                return index.mod(k, a, b)
            raise NotImplementedError(f"index expression {e!r}")
        x, y = (ops.convert(k, self._as_val(v), "f32") for v in (a, b))
        if op in ops.CMP_SYMBOL:
            return Val(k.pure(f"setp.{ops.CMP_SYMBOL[op]}.f32", "pred", x.reg, y.reg), "bool")
        if op in F32_SYMBOL:
            return ops.apply(k, F32_SYMBOL[op], [x, y], "f32")
        raise NotImplementedError(f"f32 expression {e!r}")

    def _as_val(self, v: Value) -> Val:
        if isinstance(v, Val):
            return v
        if isinstance(v, bool):
            one = index.reg_of(self.k, Aff.k(int(v)))
            return Val(self.k.pure("setp.ne.u32", "pred", one, "0"), "bool")
        return Val(index.reg_of(self.k, v), "i32")

    def _value(self, e: Expr, dtype: str) -> Val:
        """Expression ``e`` as data of ``dtype``; a literal is a constant of that type."""
        if isinstance(e, Literal) and e.dtype != "bool" and not isinstance(e.value, bool):
            return Val(ops.const(self.k, float(e.value), reg_type(dtype)), dtype)
        return ops.convert(self.k, self._as_val(self.expr(e)), dtype)

    def _int(self, e: Expr) -> Aff:
        """Expression ``e`` as an index; integer data is copied out of a variable first, since
        an index may outlive the variable's current value."""
        v = self.expr(e)
        if isinstance(v, Aff):
            return v
        if isinstance(v, bool) or not is_int(v.dtype):
            raise NotImplementedError(f"index expression {e!r} is not an integer")
        reg = ops.convert(self.k, v, "i32").reg
        if reg in self.k.variables:
            copy, reg = reg, self.k.reg("u32")
            self.k.emit("mov.b32", (reg,), (copy,))
        return Aff.of(reg)

    def _pred(self, e: Expr) -> str | bool:
        v = self.expr(e)
        if isinstance(v, bool):
            return v
        if isinstance(v, Aff):
            return index.compare(self.k, "!=", v, Aff())
        return ops.convert(self.k, v, "bool").reg

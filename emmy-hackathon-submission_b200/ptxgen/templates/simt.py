"""Register-blocked f32 GEMM: an f32 block-tiled matmul nest whose threads each own few outputs,
replaced by a kernel in which fewer threads each own a 4 x 4 block of C.

Why. In the nest Emmy writes for ``A @ B`` over f32 (the shipped ``m01_matmul_512``: 32 x 64
tiles of C on 512 threads), each thread accumulates a 2 x 2 block of C. Per k it reads 2 values
of A and 2 of B from shared memory for 4 FMAs: 4 bytes per FMA. Shared memory returns about
128 bytes per clock per SM, so the loads, not the FMAs, set the pace: a 32 x 64 tile over
K = 512 is 1 M FMAs, 32.8 k clocks of shared-memory data at 4 bytes each (about 16.7 us at
1965 MHz, where the generic build of m01 measured 15.8 us). A 4 x 4 block per thread reads 4 + 4
values per k for 16 FMAs: 2 bytes per FMA, half the clocks.

The kernel keeps the launch meta.json gives the nest (the same grid of CTAs, one per tile of C,
and the same threads per CTA), so a launcher that runs the IR's geometry runs it unchanged:

* every thread copies its share of each K step's A and B tiles (64 k a step where K allows) into
  a ring of ``STAGES`` shared-memory stages with ``cp.async.cg`` (16 bytes a copy), one commit
  group per stage;
* the first ``BM * BN / 16`` threads (whole warps) each own a 4 x 4 block of the CTA's tile.
  Per 4 k they read their 4 rows of A and 4 k-rows of B as 8 16-byte shared loads (8 lanes of a
  quarter warp read the same A row, a broadcast, and 128 contiguous bytes of B) and issue their
  64 FMAs as 32 ``fma.rn.f32x2``, two columns of a row each, with each A value duplicated into
  a register pair; the other warps only copy and meet the barriers;
* each owner stores its block with 4 ``st.global.v4``.

Each element of C is still one fused multiply-add chain over k = 0 .. K-1 in order, starting
from +0.0 (each lane of an ``fma.rn.f32x2`` is an ``fma.rn.f32``), the chain the nest's Accum
computes: the result is the same bit for bit as the generic
lowering's and the oracle's. The template applies only where it reduces the bytes per FMA: the
nest must give each thread fewer than 16 accumulators.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from dataclasses import dataclass

from ..ir import KernelOp
from ..lower import Buffer
from ..ptx import PTX_VERSION, TARGET
from .matmul import nest

TILE = 4  # rows and columns of C a compute thread owns
# K per stage, the largest that divides K, and stages in the ring. Measured on the shipped m01 on
# a B200 (CUDA graph of launches, bit-equal every time): 64 with 2 stages 10.7-10.9 us, 64 with 3
# or 4 stages 11.0, 32 with 3 or 4 11.7-12.0, 16 with 4 or 6 14.0-14.2, 128 with 2 or 3 16.0-16.3,
# 256 with 2 17.7-17.9; the generic nest 15.5-15.7
BK_CHOICES = (64, 32, 16, 8, 4)
STAGES = 2
STATIC_LIMIT = 48 << 10  # a ring this size or smaller is a static array: no launch setting needed


@dataclass(frozen=True)
class SimtPlan:
    entry: str
    params: tuple[str, ...]
    a: str
    b: str
    c: str
    m: int
    n: int
    k: int
    bm: int  # the CTA's tile of C: the nest's own
    bn: int
    bk: int  # K per stage
    block: int  # threads per CTA (the nest's)
    stages: int
    # owners a warp spans across a row of 4 x 4 blocks (the rest of it spans down): as many as
    # the row holds, up to 32. The shipped m01 (16 a row) took 11.7 us so and 13.3 with 8 across
    lanes_x: int
    # accumulate in fma.rn.f32x2 (two columns of a row per instruction; each lane is the same
    # fma.rn.f32), with each A value duplicated into a register pair. The shipped m01 took
    # 9.7-9.9 us so and 10.7-10.9 in scalar fma.rn.f32
    pairs: bool = True

    @property
    def grid(self) -> int:
        return (self.m // self.bm) * (self.n // self.bn)

    @property
    def owners(self) -> int:
        """Threads that own a 4 x 4 block of C."""
        return self.bm * self.bn // (TILE * TILE)

    @property
    def stage_bytes(self) -> int:
        return (self.bm + self.bn) * self.bk * 4

    @property
    def static(self) -> bool:
        """The ring fits a static shared array (else it is meta.json's dynamic shared memory)."""
        return self.stages * self.stage_bytes <= STATIC_LIMIT


def match(op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str], block: int,
          smem_bytes: int) -> SimtPlan | None:
    g = nest(op, buffers)
    if g is None or g.atomic or buffers[g.a].dtype != "f32":
        return None
    kloop = g.kloop
    if not kloop.axis.extent.is_static or kloop.axis.extent.as_static() != g.k:
        return None
    ext = [ax.extent.as_static() for ax in g.tile.axes]
    em, en = ext[g.mi], ext[g.ni]
    bm, bn = g.m // em, g.n // en
    # the Tile is exactly one CTA per tile of C, and the accumulators cover the tile once
    if g.tile.n_elements != em * en * block or g.accs * block != bm * bn:
        return None
    owners = bm * bn // (TILE * TILE)
    if bm % TILE or bn % 32 or owners % 32 or not 0 < owners < block or block % 32:
        return None
    if g.k % 4 or g.n % 4:
        return None
    # the ring is a static array, or the dynamic shared memory meta.json already gives the
    # nest, so a launcher that runs the IR's launch as it stands runs this kernel too
    room = max(STATIC_LIMIT, smem_bytes)
    for bk in BK_CHOICES:
        if g.k % bk == 0 and STAGES * (bm + bn) * bk * 4 <= room:
            break
    else:
        return None
    cols = bn // TILE
    lanes_x = min(cols, 32)
    if (bm // TILE) % (32 // lanes_x):
        return None
    return SimtPlan(op.name, tuple(arg_order), g.a, g.b, g.c, g.m, g.n, g.k, bm, bn, bk, block,
                    STAGES, lanes_x)


def emit(p: SimtPlan) -> str:
    e = p.entry
    t_count, kt_count = p.block, p.k // p.bk
    a_chunks, b_chunks = p.bm * p.bk // 4, p.bk * p.bn // 4  # 16-byte copies per stage
    a_part = p.bm * p.bk * 4  # bytes of a stage's A tile; its B tile follows
    cols = p.bn // TILE  # owners per row of blocks
    lines: list[str] = []

    def emit_(s: str) -> None:
        lines.append("\t" + s)

    emit_(f"ld.param.u64 %gp, [{e}_param_{p.a}];")
    emit_("cvta.to.global.u64 %ga, %gp;")
    emit_(f"ld.param.u64 %gp, [{e}_param_{p.b}];")
    emit_("cvta.to.global.u64 %gb, %gp;")
    emit_(f"ld.param.u64 %gp, [{e}_param_{p.c}];")
    emit_("cvta.to.global.u64 %gc, %gp;")
    emit_("mov.u32 %th, %tid.x;")
    emit_("mov.u32 %cta, %ctaid.x;")
    emit_(f"div.u32 %mt, %cta, {p.n // p.bn};")
    emit_(f"rem.u32 %nt, %cta, {p.n // p.bn};")
    emit_(f"mov.u32 %sbase, {'smem_ring' if p.static else 'smem_pool'};")
    # this thread's copies: chunk c = tid + j * threads, row c / (row chunks), 16 bytes at
    # column (c % row chunks) * 4; global pointers at stage 0, shared offsets within a stage
    copies = []
    for name, chunks, row_chunks, ld, rows_base, part in (
            ("a", a_chunks, p.bk // 4, p.k, f"%mt, {p.bm * p.k * 4}", 0),
            ("b", b_chunks, p.bn // 4, p.n, f"%nt, {p.bn * 4}", a_part)):
        emit_(f"mul.wide.u32 %gt, {rows_base};")
        emit_(f"add.s64 %g{name}0, %g{name}, %gt;")
        for j in range(-(-chunks // t_count)):
            tag = f"{name}{j}"
            emit_(f"add.u32 %c, %th, {j * t_count};")
            guard = None
            if (j + 1) * t_count > chunks:
                guard = f"%q{tag}"
                emit_(f"setp.lt.u32 {guard}, %c, {chunks};")
            emit_(f"div.u32 %row, %c, {row_chunks};")
            emit_(f"rem.u32 %col, %c, {row_chunks};")
            emit_(f"mul.lo.u32 %x, %row, {ld};")
            emit_("shl.b32 %y, %col, 2;")
            emit_("add.u32 %x, %x, %y;")
            emit_("mul.wide.u32 %gt, %x, 4;")
            emit_(f"add.s64 %p{tag}, %g{name}0, %gt;")
            emit_(f"mul.lo.u32 %x, %row, {row_chunks * 16};")
            emit_("shl.b32 %y, %col, 4;")
            emit_("add.u32 %x, %x, %y;")
            emit_(f"add.u32 %s{tag}, %x, {part};")
            copies.append((tag, guard, p.bk * 4 if name == "a" else p.bk * p.n * 4))
    tags = [c[0] for c in copies]

    def stage_copies(slot: str, exists: str | None) -> None:
        """This thread's copies of one stage into shared offset ``slot``; global pointers step
        to the next stage."""
        for tag, guard, step in copies:
            pred = exists
            if guard and exists:
                emit_(f"and.pred %pc, {guard}, {exists};")
                pred = "%pc"
            elif guard:
                pred = guard
            emit_(f"add.u32 %x, %sbase, {slot};")
            emit_(f"add.u32 %x, %x, %s{tag};")
            emit_(f"{'@' + pred + ' ' if pred else ''}cp.async.cg.shared.global [%x], "
                  f"[%p{tag}], 16;")
            emit_(f"add.s64 %p{tag}, %p{tag}, {step};")
        emit_("cp.async.commit_group;")

    for s in range(p.stages - 1):
        if s < kt_count:
            stage_copies(str(s * p.stage_bytes), None)
        else:
            emit_("cp.async.commit_group;")
    # an owner's block: rows 4 * ty, columns 4 * tx of the CTA's tile, where a warp's lanes
    # cover lanes_x blocks across and 32 / lanes_x down
    lx = p.lanes_x
    emit_(f"setp.lt.u32 %own, %th, {p.owners};")
    emit_("shr.u32 %x, %th, 5;")
    emit_("and.b32 %y, %th, 31;")
    emit_(f"div.u32 %ty, %x, {cols // lx};")
    emit_(f"mul.lo.u32 %ty, %ty, {32 // lx};")
    emit_(f"div.u32 %c, %y, {lx};")
    emit_("add.u32 %ty, %ty, %c;")
    emit_(f"rem.u32 %tx, %x, {cols // lx};")
    emit_(f"mul.lo.u32 %tx, %tx, {lx};")
    emit_(f"rem.u32 %c, %y, {lx};")
    emit_("add.u32 %tx, %tx, %c;")
    emit_(f"mul.lo.u32 %aoff, %ty, {TILE * p.bk * 4};")
    emit_(f"mul.lo.u32 %boff, %tx, {TILE * 4};")
    emit_(f"add.u32 %boff, %boff, {a_part};")
    for r in range(TILE * TILE):
        if p.pairs and r < 8:
            emit_(f"mov.b64 %acp{r}, 0;")
        elif not p.pairs:
            emit_(f"mov.f32 %acc{r}, 0f00000000;")
    emit_("mov.u32 %kt, 0;")
    emit_("mov.u32 %cur, 0;")
    emit_(f"mov.u32 %nxt, {(p.stages - 1) * p.stage_bytes};")
    lines.append("$L_k:")
    emit_(f"cp.async.wait_group {p.stages - 2};")
    emit_("bar.sync 0;")
    emit_(f"add.u32 %x, %kt, {p.stages - 1};")
    emit_(f"setp.lt.u32 %more, %x, {kt_count};")
    stage_copies("%nxt", "%more")
    ring = p.stages * p.stage_bytes
    emit_(f"add.u32 %nxt, %nxt, {p.stage_bytes};")
    emit_(f"setp.eq.u32 %wrap, %nxt, {ring};")
    emit_("@%wrap mov.u32 %nxt, 0;")
    emit_("@!%own bra.uni $L_skip;")
    emit_("add.u32 %sa, %sbase, %cur;")
    emit_("add.u32 %sb, %sa, %boff;")
    emit_("add.u32 %sa, %sa, %aoff;")
    for kk in range(0, p.bk, 4):
        for i in range(TILE):
            regs = ", ".join(f"%a{i * 4 + j}" for j in range(4))
            emit_(f"ld.shared.v4.f32 {{{regs}}}, [%sa+{(i * p.bk + kk) * 4}];")
        if p.pairs:
            for j in range(4):
                emit_(f"ld.shared.v2.b64 {{%bq{j * 2}, %bq{j * 2 + 1}}}, "
                      f"[%sb+{(kk + j) * p.bn * 4}];")
            for r in range(16):
                emit_(f"mov.b64 %ad{r}, {{%a{r}, %a{r}}};")
            for j in range(4):
                for i in range(TILE):
                    for h in range(2):
                        q = i * 2 + h
                        emit_(f"fma.rn.f32x2 %acp{q}, %ad{i * 4 + j}, %bq{j * 2 + h}, %acp{q};")
            continue
        for j in range(4):
            regs = ", ".join(f"%b{j * 4 + c}" for c in range(TILE))
            emit_(f"ld.shared.v4.f32 {{{regs}}}, [%sb+{(kk + j) * p.bn * 4}];")
        for j in range(4):
            for i in range(TILE):
                for c in range(TILE):
                    r = i * TILE + c
                    emit_(f"fma.rn.f32 %acc{r}, %b{j * 4 + c}, %a{i * 4 + j}, %acc{r};")
    lines.append("$L_skip:")
    emit_(f"add.u32 %cur, %cur, {p.stage_bytes};")
    emit_(f"setp.eq.u32 %wrap, %cur, {ring};")
    emit_("@%wrap mov.u32 %cur, 0;")
    emit_("add.u32 %kt, %kt, 1;")
    emit_(f"setp.lt.u32 %more, %kt, {kt_count};")
    emit_("@%more bra.uni $L_k;")
    emit_("cp.async.wait_all;")
    emit_("@!%own bra.uni $L_done;")
    # C rows mt * BM + 4 ty + i, columns nt * BN + 4 tx
    emit_(f"mul.lo.u32 %x, %mt, {p.bm};")
    emit_(f"mad.lo.u32 %x, %ty, {TILE}, %x;")
    emit_(f"mul.lo.u32 %y, %nt, {p.bn};")
    emit_(f"mad.lo.u32 %y, %tx, {TILE}, %y;")
    emit_(f"mad.lo.u32 %x, %x, {p.n}, %y;")
    emit_("mul.wide.u32 %gt, %x, 4;")
    emit_("add.s64 %gt, %gc, %gt;")
    for i in range(TILE):
        if p.pairs:
            emit_(f"st.global.v2.b64 [%gt+{i * p.n * 4}], {{%acp{i * 2}, %acp{i * 2 + 1}}};")
            continue
        regs = ", ".join(f"%acc{i * TILE + c}" for c in range(TILE))
        emit_(f"st.global.v4.f32 [%gt+{i * p.n * 4}], {{{regs}}};")
    lines.append("$L_done:")
    emit_("ret;")

    params = ",\n".join(f"\t.param .u64 {e}_param_{q}" for q in p.params)
    guards = [c[1] for c in copies if c[1]]
    decls = [
        "\t.reg .pred %own, %more, %wrap, %pc" + "".join(f", {g}" for g in guards) + ";",
        "\t.reg .b32 %th, %cta, %mt, %nt, %sbase, %c, %row, %col, %x, %y, %ty, %tx, %aoff, "
        "%boff, %kt, %cur, %nxt, %sa, %sb" + "".join(f", %s{t}" for t in tags) + ";",
        "\t.reg .b64 %gp, %ga, %gb, %gc, %gt, %ga0, %gb0" + "".join(f", %p{t}" for t in tags)
        + ";",
        "\t.reg .f32 %acc<16>, %a<16>, %b<16>;",
        "\t.reg .b64 %acp<8>, %ad<16>, %bq<8>;",
    ]
    smem = p.stages * p.stage_bytes
    head = [
        "//\n// Generated by ptxgen (B200 backend): register-blocked f32 GEMM template\n//",
        f"// @ptxgen launch grid={p.grid} block={p.block}",
        *([] if p.static else [f"// @ptxgen dynamic_smem={smem}"]),
        f"// @ptxgen simt m={p.m} n={p.n} k={p.k} bm={p.bm} bn={p.bn} bk={p.bk} "
        f"stages={p.stages} owners={p.owners}",
        "",
        f".version {PTX_VERSION}\n.target {TARGET}\n.address_size 64\n",
        (f".shared .align 16 .b8 smem_ring[{smem}];" if p.static else
         ".extern .shared .align 16 .b8 smem_pool[];"),
        "",
        f".visible .entry {e}(\n{params}\n)\n.maxntid {p.block}, 1, 1\n.minnctapersm 1\n{{",
        *decls,
        "",
    ]
    return "\n".join(head + lines + ["}", ""])

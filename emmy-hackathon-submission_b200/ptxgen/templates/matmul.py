"""The tcgen05 GEMM template: a matmul-shaped Kernel IR nest over bf16/f16 operands, replaced by a
persistent TMA + mbarrier + tcgen05.mma kernel with TMEM accumulators.

Matching (``match``). The nest Emmy writes for ``A @ B`` (reference
``examples/cse/m01_matmul_512/k_matmul_2967be.ir.txt``): a Tile whose block axes window the M
and N axes of C (and, for split-K, one more axis that offsets K), Init'ed f32 accumulators, two
shared buffers fed by cp.async copies of A and B tiles, one K loop whose inner loop loads from
the two shared buffers, multiplies and Accum-adds into the accumulators, and Writes of the
accumulators into C (atomic for split-K). The matcher checks these facts and the shapes
A [M, K], B [K, N], C [M, N] with K the K loop's extent times the splits; anything else keeps
the generic lowering.

The kernel (``emit``), one CTA per SM, persistent over the output tiles (``tile = ctaid +
i * nctaid``, so any grid size computes every tile once):

* warp 0, lane 0 -- TMA producer: ``cp.async.bulk.tensor`` loads of a 128 x 64 A tile and a
  64 x BN B tile (128-byte swizzled; B as BN/64 column chunks) per K step into a ring of
  ``stages`` shared-memory stages, each guarded by a ``full`` mbarrier (expect_tx bytes) and an
  ``empty`` one;
* warp 1 -- allocates TMEM (two BN-column f32 accumulators), and lane 0 issues
  ``tcgen05.mma.cta_group::1.kind::f16`` (M=128, N=BN, K=16, bf16/f16 in, f32 accumulate) from
  the stage's shared-memory descriptors, ``tcgen05.commit``s each stage back to its ``empty``
  barrier and each finished tile to the accumulator's ``tmem_full`` barrier;
* warps 4-7 -- epilogue: ``tcgen05.ld`` (32 lanes x 32 columns per load) of the finished
  accumulator; each warp writes its 32 x 32 block into one of its two shared-memory staging
  buffers (128-byte swizzled, so the stores are conflict-free), fences it to the async proxy,
  and one lane writes the whole block into C with a single TMA op (``cp.async.bulk.tensor``
  store, or ``cp.reduce.async.bulk.tensor`` add for split-K: whole 128-byte lines, where a
  per-thread ``red.global.add.v4`` touches 32 rows per instruction); then ``tmem_empty``. With
  two accumulators the epilogue of one tile overlaps the MMAs of the next. The tensor map over
  C covers this GPU's own buffer only, and no load multicasts.

The work is a table of segments baked into the module: (m tile, n tile, first K block, K-block
count), and CTA ``c`` takes entries ``c, c + nctaid, ...``. A plain GEMM has one whole-K segment
per output tile, in a grouped raster of its own (``raster``): groups of about sqrt(CTAs at once)
tile rows, rows fastest within a group, so the tiles running at one time read as few panels of A
and B as a near-square block of them can (config 5: 1.48 -> 1.13 GB of DRAM reads a launch
against the IR's groups of four pair rows, about 3% faster). A split-K GEMM (C
zeroed, partials added with ``red.global.add``) takes its own split count instead of the IR's:
the one that finishes soonest on ``SM_COUNT`` SMs, counting waves of CTAs times K blocks per
split plus ``SEGMENT_COST`` per segment for its epilogue (for 32 tiles of 1024 K blocks: 9
uneven splits, 288 segments in two full waves, where the IR's 4 splits fill 128 of 148 SMs
once). Segments go split-major, so the CTAs running at one time read the same few K windows of A
and B and share them in L2. The sum is the IR's (every K block of every tile is added once into
zeroed C); only the f32 association differs, as it does between atomic orders. The split-K
module carries its own kernel that zeroes C (``zero_kernel_ptx``, named in a ``// @ptxgen
zero`` line): the launcher runs it in place of a memset and starts the GEMM right after it with
programmatic stream serialization, and the GEMM's epilogue waits for it
(``griddepcontrol.wait``) before its first reduce-add. A plain GEMM with fewer tiles than SM
pairs may cut its tiles narrower (``MatmulPlan.columns``). Tensor maps live in module
``.global`` symbols that the launcher fills
(``pg_tensormap_fill``), named in ``// @ptxgen tensormap`` header lines, so the kernel's
parameters stay the plain device pointers of meta.json's arg_order. Every mbarrier wait is
bounded by ``%globaltimer``; a wait that runs out sets a bit of the module's ``ptxgen_status``
word, and the kernel winds down: the producer waits (bounded) for its own TMA loads to land, the
MMA thread for its MMAs, the epilogue lanes for their TMA writes, then TMEM is freed. Every CTA
loads its own tiles. At entry the kernel compares ``%dynamic_smem_size`` with what its layout
needs; a launch that granted less sets status bit ``SMEM_SHORT`` and every CTA returns before any
barrier exists.
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import dataclass

from ..ir import (Accum, Assign, BinaryExpr, CpAsyncCommit, CpAsyncCopy, Expr, Init, KernelOp,
                  Load, Loop, Smem, StridedLoop, Tile, Var, Write, walk)
from ..lower import Buffer
from ..ptx import PTX_VERSION, SM_COUNT, TARGET

BM, BK = 128, 64  # tile rows (the MMA's M) and K per stage (64 bf16 = one 128-byte swizzle row)
UMMA_K = 16
MAX_STAGES = 6
WAIT_NS = 2_000_000_000  # a bounded wait gives up after 2 s of %globaltimer
MIN_SEGMENT = 8  # K blocks a split-K segment has at least
SEGMENT_COST = 2  # a segment's epilogue, in K blocks of MMA time, when choosing the split count
EPILOGUE_WARPS = (4, 5, 6, 7)
BAR_BYTES = 8
SMEM_SHORT = 8  # status bit: the launch gave less dynamic shared memory than the layout needs
NARROW = (192, 128, 64)  # widths a mixed-width plan may cut beside whole 256-column tiles
MIXED_GAIN = 0.05  # ... used only when the cost model finishes that much sooner than whole tiles
# a pair's time for one K block of a tile of each width, against a whole tile's, measured on a
# B200 with one tile per pair (K = 8192): the loads of A and B and the pipeline around the MMAs,
# not the MMAs, set the pace of a narrow tile, so a narrower tile is barely faster
K_BLOCK_TIME = {256: 1.0, 192: 0.98, 128: 0.95, 64: 0.90}
# what cutting a tail tile costs per piece beyond the first, in K blocks of MMA time: the
# partials written and summed. Set from config 5's shares on a B200: the 1/4 share's tail in two
# pieces took 174.3 us against 184.0 for whole tiles; the 1/8 share's in four took 104.7 against
# 96.0, so four pieces must not pay
TAIL_FIXUP = 16
ROLE_WHOLE, ROLE_PIECE = 0, 1  # a work-table entry: a whole tile, or a piece of a tail tile
ZERO_GRID, ZERO_BLOCK = SM_COUNT, 256  # launch of a split-K module's kernel that zeroes C
SMEM_LIMIT = 232448  # dynamic shared memory one CTA may opt into on sm_100 (227 KiB)
STAGE_BLOCK = 32  # rows and columns of the f32 block an epilogue warp stages per TMA op
STAGE_BUF = STAGE_BLOCK * STAGE_BLOCK * 4  # 4 KiB: 32 rows of 128 bytes, 128-byte swizzled


@dataclass(frozen=True)
class MatmulPlan:
    entry: str
    params: tuple[str, ...]
    a: str
    b: str
    c: str
    dtype: str  # of A and B: bf16 | f16
    m: int
    n: int
    k: int
    bn: int
    splits: int
    block: int
    stages: int
    atomic: bool
    schedule: tuple[tuple[int, int, int], ...]  # (m tile, n tile, split) per tile index
    pair: bool = False  # two CTAs (an SM pair) per 256-row tile, cta_group::2
    # the epilogue stages each warp's 32 x 32 blocks of C in shared memory and writes them
    # with one TMA op each (a reduce-add for split-K); False: per-thread global stores/reds
    staged: bool = True
    # a plain pair GEMM may cut some tiles narrower to even out the pairs' work (``columns``);
    # False keeps whole tiles
    mixed: bool = True
    # a plain GEMM whose last wave of tiles is part full may cut those tiles along K (``tail``);
    # False keeps whole tiles
    stream_k: bool = True

    @property
    def kc(self) -> int:
        return self.k // self.splits

    @property
    def tiles(self) -> int:
        return len(self.schedule)

    @property
    def stage_bytes(self) -> int:
        return (BM * BK + BK * self.bn) * 2

    def segments(self) -> tuple[tuple[tuple[int, int, int, int], ...], int]:
        """The kernel's work table, (m tile, n tile, first K block, K blocks) per entry, and the
        grid it is laid out for."""
        kbs = self.k // BK
        rows = 2 if self.pair else 1  # IR tiles (128 rows) per table tile
        if not self.atomic:  # one whole-K segment per tile (a plain GEMM has no split)
            if self.tail() is not None:
                table = tuple(e[:4] for e in self.tail_table())
                return table, min(SM_COUNT // rows, len(table)) * rows
            table = tuple((mt, nt, 0, kbs) for mt, nt in self.order())
            return table, len(table) * rows
        tiles = list(dict.fromkeys((mt // rows, nt) for mt, nt, _ in self.schedule))
        slots = SM_COUNT // rows
        best = (math.inf, 1)
        for splits in range(1, max(1, kbs // MIN_SEGMENT) + 1):
            waves = -(-len(tiles) * splits // slots)
            best = min(best, (waves * (-(-kbs // splits) + SEGMENT_COST), splits))
        splits = best[1]
        cut = [j * kbs // splits for j in range(splits + 1)]
        table = tuple((mt, nt, cut[j], cut[j + 1] - cut[j])
                      for j in range(splits) for mt, nt in tiles)
        return table, min(slots, len(table)) * rows

    def tail(self) -> tuple[int, int] | None:
        """(whole-tile entries, pieces per tail tile) for a plain GEMM whose tiles leave the last
        wave of CTAs (pairs) part full, or None. The whole waves keep whole tiles; each of the
        ``rest`` tiles after them is cut along K into ``q`` pieces, so that the pieces spread
        over every CTA. A piece costs its K blocks plus ``SEGMENT_COST``, and the last piece of a
        tail tile adds the others' partials, ``TAIL_FIXUP`` a partial; the cut is taken when it
        finishes ``MIXED_GAIN`` sooner than a last wave of whole tiles (config 5's 1/4 share:
        three waves and 34 tiles in two pieces; its 1/8 share keeps whole tiles)."""
        if not self.stream_k or self.atomic or self.columns() is not None:
            return None
        kbs = self.k // BK
        slots = SM_COUNT // (2 if self.pair else 1)
        waves, rest = divmod(len(self.order()), slots)
        if not waves or not rest:
            return None
        best: tuple[float, int | None] = (
            (1 - MIXED_GAIN) * (waves + 1) * (kbs + SEGMENT_COST), None)
        for q in range(2, kbs // MIN_SEGMENT + 1):
            rounds = -(-rest * q // slots)
            cost = (waves * (kbs + SEGMENT_COST) + rounds * (-(-kbs // q) + SEGMENT_COST)
                    + TAIL_FIXUP * (q - 1))
            if cost < best[0]:
                best = (cost, q)
        return None if best[1] is None else (waves * slots, best[1])

    def tail_table(self) -> tuple[tuple[int, ...], ...]:
        """The work table of a plan with a ``tail``: (m tile, n tile, first K block, K blocks,
        role, piece, pieces, tail tile) per entry. The whole tiles come first, in raster order;
        then the pieces, split-major (piece j of every tail tile, then piece j + 1), so the
        pieces running at once read the same K window of A and B."""
        whole, q = self.tail()
        kbs = self.k // BK
        order = self.order()
        table = [(mt, nt, 0, kbs, ROLE_WHOLE, 0, 0, 0) for mt, nt in order[:whole]]
        cut = [j * kbs // q for j in range(q + 1)]
        table += [(mt, nt, cut[j], cut[j + 1] - cut[j], ROLE_PIECE, j, q, u)
                  for j in range(q) for u, (mt, nt) in enumerate(order[whole:])]
        return tuple(table)

    def order(self) -> list[tuple[int, int]]:
        """A plain GEMM's table tiles (m tile, n tile) in the order the CTAs take them."""
        rows = 2 if self.pair else 1
        return raster(self.m // (BM * rows), self.n // self.bn,
                      math.isqrt(SM_COUNT // rows))

    def columns(self) -> tuple[tuple[tuple[int, int, int], ...], int] | None:
        """A plain pair GEMM's tiles in mixed widths, for when whole 256-column tiles would
        leave the last wave of SM pairs part-empty: (256-row band, first column, width) per
        entry (width 0: a gap the pair skips) and the grid; None keeps the uniform table.

        Each band of C is cut into whole 256-column tiles and, at its right end, tiles of one
        narrower width ``w`` from ``NARROW`` (as many in every band as keep the rest a multiple
        of 256 columns). The tiles go to the pairs widest first, each to the pair with the least
        work so far (a tile costs its K blocks at its width's ``K_BLOCK_TIME`` plus
        ``SEGMENT_COST``; ties to the lowest pair, so the whole tiles keep the IR's order
        round-robin), and the table lists them round by round: entry ``r * used + q`` is pair
        ``q``'s ``r``-th tile, which the kernel's ``cluster + i * nclusters`` walk hands it. The
        plan with the shortest longest pair wins if it beats whole tiles by ``MIXED_GAIN``.
        With the measured times that happens where the tiles do not fill one wave of pairs (a
        1024^3 GEMM's 16 tiles become 64 of 64 columns); a last wave that is only part full
        stays as it is, since a narrower tile is barely faster per K block. Every element of C
        is still one tile's whole K loop, in the same K order."""
        if not self.mixed or self.atomic or not self.pair or self.n % 256:
            return None
        kbs = self.k // BK
        pairs = SM_COUNT // 2
        bands = self.m // (2 * BM)
        order = self.order()

        def cost(w: int) -> float:
            return kbs * K_BLOCK_TIME[w] + SEGMENT_COST

        best: tuple[float, list | None] = (
            (1 - MIXED_GAIN) * -(-len(order) // pairs) * cost(256), None)
        for w in NARROW:
            step = 256 // math.gcd(w, 256)  # narrow tiles a band adds at a time
            for groups in range(1, min(bands * (self.n // (w * step)),
                                       -(-2 * pairs // step)) + 1):
                per_band = [groups // bands + (b < groups % bands) for b in range(bands)]
                whole = [(self.n - g * step * w) // 256 for g in per_band]
                tiles = [(mt, nt * 256, 256) for mt, nt in order if nt < whole[mt]]
                tiles += [(mt, whole[mt] * 256 + j * w, w)
                          for mt in range(bands) for j in range(per_band[mt] * step)]
                lists, span = _spread([t[2] for t in tiles], pairs, cost)
                if span < best[0]:
                    best = (span, [[tiles[i] for i in q] for q in lists if q])
        if best[1] is None:
            return None
        lists = best[1]
        used, rounds = len(lists), max(map(len, lists))
        table = tuple(lists[q][r] if r < len(lists[q]) else (0, 0, 0)
                      for r in range(rounds) for q in range(used))
        return table, 2 * used


def raster(rows: int, cols: int, group: int) -> list[tuple[int, int]]:
    """Every (row, column) of a rows x cols grid of tiles, in groups of ``group`` rows (the last
    group may be shorter), column by column within a group, rows fastest."""
    out = []
    for g0 in range(0, rows, group):
        height = min(group, rows - g0)
        out += [(g0 + r, c) for c in range(cols) for r in range(height)]
    return out


def _spread(widths: list[int], pairs: int, cost) -> tuple[list[list[int]], float]:
    """Tile indexes per pair, widest first, each to the least-loaded pair (the lowest on a
    tie), and the longest pair's load."""
    import heapq

    heap = [(0.0, q) for q in range(pairs)]
    lists: list[list[int]] = [[] for _ in range(pairs)]
    for i in sorted(range(len(widths)), key=lambda i: -widths[i]):
        load, q = heapq.heappop(heap)
        lists[q].append(i)
        heapq.heappush(heap, (load + cost(widths[i]), q))
    return lists, max(load for load, _ in heap)


# --- matching ----------------------------------------------------------------------------------


def _names_in(e: object) -> set[str]:
    out: set[str] = set()
    if isinstance(e, Var):
        out.add(e.name)
    elif isinstance(e, BinaryExpr):
        out |= _names_in(e.left) | _names_in(e.right)
    elif isinstance(e, tuple):
        for x in e:
            out |= _names_in(x)
    elif isinstance(e, Expr):
        for f in getattr(e, "__dataclass_fields__", {}):
            out |= _names_in(getattr(e, f))
    return out


@dataclass(frozen=True)
class Nest:
    """A block-tiled matmul nest as Emmy writes it, whatever the operands' type: C [M, N] (+)=
    A [M, K] @ B [K, N] through two shared tiles fed by cp.async copies, one K loop with one
    inner loop of loads, products and Accum adds into Init'ed f32 accumulators, and Writes of the
    accumulators into C (atomic for split-K)."""

    tile: Tile
    kloop: Loop | StridedLoop
    copies: tuple[CpAsyncCopy, ...]
    accs: int  # accumulators per thread
    a: str
    b: str
    c: str
    m: int
    n: int
    k: int
    atomic: bool
    mi: int  # the Tile's block axis over M
    ni: int  # the Tile's block axis over N


def nest(op: KernelOp, buffers: Mapping[str, Buffer]) -> Nest | None:
    """The facts of the nest ``op`` holds, or None when it is not one (see ``Nest``)."""
    t = op.body
    if not isinstance(t, Tile) or not t.is_static_grid or t.aux_threads:
        return None
    body = t.body
    inits = [s for s in body if isinstance(s, Init)]
    smems = [s for s in body if isinstance(s, Smem)]
    loops = [s for s in body if isinstance(s, Loop | StridedLoop)]
    writes = [s for s in body if isinstance(s, Write)]
    allowed = (Init, Smem, CpAsyncCopy, CpAsyncCommit, Loop, StridedLoop, Write)
    if not all(isinstance(s, allowed) for s in body):
        return None
    if len(smems) != 2 or len(loops) != 1 or not writes or not inits:
        return None
    kloop = loops[0]
    copies = [s for s in walk(body) if isinstance(s, CpAsyncCopy)]
    feeds = {c.smem: c.src for c in copies}
    if len(feeds) != 2 or len(set(feeds.values())) != 2:
        return None
    # the inner loop: loads from the two shared buffers, multiply, Accum add
    inner = [s for s in kloop.body if isinstance(s, Loop | StridedLoop)]
    if len(inner) != 1:
        return None
    loads, prods, accs = {}, {}, []
    for s in inner[0].body:
        if isinstance(s, Load) and s.input in feeds and len(s.names) == 1:
            loads[s.names[0]] = s.input
        elif isinstance(s, Assign) and s.op.name in ("multiply", "mul") and len(s.args) == 2:
            prods[s.name] = tuple(s.args)
        elif isinstance(s, Accum) and s.op.name in ("add", "sum") and s.base is None:
            accs.append(s)
        else:
            return None
    init_names = {i.name for i in inits if i.identity == 0.0 and i.dtype.name == "f32"}
    for a in accs:
        pair = prods.get(a.value)
        if pair is None or a.name not in init_names or (a.dtype and a.dtype.name != "f32"):
            return None
        if {loads.get(pair[0]), loads.get(pair[1])} != set(feeds):
            return None
    if len(accs) != len(init_names):
        return None
    outs = {w.output for w in writes}
    if len(outs) != 1:
        return None
    c = outs.pop()
    written = {v for w in writes for v in w.values}
    if written != {a.name for a in accs} or len({w.atomic for w in writes}) != 1:
        return None
    atomic = writes[0].atomic
    cbuf = buffers.get(c)
    if cbuf is None or cbuf.dtype != "f32" or len(cbuf.shape) != 2:
        return None
    m, n = cbuf.shape
    # decide A and B by which shared buffer the inner loads index along the K loop's axis first
    a_name, b_name = _which_is_a(inner[0], feeds, loads, buffers, m, n)
    if a_name is None or b_name is None:
        return None
    abuf, bbuf = buffers[a_name], buffers[b_name]
    if abuf.dtype != bbuf.dtype:
        return None
    k = abuf.shape[1]
    if abuf.shape[0] != m or bbuf.shape != (k, n):
        return None
    # block axes: the ones windowing M and N, plus an optional split axis
    # (the row index of C's Writes names the M block axis, the column index the N one)
    axes = list(t.axes)
    if any(len(w.index) != 2 for w in writes):
        return None
    row_names = set().union(*(_names_in(w.index[0]) for w in writes))
    col_names = set().union(*(_names_in(w.index[1]) for w in writes))
    mb = [i for i, ax in enumerate(axes) if ax.window is not None and ax.name in row_names and
          ax.window.parent.extent.as_static() == m and m % ax.extent.as_static() == 0]
    nb = [i for i, ax in enumerate(axes) if ax.window is not None and ax.name in col_names and
          ax.window.parent.extent.as_static() == n and n % ax.extent.as_static() == 0 and
          i not in mb]
    if len(mb) != 1 or len(nb) != 1:
        return None
    return Nest(t, kloop, tuple(copies), len(accs), a_name, b_name, c, m, n, k, atomic,
                mb[0], nb[0])


def match(op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str], block: int,
          smem_bytes: int) -> MatmulPlan | None:
    g = nest(op, buffers)
    if g is None or buffers[g.a].dtype not in ("bf16", "f16"):
        return None
    t, kloop, copies, atomic = g.tile, g.kloop, g.copies, g.atomic
    a_name, b_name, c, m, n, k, mi, ni = g.a, g.b, g.c, g.m, g.n, g.k, g.mi, g.ni
    abuf = buffers[a_name]
    axes = list(t.axes)
    if m // axes[mi].extent.as_static() != BM:
        return None
    bn = n // axes[ni].extent.as_static()
    if bn not in (64, 128, 256) or g.accs * block != BM * bn:
        return None
    copy_names = set().union(*(_names_in(cp.src_index) for cp in copies))
    extents = [ax.extent.as_static() for ax in axes]
    strides = [math.prod(extents[i + 1:]) for i in range(len(extents))]
    # a split axis is a block axis (its stride spans whole blocks) that offsets the copies' K
    split_axes = [i for i, ax in enumerate(axes) if i not in (mi, ni) and ax.window is None and
                  ax.name in copy_names and strides[i] % block == 0 and extents[i] > 1]
    if len(split_axes) > 1:
        return None
    si = split_axes[0] if split_axes else None
    splits = extents[si] if si is not None else 1
    if (splits > 1) != atomic:
        return None
    if not kloop.axis.extent.is_static or kloop.axis.extent.as_static() * splits != k:
        return None
    block_axes = [i for i in (mi, ni, si) if i is not None]
    if any(strides[i] % block for i in block_axes):
        return None
    thread_cells = math.prod(extents[i] for i in range(len(axes)) if i not in block_axes)
    if thread_cells != block or block < 256 or block % 128:
        return None
    kc = k // splits
    if kc % BK or k % 8 or n % 8:
        return None
    stage = (BM * BK + BK * bn) * 2
    stages = min(MAX_STAGES, (smem_bytes - 2048) // stage)
    if stages < 2:
        return None
    sched = _schedule(t, block, mi, ni, si)
    pair = bn == 256 and m % (2 * BM) == 0
    return MatmulPlan(op.name, tuple(arg_order), a_name, b_name, c, abuf.dtype, m, n, k, bn,
                      splits, block, stages, atomic, sched, pair)


def _which_is_a(inner: Loop | StridedLoop, feeds: dict[str, str], loads: dict[str, str],
                buffers: Mapping[str, Buffer], m: int, n: int) -> tuple[str | None, str | None]:
    """A is the operand whose shared tile the inner loop indexes with its axis last (row-major
    [rows, k]); B the one it indexes with its axis first ([k, cols])."""
    axis = inner.axis.name
    a = b = None
    for s in inner.body:
        if not isinstance(s, Load) or s.input not in feeds or len(s.index) != 2:
            continue
        first, last = _names_in(s.index[0]), _names_in(s.index[1])
        if axis in last and axis not in first:
            a = feeds[s.input] if a in (None, feeds[s.input]) else "!"
        elif axis in first and axis not in last:
            b = feeds[s.input] if b in (None, feeds[s.input]) else "!"
    if a in (None, "!") or b in (None, "!") or a == b:
        return None, None
    return a, b


def _schedule(t: Tile, block: int, mi: int, ni: int, si: int | None
              ) -> tuple[tuple[int, int, int], ...]:
    """(m tile, n tile, split) of each CTA index, by the Tile's own decode of gid = cta*block:
    row-major over the axes, with Emmy's grouped raster order for a raster pair."""
    extents = list(t.extents)
    strides = [math.prod(extents[i + 1:]) for i in range(len(extents))]
    names = [a.name for a in t.axes]
    raster = None
    if t.raster_group and t.raster_axes and all(x in names for x in t.raster_axes):
        ri, rj = (names.index(x) for x in t.raster_axes)
        if rj == ri + 1:
            gi, oi = (ri, rj) if t.raster_orient == "m" else (rj, ri)
            g = min(t.raster_group, extents[gi])
            if extents[gi] > 1 and g > 1:
                raster = (gi, oi, g)
    out = []
    for cta in range(t.n_elements // block):
        gid = cta * block
        vals = [(gid // strides[i]) % extents[i] if i else gid // strides[i]
                for i in range(len(extents))]
        if raster is not None:
            gi, oi, g = raster
            ea, eb = extents[gi], extents[oi]
            sub = gid // strides[max(gi, oi)]
            if min(gi, oi):
                sub %= ea * eb
            grp, r = sub // (g * eb), sub % (g * eb)
            gsz = min(ea - grp * g, g) if ea % g else g
            vals[gi], vals[oi] = grp * g + r % gsz, r // gsz
        out.append((vals[mi], vals[ni], vals[si] if si is not None else 0))
    return tuple(out)


# --- emission ----------------------------------------------------------------------------------


class _Text:
    def __init__(self) -> None:
        self.lines: list[str] = []
        self.regs: dict[str, str] = {}
        self._n = 0

    def reg(self, name: str, typ: str) -> str:
        # bit types: tcgen05 operands want .b32 registers, and a .bN register serves any
        # instruction type of that width
        self.regs.setdefault(name, {"u32": "b32", "u64": "b64"}.get(typ, typ))
        return f"%{name}"

    def finish(self) -> list[str]:
        """The body with every template register renamed %m_<name>, so none can collide with a
        special register (%tid, %ctaid, ...)."""
        import re

        names = sorted(self.regs, key=len, reverse=True)
        pat = re.compile(r"%(" + "|".join(map(re.escape, names)) + r")(?![\w.])")
        return [pat.sub(r"%m_\1", line) for line in self.lines]

    def label(self, hint: str) -> str:
        self._n += 1
        return f"$M_{hint}_{self._n}"

    def __call__(self, line: str) -> None:
        self.lines.append(line if line.endswith(":") else f"\t{line}")


def bounded_wait(x: _Text, bar_addr: str, parity: str, code: int, fail: str,
                 limit_ns: int = WAIT_NS, sem: str = "", warp: bool = False) -> None:
    """An mbarrier wait that gives up: it polls ``try_wait.parity`` until the phase of
    ``parity`` completes or ``limit_ns`` of %globaltimer pass; then it sets bit ``code`` of the
    module's ``ptxgen_status`` word and branches to ``fail``. ``sem`` is the wait's memory
    order (``.acquire.cluster`` for a barrier another CTA of the cluster arrives at).

    ``warp=False`` is for one thread (the TMA producer, the MMA issuer): it leaves the poll the
    moment it sees the phase or runs out of time. ``warp=True`` is for a whole converged warp
    that goes on to warp-collective ``.sync.aligned`` instructions (the epilogue's
    ``tcgen05.ld``): every lane keeps polling until all 32 have seen the phase
    (``vote.sync.all``) or none has time left (``vote.sync.any`` on the time check), so the
    warp takes exactly one of the two exits, together. Polling again after seeing the phase is
    safe because the barriers this waits on cannot complete their next phase before this warp
    arrives on its partner barrier."""
    top, ok = x.label("wait"), x.label("waited")
    x(f"mov.u64 {x.reg('w_t0', 'u64')}, %globaltimer;")
    x(f"{top}:")
    x(f"mbarrier.try_wait.parity{sem}.shared::cta.b64 {x.reg('pw', 'pred')}, [{bar_addr}], "
      f"{parity};")
    if warp:
        x("vote.sync.all.pred %pw, %pw, -1;")
        x(f"@%pw bra.uni {ok};")
    else:
        x(f"@%pw bra {ok};")
    x(f"mov.u64 {x.reg('w_t1', 'u64')}, %globaltimer;")
    x("sub.u64 %w_t1, %w_t1, %w_t0;")
    x(f"setp.lt.u64 {x.reg('pw2', 'pred')}, %w_t1, {limit_ns};")
    if warp:
        x("vote.sync.any.pred %pw2, %pw2, -1;")
        x(f"@%pw2 bra.uni {top};")
        x(f"mov.u32 {x.reg('w_lane', 'u32')}, %laneid;")
        x("setp.eq.u32 %pw, %w_lane, 0;")
        x(f"@%pw red.global.or.b32 [ptxgen_status], {1 << code};")
    else:
        x(f"@%pw2 bra {top};")
        x(f"red.global.or.b32 [ptxgen_status], {1 << code};")
    x(f"bra.uni {fail};")
    x(f"{ok}:")


def wait_probe_ptx(limit_ns: int, code: int = 7, warp: bool = False,
                   arrive: bool = False) -> str:
    """A one-warp kernel that waits on an mbarrier through ``bounded_wait``, to test both of
    its exits without hanging a GPU. Without ``arrive`` nothing ever arrives at the barrier, so
    the wait must give up after ``limit_ns`` and set status bit ``code``; with ``arrive`` lane 0
    arrives first, so the wait must succeed and leave the status word alone. With ``warp`` all
    32 lanes wait in the warp-uniform form and then meet at a ``bar.warp.sync`` (which needs the
    whole warp, as the epilogue's ``tcgen05.ld`` does); otherwise lane 0 alone waits."""
    x = _Text()
    x(f"mov.u32 {x.reg('smem', 'u32')}, probe_bar;")
    x(f"mov.u32 {x.reg('tid', 'u32')}, %tid.x;")
    x(f"setp.ne.u32 {x.reg('p', 'pred')}, %tid, 0;")
    x("@%p bra $P_inited;")
    x("mbarrier.init.shared::cta.b64 [%smem], 1;")
    x("fence.mbarrier_init.release.cluster;")
    if arrive:
        x("mbarrier.arrive.shared::cta.b64 _, [%smem];")
    x("$P_inited:")
    x("bar.warp.sync -1;")
    if not warp:
        x("@%p bra $P_done;")
    bounded_wait(x, "%smem", "0", code, "$P_done", limit_ns, warp=warp)
    x("$P_done:")
    if warp:
        x("bar.warp.sync -1;")
    x("ret;")
    decls = "\n".join(f"\t.reg .{t} %m_{n};" for n, t in x.regs.items())
    return "\n".join([
        f".version {PTX_VERSION}\n.target {TARGET}\n.address_size 64\n",
        ".global .align 4 .u32 ptxgen_status;",
        ".visible .entry wait_probe(\n\t.param .u64 wait_probe_param_unused\n)\n"
        ".maxntid 32, 1, 1\n{",
        "\t.shared .align 8 .b64 probe_bar;", decls, *x.finish(), "}", ""])


def _desc_hi(sbo: int, swizzle128: bool = True) -> int:
    """Bits 32-63 of a tcgen05 shared-memory descriptor: stride byte offset (>>4) at 32,
    the sm_100 descriptor version 1 at 46, the 128-byte swizzle mode (2) at 61."""
    return (sbo >> 4) | (1 << 14) | ((2 if swizzle128 else 0) << 29)


def instr_desc(dtype: str, bn: int, a_mn_major: bool = False, b_mn_major: bool = True,
               m: int = BM) -> int:
    """The 32-bit instruction descriptor of tcgen05.mma.kind::f16: f32 accumulator (bit 4),
    A/B format bf16 = 1 or f16 = 0 (bits 7, 10), A/B major-ness (bits 15, 16: 1 = MN-major),
    N >> 3 at bit 17, M >> 4 at bit 24 (M = 256 for a CTA pair's cta_group::2 MMA)."""
    fmt = 1 if dtype == "bf16" else 0
    return ((1 << 4) | (fmt << 7) | (fmt << 10) | (int(a_mn_major) << 15) |
            (int(b_mn_major) << 16) | ((bn >> 3) << 17) | ((m >> 4) << 24))


def emit(p: MatmulPlan) -> str:
    e = p.entry
    x = _Text()
    cols = p.columns()
    mixed = cols is not None  # per-entry width and first column (pair GEMMs only)
    tail = None if mixed else p.tail()  # whole-tile entries and pieces per tail tile
    if mixed:
        table, ctas = cols
    elif tail:
        table, ctas = p.tail_table(), p.segments()[1]
    else:
        table, ctas = p.segments()
    entries = len(table)
    pair = p.pair
    g = 2 if pair else 1  # the tcgen05 cta_group
    nb = p.bn // g  # B columns this CTA loads (a pair splits B by columns)
    a_stage = BM * BK * 2  # 16 KiB
    b_chunk = BK * 64 * 2  # 8 KiB: 64 K rows x 64 columns
    b_stage = BK * nb * 2
    stages = MAX_STAGES if pair else p.stages
    staging = 2 * STAGE_BUF * len(EPILOGUE_WARPS) if p.staged else 0
    while stages > 2 and 1024 + stages * (a_stage + b_stage) + staging + 256 > SMEM_LIMIT:
        stages -= 1  # the staging buffers take the place of a stage where both do not fit
    stage_tx = g * (a_stage + b_stage)  # bytes the MMA's full barrier waits for
    b_off = stages * a_stage
    epi_off = stages * (a_stage + b_stage)  # 1024-byte aligned: whole stages before it
    bar_off = epi_off + staging
    full, empty = 0, stages * BAR_BYTES
    tfull = 2 * stages * BAR_BYTES
    tempty = tfull + 2 * BAR_BYTES
    drain = tempty + 2 * BAR_BYTES
    slot = drain + BAR_BYTES
    smem_total = 1024 + bar_off + slot + 16
    tmem_cols = 2 * p.bn if 2 * p.bn <= 512 else p.bn
    accs = tmem_cols // p.bn
    if tmem_cols > 256:
        # a CTA holding more than half of TMEM must be alone on its SM: ask for more than half
        # of the SM's shared memory
        smem_total = max(smem_total, 120 * 1024)
    idesc = instr_desc(p.dtype, p.bn, m=g * BM)
    a_hi = _desc_hi(1024)  # K-major A: 8-row groups 1024 bytes apart
    b_hi = _desc_hi(1024)  # MN-major B: 8-row (K) groups 1024 bytes apart
    b_lbo = (BK * 128) >> 4  # MN-major B: 64-column swizzle atoms BK*128 bytes apart
    ept = 32 * len(EPILOGUE_WARPS)

    u32, u64, pred = "u32", "u64", "pred"
    r = lambda n, t=u32: x.reg(n, t)  # noqa: E731

    def wait(bar_addr: str, parity: str, code: int, fail: str, sem: str = "",
             warp: bool = False) -> None:
        bounded_wait(x, bar_addr, parity, code, fail, sem=sem, warp=warp)

    def sched_lookup(skip: str) -> None:
        """Entry %t of the table into %mt, %nt, %kb0, %cnt (mixed widths: %mt, %col, %wid,
        %cnt, with %kb0 0); an empty entry branches to skip."""
        x(f"mul.wide.u32 {r('s_off', u64)}, %t, {16 if tail else 8};")
        x(f"add.s64 %s_off, {r('sched', u64)}, %s_off;")
        if tail:  # (..., role | piece << 8 | pieces << 16, tail tile)
            x(f"ld.global.nc.v4.u32 {{{r('code')}, {r('code2')}, {r('code3')}, {r('tu')}}}, "
              "[%s_off];")
            x(f"and.b32 {r('role')}, %code3, 255;")
            x(f"bfe.u32 {r('pj')}, %code3, 8, 8;")
        else:
            x(f"ld.global.nc.v2.u32 {{{r('code')}, {r('code2')}}}, [%s_off];")
        x(f"and.b32 {r('mt')}, %code, 65535;")
        if mixed:
            x(f"shr.u32 {r('col')}, %code, 16;")
            x("shl.b32 %col, %col, 5;")
            x(f"and.b32 {r('wid')}, %code2, 65535;")
            x(f"mov.u32 {r('kb0')}, 0;")
        else:
            x(f"shr.u32 {r('nt')}, %code, 16;")
            x(f"and.b32 {r('kb0')}, %code2, 65535;")
        x(f"shr.u32 {r('cnt')}, %code2, 16;")
        x("setp.eq.u32 %p, %cnt, 0;")
        x(f"@%p bra {skip};")

    def advance_stage() -> None:
        x("add.u32 %it, %it, 1;")
        x("add.u32 %s, %s, 1;")
        x(f"setp.eq.u32 {r('pwrap', pred)}, %s, {stages};")
        x("@%pwrap mov.u32 %s, 0;")
        x("@%pwrap xor.b32 %ph, %ph, 1;")

    def cta_sync() -> None:
        """All threads of the CTA, or of both CTAs of a pair (whose barriers and TMEM the
        other CTA uses), meet."""
        if pair:
            x("barrier.cluster.arrive.release;")
            x("barrier.cluster.wait.acquire;")
        else:
            x("barrier.sync 0;")

    def advance_acc() -> None:
        x("add.u32 %tc, %tc, 1;")
        x("add.u32 %ab, %ab, 1;")
        x(f"setp.eq.u32 {r('pawrap', pred)}, %ab, {accs};")
        x("@%pawrap mov.u32 %ab, 0;")
        x("@%pawrap xor.b32 %aph, %aph, 1;")

    # --- set-up: pointers, ids, shared-memory carve-up, barriers, TMEM -----------------------
    x(f"ld.param.u64 {r('c_ptr', u64)}, [{e}_param_{p.c}];")
    x("cvta.to.global.u64 %c_ptr, %c_ptr;")
    x(f"mov.u32 {r('tid')}, %tid.x;")
    x(f"setp.eq.u32 {r('ptrue', pred)}, %tid, %tid;")
    if pair:  # a pair walks the table by cluster; rank 0 is the pair's leader
        x(f"mov.u32 {r('rank')}, %cluster_ctarank;")
        x(f"setp.eq.u32 {r('plead', pred)}, %rank, 0;")
        x(f"mov.u32 {r('cta')}, %clusterid.x;")
        x(f"mov.u32 {r('ncta')}, %nclusterid.x;")
    else:
        x(f"mov.u32 {r('cta')}, %ctaid.x;")
        x(f"mov.u32 {r('ncta')}, %nctaid.x;")
    x(f"shr.u32 {r('warp')}, %tid, 5;")
    x(f"and.b32 {r('lane')}, %tid, 31;")
    x(f"mov.u32 {r('smem')}, smem_pool;")
    x("add.u32 %smem, %smem, 1023;")
    x("and.b32 %smem, %smem, -1024;")  # stages need 1024-byte alignment (128-byte swizzle)
    # the launch must have granted the whole layout; otherwise every CTA leaves at once (before
    # any barrier or TMEM exists), with a status bit, instead of touching memory past its end
    x(f"mov.u32 {r('dyn')}, %dynamic_smem_size;")
    x(f"mov.u32 {r('dyn_end')}, smem_pool;")
    x("add.u32 %dyn_end, %dyn_end, %dyn;")
    x(f"add.u32 {r('dyn_need')}, %smem, {bar_off + slot + 8};")
    x(f"setp.gt.u32 {r('pshort', pred)}, %dyn_need, %dyn_end;")
    x(f"setp.eq.u32 {r('pshort0', pred)}, %tid, 0;")
    x("and.pred %pshort0, %pshort0, %pshort;")
    x(f"@%pshort0 red.global.or.b32 [ptxgen_status], {1 << SMEM_SHORT};")
    x("@%pshort ret;")
    x(f"add.u32 {r('bars')}, %smem, {bar_off};")
    x(f"mov.u64 {r('tmap_a', u64)}, {e}_tmap_a;")
    x("cvta.global.u64 %tmap_a, %tmap_a;")
    x(f"mov.u64 {r('tmap_b', u64)}, {e}_tmap_b;")
    x("cvta.global.u64 %tmap_b, %tmap_b;")
    if p.staged:
        x(f"mov.u64 {r('tmap_c', u64)}, {e}_tmap_c;")
        x("cvta.global.u64 %tmap_c, %tmap_c;")
    x(f"mov.u64 %sched, {e}_sched;")
    x(f"setp.eq.u32 {r('p', pred)}, %tid, 0;")
    init_done = x.label("init_done")
    x(f"@!%p bra {init_done};")
    for s in range(stages):
        x(f"mbarrier.init.shared::cta.b64 [%bars+{full + 8 * s}], 1;")
        x(f"mbarrier.init.shared::cta.b64 [%bars+{empty + 8 * s}], 1;")
    for a in range(2):
        x(f"mbarrier.init.shared::cta.b64 [%bars+{tfull + 8 * a}], 1;")
        # the leader's accumulator is released by both CTAs' epilogues
        x(f"mbarrier.init.shared::cta.b64 [%bars+{tempty + 8 * a}], {g * ept};")
    x(f"mbarrier.init.shared::cta.b64 [%bars+{drain}], 1;")
    x("fence.mbarrier_init.release.cluster;")
    x("fence.proxy.async.shared::cta;")
    x("prefetch.tensormap [%tmap_a];")
    x("prefetch.tensormap [%tmap_b];")
    if p.staged:
        x("prefetch.tensormap [%tmap_c];")
    x(f"{init_done}:")
    alloc_done = x.label("alloc_done")
    x("setp.eq.u32 %p, %warp, 1;")
    x(f"@!%p bra {alloc_done};")
    x(f"add.u32 {r('slot')}, %bars, {slot};")
    # a pair allocates the same columns in both CTAs: warp 1 of each runs the alloc
    x(f"tcgen05.alloc.cta_group::{g}.sync.aligned.shared::cta.b32 [%slot], {tmem_cols};")
    x(f"tcgen05.relinquish_alloc_permit.cta_group::{g}.sync.aligned;")
    x(f"{alloc_done}:")
    x("tcgen05.fence::before_thread_sync;")
    cta_sync()  # not .aligned: warps 0 and 1 arrive from divergent branches
    x("tcgen05.fence::after_thread_sync;")
    x(f"ld.shared.b32 {r('tmem')}, [%bars+{slot}];")
    teardown = "$M_teardown"
    producer, mma, epi = "$M_producer", "$M_mma", "$M_epilogue"
    x("setp.eq.u32 %p, %warp, 0;")
    x(f"@%p bra {producer};")
    x("setp.eq.u32 %p, %warp, 1;")
    x(f"@%p bra {mma};")
    x(f"setp.ge.u32 %p, %warp, {EPILOGUE_WARPS[0]};")
    x(f"setp.le.u32 {r('q', pred)}, %warp, {EPILOGUE_WARPS[-1]};")
    x("and.pred %p, %p, %q;")
    x(f"@%p bra {epi};")
    x(f"bra.uni {teardown};")

    # --- producer: TMA loads into the stage ring ---------------------------------------------
    x(f"{producer}:")
    x("setp.ne.u32 %p, %lane, 0;")
    x(f"@%p bra {teardown};")
    for n in ("it", "s", "ph"):
        x(f"mov.u32 {r(n)}, 0;")
    x(f"mov.u32 {r('t')}, %cta;")
    p_tile, p_k, p_drain, p_noempty, p_next = (
        x.label(h) for h in ("p_tile", "p_k", "p_drain", "p_noempty", "p_next"))
    x(f"{p_tile}:")
    x(f"setp.ge.u32 %p, %t, {entries};")
    x(f"@%p bra {p_drain};")
    sched_lookup(p_next)
    if mixed:  # this CTA's half: rows rank*128 of the band, B columns rank*wid/2 of the tile
        x(f"shl.b32 {r('half')}, %rank, 7;")
        x(f"mad.lo.u32 {r('m0')}, %mt, {g * BM}, %half;")
        x(f"shr.u32 {r('hw')}, %wid, 1;")
        x(f"mad.lo.u32 {r('n0')}, %rank, %hw, %col;")
        # a half of 64 columns or fewer is one 64-column chunk of B; the second is not loaded
        x(f"setp.gt.u32 {r('pb2', pred)}, %hw, 64;")
        x(f"selp.u32 {r('tx')}, {stage_tx}, {stage_tx - g * b_chunk}, %pb2;")
    elif pair:  # this CTA's half: rows rank*128 of the 256-row tile, B columns rank*128
        x(f"shl.b32 {r('half')}, %rank, 7;")
        x(f"mad.lo.u32 {r('m0')}, %mt, {g * BM}, %half;")
        x(f"mad.lo.u32 {r('n0')}, %nt, {p.bn}, %half;")
    else:
        x(f"shl.b32 {r('m0')}, %mt, 7;")
        x(f"mul.lo.u32 {r('n0')}, %nt, {p.bn};")
    x(f"mul.lo.u32 {r('kk')}, %kb0, {BK};")
    x(f"mov.u32 {r('kb')}, 0;")
    x(f"{p_k}:")
    x(f"setp.lt.u32 %p, %it, {stages};")
    x(f"@%p bra {p_noempty};")
    x(f"mad.lo.u32 {r('ebar')}, %s, 8, %bars;")
    x(f"add.u32 %ebar, %ebar, {empty};")
    x(f"xor.b32 {r('par')}, %ph, 1;")
    wait("%ebar", "%par", 1, p_drain)
    x(f"{p_noempty}:")
    x(f"mad.lo.u32 {r('fbar')}, %s, 8, %bars;")
    if pair:
        # both CTAs' loads land on the leader's full barrier, which the MMA waits on; the
        # leader expects the bytes of both halves
        x(f"@%plead mbarrier.arrive.expect_tx.shared::cta.b64 _, [%fbar], "
          f"{'%tx' if mixed else stage_tx};")
        x(f"mapa.shared::cluster.u32 {r('fbar_l')}, %fbar, 0;")
        tma, bar = ("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global"
                    ".mbarrier::complete_tx::bytes"), "%fbar_l"
    else:
        x(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [%fbar], {stage_tx};")
        tma, bar = ("cp.async.bulk.tensor.2d.shared::cluster.global.tile"
                    ".mbarrier::complete_tx::bytes"), "%fbar"
    x(f"mad.lo.u32 {r('adst')}, %s, {a_stage}, %smem;")
    x(f"{tma} [%adst], [%tmap_a, {{%kk, %m0}}], [{bar}];")
    x(f"mad.lo.u32 {r('bdst')}, %s, {b_stage}, %smem;")
    x(f"add.u32 %bdst, %bdst, {b_off};")
    for cidx in range(nb // 64):
        x(f"add.u32 {r('ncol')}, %n0, {cidx * 64};")
        x(f"add.u32 {r('bdc')}, %bdst, {cidx * b_chunk};")
        guard = "@%pb2 " if mixed and cidx else ""
        x(f"{guard}{tma} [%bdc], [%tmap_b, {{%ncol, %kk}}], [{bar}];")
    advance_stage()
    x(f"add.u32 %kk, %kk, {BK};")
    x("add.u32 %kb, %kb, 1;")
    x("setp.lt.u32 %p, %kb, %cnt;")
    x(f"@%p bra {p_k};")
    x(f"{p_next}:")
    x("add.u32 %t, %t, %ncta;")
    x(f"bra.uni {p_tile};")
    # drain: the loads of the last issued stages have landed before the CTA may exit (a
    # pair's loads all land on the leader's barriers, so the leader drains for both, and the
    # other CTA waits for it at the teardown's cluster barrier)
    x(f"{p_drain}:")
    if pair:
        x(f"@!%plead bra {teardown};")
    for j in range(1, stages + 1):
        skip = x.label("drain_skip")
        x(f"setp.lt.u32 %p, %it, {j};")
        x(f"@%p bra {skip};")
        x(f"sub.u32 {r('db')}, %it, {j};")
        x(f"rem.u32 {r('ds')}, %db, {stages};")
        x(f"div.u32 {r('du')}, %db, {stages};")
        x("and.b32 %du, %du, 1;")
        x(f"mad.lo.u32 {r('dbar')}, %ds, 8, %bars;")
        wait("%dbar", "%du", 5, teardown)
        x(f"{skip}:")
    x(f"bra.uni {teardown};")

    # --- MMA issuer --------------------------------------------------------------------------
    x(f"{mma}:")
    x("setp.ne.u32 %p, %lane, 0;")
    x(f"@%p bra {teardown};")
    if pair:  # the leader issues the pair's MMAs
        x(f"@!%plead bra {teardown};")
        x(f"mov.b16 {r('pmask', 'b16')}, 3;")
    commit = (f"tcgen05.commit.cta_group::{g}.mbarrier::arrive::one.shared::cluster"
              + (".multicast::cluster.b64 [{}], %pmask;" if pair else ".b64 [{}];"))
    for n in ("it", "s", "ph", "tc", "ab", "aph"):
        x(f"mov.u32 {r(n)}, 0;")
    x("mov.u32 %t, %cta;")
    x(f"mov.u32 {r('idesc')}, {idesc};")
    idesc_n0 = instr_desc(p.dtype, 0, m=g * BM)  # the descriptor without its N field
    m_tile, m_k, m_end, m_free, m_next = (
        x.label(h) for h in ("m_tile", "m_k", "m_end", "m_free", "m_next"))
    x(f"{m_tile}:")
    x(f"setp.ge.u32 %p, %t, {entries};")
    x(f"@%p bra {m_end};")
    sched_lookup(m_next)
    x(f"setp.lt.u32 %p, %tc, {accs};")
    x(f"@%p bra {m_free};")
    x(f"mad.lo.u32 {r('tebar')}, %ab, 8, %bars;")
    x(f"add.u32 %tebar, %tebar, {tempty};")
    x("xor.b32 %par, %aph, 1;")
    wait("%tebar", "%par", 3, m_end, ".acquire.cluster" if pair else "")
    x(f"{m_free}:")
    x("tcgen05.fence::after_thread_sync;")
    if mixed:  # N = the tile's width, at bit 17 in units of 8
        x(f"shr.u32 {r('idn')}, %wid, 3;")
        x("shl.b32 %idn, %idn, 17;")
        x(f"or.b32 %idesc, %idn, {idesc_n0};")
    x(f"mad.lo.u32 {r('dtm')}, %ab, {p.bn}, %tmem;")
    x("mov.u32 %kb, 0;")
    x(f"{m_k}:")
    x("mad.lo.u32 %fbar, %s, 8, %bars;")
    wait("%fbar", "%ph", 2, m_end)
    x("tcgen05.fence::after_thread_sync;")
    x(f"mad.lo.u32 {r('aaddr')}, %s, {a_stage}, %smem;")
    x(f"mad.lo.u32 {r('baddr')}, %s, {b_stage}, %smem;")
    x(f"add.u32 %baddr, %baddr, {b_off};")
    x(f"shr.u32 {r('alo')}, %aaddr, 4;")
    x("and.b32 %alo, %alo, 16383;")
    x(f"or.b32 %alo, %alo, {1 << 16};")  # LBO field 1 (unused by a 128-byte swizzled K-major)
    x(f"shr.u32 {r('blo')}, %baddr, 4;")
    x("and.b32 %blo, %blo, 16383;")
    x(f"or.b32 %blo, %blo, {b_lbo << 16};")
    x(f"setp.ne.u32 {r('pacc', pred)}, %kb, 0;")
    for kk in range(BK // UMMA_K):
        # K step kk: A advances 32 bytes inside the swizzle row, B 16 rows of 128 bytes
        x(f"add.u32 {r('alo_k')}, %alo, {kk * (UMMA_K * 2 >> 4)};")
        x(f"add.u32 {r('blo_k')}, %blo, {kk * (UMMA_K * 128 >> 4)};")
        x(f"mov.b64 {r('adesc', 'b64')}, {{%alo_k, {a_hi}}};")
        x(f"mov.b64 {r('bdesc', 'b64')}, {{%blo_k, {b_hi}}};")
        acc = "%pacc" if kk == 0 else r("ptrue", pred)
        x(f"tcgen05.mma.cta_group::{g}.kind::f16 [%dtm], %adesc, %bdesc, %idesc, {acc};")
    x("mad.lo.u32 %ebar, %s, 8, %bars;")
    x(f"add.u32 %ebar, %ebar, {empty};")
    x(commit.format("%ebar"))  # the stage is free again (in both CTAs of a pair)
    advance_stage()
    x("add.u32 %kb, %kb, 1;")
    x("setp.lt.u32 %p, %kb, %cnt;")
    x(f"@%p bra {m_k};")
    x(f"mad.lo.u32 {r('tfbar')}, %ab, 8, %bars;")
    x(f"add.u32 %tfbar, %tfbar, {tfull};")
    x(commit.format("%tfbar"))  # the accumulator is ready (for both CTAs' epilogues)
    advance_acc()
    x(f"{m_next}:")
    x("add.u32 %t, %t, %ncta;")
    x(f"bra.uni {m_tile};")
    x(f"{m_end}:")
    x(f"add.u32 {r('dr')}, %bars, {drain};")
    x(f"tcgen05.commit.cta_group::{g}.mbarrier::arrive::one.shared::cluster.b64 [%dr];")
    wait("%dr", "0", 6, teardown)
    x(f"bra.uni {teardown};")

    # --- epilogue: TMEM -> registers -> C ------------------------------------------------------
    vals = [r(f"v{i}", "b32") for i in range(32)]
    tma_out = ("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group"
               if p.atomic else "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group")

    def stage_block(chunk: int) -> None:
        """The warp's 32 x 32 block (each lane one row, in %v0..%v31) into its staging buffer
        ``chunk & 1``, then one TMA op of the whole block into C: rows srow.., columns
        scol + 32*chunk... Lane 0 first waits until the TMA op issued two blocks ago has read
        that buffer. Lane L writes its row's 16-byte piece j at piece j ^ (L & 7) of row L (the
        128-byte swizzle the tensor map names), so the 8 lanes of each quarter-warp store to
        all 32 banks at once."""
        buf, lane_base = (("%sb1", "%sbuf1") if chunk & 1 else ("%sb0", "%sbuf0"))
        x("@%plane0 cp.async.bulk.wait_group.read 1;")
        x("bar.warp.sync -1;")
        for j in range(8):
            x(f"xor.b32 {r('saddr')}, {lane_base}, {j * 16};")
            x(f"st.shared.v4.b32 [%saddr], {{{', '.join(vals[4 * j:4 * j + 4])}}};")
        x("fence.proxy.async.shared::cta;")  # the generic stores, before the TMA reads them
        x("bar.warp.sync -1;")
        x(f"add.u32 {r('sx')}, %scol, {chunk * STAGE_BLOCK};")
        x(f"@%plane0 {tma_out} [%tmap_c, {{%sx, %srow}}], [{buf}];")
        x("@%plane0 cp.async.bulk.commit_group;")

    wpt = len(EPILOGUE_WARPS) * g  # epilogue warps a table tile's rows are spread over
    warp_bytes = 32 * p.bn * 4  # one warp's 32 rows of a tile, f32

    def tail_piece(q: int) -> None:
        """A piece of a tail tile. Every piece's warp stores its 32 rows of the partial sum into
        its own slot of the module's workspace (``_ws``: [tail tile][piece][warp][chunk][16-byte
        word][lane], so each store instruction covers 512 contiguous bytes), then lane 0 adds
        one to the tile's counter for this warp (``_cnt``, release and acquire at GPU scope,
        after a fence in every lane). The warp whose add completes the count -- the last of
        the tile's ``q`` pieces to get there -- sums the ``q`` partials in piece order (its own
        read again from TMEM, the others from the workspace through L2), stores the sum into C
        as a whole tile's epilogue does, and clears the counter for the next launch. Nothing
        waits on another CTA, and the sum's order does not depend on which piece ends last."""
        x(f"mov.u64 {r('wsb', u64)}, {e}_ws;")
        x(f"mov.u64 {r('cnb', u64)}, {e}_cnt;")
        if pair:
            x(f"mad.lo.u32 {r('wslot')}, %rank, {len(EPILOGUE_WARPS)}, %quad;")
        else:
            x(f"mov.u32 {r('wslot')}, %quad;")
        # this lane's word in piece 0's slot of its warp, and in its own piece's slot
        x(f"mul.lo.u32 {r('wsi')}, %tu, {q * wpt};")
        x("add.u32 %wsi, %wsi, %wslot;")
        x(f"mul.wide.u32 {r('wsu', u64)}, %wsi, {warp_bytes};")
        x(f"mul.wide.u32 {r('wln', u64)}, %lane, 16;")
        x("add.s64 %wsu, %wsu, %wln;")
        x("add.s64 %wsu, %wsu, %wsb;")
        x(f"mul.wide.u32 {r('wso', u64)}, %pj, {wpt * warp_bytes};")
        x(f"add.s64 {r('wsl', u64)}, %wsu, %wso;")
        for chunk in range(p.bn // 32):
            x(f"add.u32 {r('tcol')}, %taddr, {chunk * 32};")
            x(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(vals)}}}, [%tcol];")
            x("tcgen05.wait::ld.sync.aligned;")
            for j in range(8):
                x(f"st.global.v4.b32 [%wsl+{(chunk * 8 + j) * 512}], "
                  f"{{{', '.join(vals[4 * j:4 * j + 4])}}};")
        done = x.label("piece_done")
        x("fence.acq_rel.gpu;")
        x("bar.warp.sync -1;")
        x(f"mad.lo.u32 {r('cni')}, %tu, {wpt}, %wslot;")
        x(f"mul.wide.u32 {r('cno', u64)}, %cni, 4;")
        x("add.s64 %cnb, %cnb, %cno;")
        x(f"setp.eq.u32 {r('pl0', pred)}, %lane, 0;")
        x(f"@%pl0 atom.acq_rel.gpu.global.add.u32 {r('old')}, [%cnb], 1;")
        x("shfl.sync.idx.b32 %old, %old, 0, 31, -1;")
        x(f"setp.ne.u32 %p, %old, {q - 1};")
        x(f"@%p bra.uni {done};")  # not the last piece: its partial is in the workspace
        x("fence.acq_rel.gpu;")
        ws = [r(f"w{i}", "b32") for i in range(32)]
        for chunk in range(p.bn // 32):
            for v in vals:
                x(f"mov.b32 {v}, 0x80000000;")  # -0.0: adding it changes no value
            for jj in range(q):
                own, add = x.label("own"), x.label("add")
                x(f"setp.eq.u32 %p, %pj, {jj};")
                x(f"@%p bra.uni {own};")
                for j in range(8):
                    x(f"ld.global.cg.v4.f32 {{{', '.join(ws[4 * j:4 * j + 4])}}}, "
                      f"[%wsu+{jj * wpt * warp_bytes + (chunk * 8 + j) * 512}];")
                x(f"bra.uni {add};")
                x(f"{own}:")
                x(f"add.u32 {r('tcol')}, %taddr, {chunk * 32};")
                x(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ws)}}}, [%tcol];")
                x("tcgen05.wait::ld.sync.aligned;")
                x(f"{add}:")
                for v, w in zip(vals, ws):
                    x(f"add.rn.f32 {v}, {v}, {w};")
            store_chunk(chunk)
        x("@%pl0 st.relaxed.gpu.global.u32 [%cnb], 0;")
        x(f"{done}:")

    x(f"{epi}:")
    if p.atomic:
        # C is zeroed by the module's zero kernel, which may still run when this kernel was
        # launched early (PG_LAUNCH_EARLY): nothing adds into C before that kernel has ended and
        # its stores are visible. Without an early launch there is nothing to wait for.
        x("griddepcontrol.wait;")
    x(f"sub.u32 {r('quad')}, %warp, {EPILOGUE_WARPS[0]};")
    x(f"shl.b32 {r('lanebase')}, %quad, 21;")  # TMEM lane (quad*32) in bits 16..31
    if p.staged:
        # two staging buffers per warp after the stage ring; each lane's swizzled row base
        x(f"mad.lo.u32 {r('sb0')}, %quad, {2 * STAGE_BUF}, %smem;")
        x(f"add.u32 %sb0, %sb0, {epi_off};")
        x(f"add.u32 {r('sb1')}, %sb0, {STAGE_BUF};")
        x(f"and.b32 {r('sswz')}, %lane, 7;")
        x("shl.b32 %sswz, %sswz, 4;")
        x(f"mad.lo.u32 %sswz, %lane, {STAGE_BLOCK * 4}, %sswz;")
        x(f"add.u32 {r('sbuf0')}, %sb0, %sswz;")
        x(f"add.u32 {r('sbuf1')}, %sb1, %sswz;")
        x(f"setp.eq.u32 {r('plane0', pred)}, %lane, 0;")
    for n in ("tc", "ab", "aph"):
        x(f"mov.u32 %{n}, 0;")
    x("mov.u32 %t, %cta;")
    e_tile, e_next = x.label("e_tile"), x.label("e_next")
    x(f"{e_tile}:")
    x(f"setp.ge.u32 %p, %t, {entries};")
    x(f"@%p bra {teardown};")
    sched_lookup(e_next)
    x("mad.lo.u32 %tfbar, %ab, 8, %bars;")
    x(f"add.u32 %tfbar, %tfbar, {tfull};")
    wait("%tfbar", "%aph", 4, teardown, warp=True)  # the whole warp goes on to tcgen05.ld
    x("tcgen05.fence::after_thread_sync;")
    # this thread's row of C and the accumulator's columns in TMEM (a pair's CTA holds rows
    # rank*128 of the 256-row tile, all BN columns)
    if pair:
        x("shl.b32 %half, %rank, 7;")
        x(f"mad.lo.u32 %m0, %mt, {g * BM}, %half;")
    else:
        x("shl.b32 %m0, %mt, 7;")
    x(f"add.u32 {r('taddr')}, %tmem, %lanebase;")
    x(f"mad.lo.u32 %taddr, %ab, {p.bn}, %taddr;")
    if p.staged:
        # this warp's rows of C start at m0 + quad*32; its blocks at columns nt*BN + 32*chunk
        x(f"mad.lo.u32 {r('srow')}, %quad, {STAGE_BLOCK}, %m0;")
        if mixed:
            x(f"mov.u32 {r('scol')}, %col;")
        else:
            x(f"mul.lo.u32 {r('scol')}, %nt, {p.bn};")
    else:
        x(f"mad.lo.u32 {r('row')}, %quad, 32, %lane;")
        x("add.u32 %row, %row, %m0;")
        x(f"mul.wide.u32 {r('crow', u64)}, %row, {p.n * 4};")
        if mixed:
            x("shl.b32 %n0, %col, 2;")
        else:
            x(f"mul.lo.u32 %n0, %nt, {p.bn * 4};")
        x(f"cvt.u64.u32 {r('ncol64', u64)}, %n0;")
        x("add.s64 %crow, %crow, %ncol64;")
        x("add.s64 %crow, %crow, %c_ptr;")
    def store_chunk(chunk: int) -> None:
        """%v0..%v31 (this lane's row, columns 32*chunk..) into C."""
        if p.staged:
            stage_block(chunk)
            return
        for j in range(8):
            quad = ", ".join(vals[4 * j:4 * j + 4])
            off = chunk * 128 + j * 16
            if p.atomic:
                x(f"red.global.add.v4.f32 [%crow+{off}], {{{quad}}};")
            else:
                x(f"st.global.v4.b32 [%crow+{off}], {{{quad}}};")

    if tail:
        piece, released = x.label("piece"), x.label("released")
        x("setp.ne.u32 %p, %role, 0;")
        x(f"@%p bra.uni {piece};")  # the role is the same in every lane
    chunks_done = x.label("chunks_done")
    for chunk in range(p.bn // 32):
        if mixed and chunk >= 2:  # a tile of width wid has wid/32 blocks (64 at the least)
            x(f"setp.le.u32 %p, %wid, {chunk * 32};")
            x(f"@%p bra {chunks_done};")
        x(f"add.u32 {r('tcol')}, %taddr, {chunk * 32};")
        x(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(vals)}}}, [%tcol];")
        x("tcgen05.wait::ld.sync.aligned;")
        store_chunk(chunk)
    if mixed:
        x(f"{chunks_done}:")
    if tail:
        x(f"bra.uni {released};")
        x(f"{piece}:")
        tail_piece(tail[1])
        x(f"{released}:")
    x("tcgen05.fence::before_thread_sync;")
    x("mad.lo.u32 %tebar, %ab, 8, %bars;")
    x(f"add.u32 %tebar, %tebar, {tempty};")
    if pair:  # the leader's barrier, which its MMA waits on
        x(f"mapa.shared::cluster.u32 {r('tebar_l')}, %tebar, 0;")
        x("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%tebar_l];")
    else:
        x("mbarrier.arrive.shared::cta.b64 _, [%tebar];")
    advance_acc()
    x(f"{e_next}:")
    x("add.u32 %t, %t, %ncta;")
    x(f"bra.uni {e_tile};")

    # --- teardown ----------------------------------------------------------------------------
    x(f"{teardown}:")
    if p.staged:  # the epilogue's TMA ops have finished with its staging buffers
        x("cp.async.bulk.wait_group 0;")
    x("tcgen05.fence::before_thread_sync;")
    cta_sync()
    x("setp.ne.u32 %p, %warp, 1;")
    x("@%p bra $M_exit;")
    x("bar.warp.sync -1;")
    x("tcgen05.fence::after_thread_sync;")
    x(f"tcgen05.dealloc.cta_group::{g}.sync.aligned.b32 %tmem, {tmem_cols};")
    x("$M_exit:")
    x("ret;")

    # --- module ------------------------------------------------------------------------------
    sched_words = []
    kbs = p.k // BK
    # mixed widths: (band | first column / 32 << 16, width | K blocks << 16); else
    # (m tile | n tile << 16, first K block | K blocks << 16)
    words = ([(mt, col // 32, w, kbs if w else 0) for mt, col, w in table] if mixed
             else [e[:4] for e in table])
    for i, (w0, w1, w2, w3) in enumerate(words):
        if max(w0, w1, w2, w3) >= 1 << 16:
            raise NotImplementedError("matmul template: more tiles than the schedule encodes")
        sched_words += [str(w0 | w1 << 16), str(w2 | w3 << 16)]
        if tail:
            _, _, _, _, role, piece_j, pieces, tu = table[i]
            sched_words += [str(role | piece_j << 8 | pieces << 16), str(tu)]
    n_tail = len(p.order()) - tail[0] if tail else 0
    rows = [", ".join(sched_words[i:i + 16]) for i in range(0, len(sched_words), 16)]
    params = ",\n".join(f"\t.param .u64 {e}_param_{q}" for q in p.params)
    decls = "\n".join(f"\t.reg .{t} %m_{n};" for n, t in x.regs.items())
    esz = 2
    head = [
        "//\n// Generated by ptxgen (B200 backend): tcgen05 GEMM template\n//",
        f"// @ptxgen launch grid={ctas} block={p.block} persistent=1"
        + (f" cluster={g}" if pair else ""),
        f"// @ptxgen dynamic_smem={smem_total}",
        f"// @ptxgen tensormap symbol={e}_tmap_a buffer={p.a} dtype={p.dtype} "
        f"dims={p.k},{p.m} strides={p.k * esz} box={BK},{BM} swizzle=128",
        f"// @ptxgen tensormap symbol={e}_tmap_b buffer={p.b} dtype={p.dtype} "
        f"dims={p.n},{p.k} strides={p.n * esz} box=64,{BK} swizzle=128",
        *([f"// @ptxgen tensormap symbol={e}_tmap_c buffer={p.c} dtype=f32 dims={p.n},{p.m} "
           f"strides={p.n * 4} box={STAGE_BLOCK},{STAGE_BLOCK} swizzle=128"] if p.staged else []),
        *([f"// @ptxgen zero entry={e}_zero buffer={p.c} grid={ZERO_GRID} block={ZERO_BLOCK}"]
          if p.atomic else []),
        f"// @ptxgen matmul m={p.m} n={p.n} k={p.k} bn={p.bn} splits={p.splits} "
        f"stages={stages} tiles={p.tiles} segments={entries} cta_group={g}"
        + (" widths=mixed" if mixed else "")
        + (f" tail={tail[0]},{tail[1]}" if tail else ""),
        "",
        f".version {PTX_VERSION}\n.target {TARGET}\n.address_size 64\n",
        ".extern .shared .align 1024 .b8 smem_pool[];",
        f".global .align 64 .b8 {e}_tmap_a[128];",
        f".global .align 64 .b8 {e}_tmap_b[128];",
        *([f".global .align 64 .b8 {e}_tmap_c[128];"] if p.staged else []),
        ".global .align 4 .u32 ptxgen_status;",
        *([f".global .align 16 .b8 {e}_ws[{n_tail * tail[1] * wpt * warp_bytes}];",
           f".global .align 4 .u32 {e}_cnt[{n_tail * wpt}];"] if tail else []),
        f".global .align {16 if tail else 8} .u32 {e}_sched[{len(sched_words)}] = {{\n\t"
        + ",\n\t".join(rows) + "\n};",
        "",
        f".visible .entry {e}(\n{params}\n)\n.maxntid {p.block}, 1, 1\n.minnctapersm 1\n"
        + (".reqnctapercluster 2, 1, 1\n" if pair else "") + "{",
        decls,
    ]
    tail = [zero_kernel_ptx(f"{e}_zero", p.m * p.n * 4)] if p.atomic else []
    return "\n".join(head + x.finish() + ["}", ""] + tail)


def zero_kernel_ptx(entry: str, nbytes: int) -> str:
    """The entry that zeroes a split-K GEMM's C (``nbytes``, a multiple of 16) ahead of it:
    ``ZERO_GRID`` x ``ZERO_BLOCK`` threads store 16 zero bytes at a time in a grid-stride
    loop. Its first instruction lets the launch that follows it on the stream start at once
    (``griddepcontrol.launch_dependents``), so that launch's set-up and MMAs overlap this one;
    the GEMM's epilogue waits for this kernel (``griddepcontrol.wait``) before adding into C."""
    chunks = nbytes // 16
    threads = ZERO_GRID * ZERO_BLOCK
    return "\n".join([
        f".visible .entry {entry}(\n\t.param .u64 {entry}_param_c\n)\n"
        f".maxntid {ZERO_BLOCK}, 1, 1\n{{",
        "\t.reg .pred %z_p;", "\t.reg .b32 %z_i, %z_t;", "\t.reg .b64 %z_c, %z_a;",
        "\tgriddepcontrol.launch_dependents;",
        f"\tld.param.u64 %z_c, [{entry}_param_c];",
        "\tcvta.to.global.u64 %z_c, %z_c;",
        "\tmov.u32 %z_i, %ctaid.x;",
        "\tmov.u32 %z_t, %tid.x;",
        f"\tmad.lo.u32 %z_i, %z_i, {ZERO_BLOCK}, %z_t;",
        f"\tsetp.ge.u32 %z_p, %z_i, {chunks};",
        "\t@%z_p bra $Z_done;",
        "$Z_loop:",
        "\tmul.wide.u32 %z_a, %z_i, 16;",
        "\tadd.s64 %z_a, %z_c, %z_a;",
        "\tst.global.v4.b32 [%z_a], {0, 0, 0, 0};",
        f"\tadd.u32 %z_i, %z_i, {threads};",
        f"\tsetp.lt.u32 %z_p, %z_i, {chunks};",
        "\t@%z_p bra $Z_loop;",
        "$Z_done:",
        "\tret;",
        "}", ""])

"""Multi-GPU partitioning of the benchmark configurations: one process per GPU.

A rank runs the same kernel on a contiguous share of the configuration:

* pointwise add / gelu chain / row softmax: the element (or row) axis splits into ``world``
  contiguous ranges; each rank holds its inputs and writes its outputs, which stay sharded;
* GEMM and split-K GEMM: the M axis splits; each rank holds its rows of A and C and all of B,
  with no collective;
* split-K GEMM along K instead (``ksplit=True``): each rank holds 1/N of A (its columns) and of
  B (its rows), computes all of C as a partial sum, and the ranks reduce-scatter C by rows
  over NCCL (the split-K reduction across GPUs), each keeping its M/N rows of the product.
  Measured at 2 ranks it lost to the M split (93.7 µs against 58.6: a 62 µs kernel of short
  segments, then 31 µs of reduce-scatter for 4 MB), so it is not the default;
* full sum: the element axis splits; each rank reduces its share to one partial, and an
  all-reduce of those partials combines them.

By default the ranks split the configuration's fixed size (strong scaling: the same problem at
every rank count); ``weak=True`` instead gives each rank a benchmark-sized share of a problem
``world`` times larger along the split axis.

``local_problem`` returns the rank's Plan: its Kernel IR problem (every rank's has the same
shape, so each rank compiles the same module), which arguments are split (``sharded``, along
``axes``), and which outputs are summed across ranks (``allreduce``) or summed and split by rows
(``reduce_scatter``). ``slice_inputs`` and ``combine`` apply that contract to concrete arrays.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from . import problems
from .problems import ProblemSpec


@dataclass(frozen=True)
class Plan:
    name: str
    world: int
    spec: ProblemSpec
    sharded: tuple[str, ...] = ()  # arguments split rank-contiguously (along ``axes``)
    allreduce: tuple[str, ...] = ()  # outputs summed across ranks after the kernel
    units: str = "bytes"  # what ``work`` counts: "bytes" (HBM) or "flops" (tensor)
    work: int = 0  # algorithmic bytes or flops of one rank's step
    extra: dict[str, Any] = field(default_factory=dict)
    # the axis each sharded argument is split along (default: its first)
    axes: dict[str, int] = field(default_factory=dict)
    # outputs each rank computes in full as a partial sum, then reduce-scatters by rows: the
    # ranks' partials are summed and rank r keeps rows [r*M/N, (r+1)*M/N)
    reduce_scatter: tuple[str, ...] = ()

    def slice_inputs(self, full: dict[str, np.ndarray], rank: int) -> dict[str, np.ndarray]:
        """This rank's input arrays, cut from the whole problem's."""
        out = {}
        for name, arr in full.items():
            if name in self.sharded:
                axis = self.axes.get(name, 0)
                n = arr.shape[axis] // self.world
                out[name] = np.take(arr, np.arange(rank * n, (rank + 1) * n), axis=axis)
            else:
                out[name] = arr
        return out

    def combine(self, local: dict[str, np.ndarray], group: Any = None) -> dict[str, np.ndarray]:
        """Finish a rank's outputs: all-reduce (sum) the ``allreduce`` ones across ``group``
        (a torch.distributed group; None is the default group); sum the ``reduce_scatter`` ones
        and keep this rank's rows. Sharded outputs stay local."""
        if (not self.allreduce and not self.reduce_scatter) or self.world == 1:
            return local
        import torch
        import torch.distributed as dist

        out = dict(local)
        for name in (*self.allreduce, *self.reduce_scatter):
            t = torch.from_numpy(np.ascontiguousarray(local[name]))
            dist.all_reduce(t, group=group)
            out[name] = t.numpy()
        rank = dist.get_rank(group)
        for name in self.reduce_scatter:
            rows = out[name].shape[0] // self.world
            out[name] = out[name][rank * rows:(rank + 1) * rows]
        return out


SIZES: dict[str, tuple[int, ...]] = {
    "c1_vector_add": (1 << 24,), "c2_gelu_chain": (8192, 8192), "c3_row_softmax": (16384, 4096),
    "c4_full_sum": (1 << 30,), "c5_matmul": (8192, 8192, 8192),
    "c5b_matmul_splitk": (1024, 1024, 65536),
}


SPLIT_AXIS: dict[str, str] = {
    "c1_vector_add": "elements", "c2_gelu_chain": "rows", "c3_row_softmax": "rows",
    "c4_full_sum": "elements (per-rank partials summed across ranks)",
    "c5_matmul": "rows of A and C (B replicated)",
    "c5b_matmul_splitk": "rows of A and C (B replicated)",
}


def _split(total: int, world: int, what: str) -> int:
    if total % world:
        raise ValueError(f"{what} of {total} does not split over {world} ranks")
    return total // world


def _c1(world: int, size: tuple[int, ...]) -> Plan:
    n = _split(size[0], world, "elements")
    return Plan("c1_vector_add", world, problems.pointwise_add(n), ("x", "y", "add"),
                work=12 * n)


def _c2(world: int, size: tuple[int, ...]) -> Plan:
    rows, cols = size
    r = _split(rows, world, "rows")
    return Plan("c2_gelu_chain", world, problems.gelu_chain(r, cols), ("x", "s", "mul_1"),
                work=4 * r * cols + 4 * r + 8)


def _c3(world: int, size: tuple[int, ...]) -> Plan:
    rows, cols = size
    r = _split(rows, world, "rows")
    return Plan("c3_row_softmax", world, problems.row_softmax(r, cols), ("x", "softmax"),
                work=8 * r * cols)


def _c4(world: int, size: tuple[int, ...]) -> Plan:
    n = _split(size[0], world, "elements")
    blocks = 148 * 8 if n >= (1 << 24) else max(1, min(148 * 8, n // (256 * 16)))
    return Plan("c4_full_sum", world, problems.full_sum(n, blocks=blocks), ("x",),
                allreduce=("sum_1",), work=4 * n + 4)


def _c5(world: int, size: tuple[int, ...]) -> Plan:
    m, n, k = size
    ml = _split(m, world, "rows of A")
    return Plan("c5_matmul", world, problems.matmul(ml, n, k), ("x0", "matmul"), units="flops",
                work=2 * ml * n * k)


def _c5b_k(world: int, size: tuple[int, ...]) -> Plan:
    """Split-K GEMM across ranks along K: rank r holds columns K_r of A and rows K_r of B (1/N
    of each operand), computes the whole of C from them as a partial sum with the split-K
    template, and the ranks reduce-scatter C by rows (the split-K reduction across GPUs), so
    each ends with its M/N rows of the product, as the row split leaves them."""
    m, n, k = size
    if world == 1:
        return _c5b(world, size)
    _split(m, world, "rows of C")
    kl = _split(k, world, "K")
    split = 4 if kl % (4 * 64) == 0 else 1
    return Plan("c5b_matmul_splitk", world,
                problems.matmul(m, n, kl, split_k=split, raster_group=None), ("x0", "x1"),
                units="flops", work=2 * m * n * kl, axes={"x0": 1, "x1": 0},
                reduce_scatter=("matmul",))


def _c5b(world: int, size: tuple[int, ...]) -> Plan:
    """Split-K GEMM split along M (rows of A and C; B replicated), no collective."""
    m, n, k = size
    ml = _split(m, world, "rows of A")
    # four K splits per 1024 rows, more when a rank holds fewer rows, so each rank keeps enough
    # CTAs to fill its SMs
    split = 4 * max(1, 1024 // ml)
    if k % (split * 64):
        split = 4
    return Plan("c5b_matmul_splitk", world,
                problems.matmul(ml, n, k, split_k=split, raster_group=None),
                ("x0", "matmul"), units="flops", work=2 * ml * n * k)


BUILDERS: dict[str, Callable[[int, tuple[int, ...]], Plan]] = {
    "c1_vector_add": _c1, "c2_gelu_chain": _c2, "c3_row_softmax": _c3, "c4_full_sum": _c4,
    "c5_matmul": _c5, "c5b_matmul_splitk": _c5b,
}


def local_problem(name: str, world: int = 1, size: tuple[int, ...] | None = None,
                  weak: bool = False, ksplit: bool = False) -> Plan:
    """The plan one of ``world`` ranks runs for configuration ``name``. ``size`` is the whole
    problem (default: the benchmark size). With ``weak`` the whole problem is ``world`` times
    that size along the sharded axis, so each rank keeps a benchmark-sized share (weak scaling);
    otherwise the ranks split the given size (strong scaling)."""
    if name not in BUILDERS:
        raise KeyError(f"unknown configuration {name!r} (have {', '.join(BUILDERS)})")
    whole = tuple(size) if size is not None else SIZES[name]
    if weak:
        whole = (whole[0] * world, *whole[1:])
    if ksplit and name == "c5b_matmul_splitk":  # the K split, for comparison
        return _c5b_k(world, whole)
    return BUILDERS[name](world, whole)

"""Multi-GPU partitioning of the benchmark configurations: one process per GPU.

Each configuration's Tile axis is independent work, so a rank runs the same kernel on a
contiguous share of it, with no collective on the data path:

* pointwise add / gelu chain / row softmax: the element (or row) axis splits into ``world``
  contiguous ranges; each rank holds its inputs and writes its outputs, which stay sharded;
* GEMM (and split-K GEMM): the M axis splits; each rank holds its rows of A and C and all of B
  (split-K also splits further along K inside the rank so every rank keeps the same number of
  CTAs);
* full sum: the element axis splits; each rank reduces its share to one partial, and the only
  collective of the whole path, one NCCL all-reduce of those partials, combines them.

``local_problem`` returns the rank's Kernel IR problem and the combine step; every rank's problem
has the same shape, so each rank compiles the same module.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

from . import problems
from .problems import ProblemSpec


@dataclass(frozen=True)
class Plan:
    name: str
    world: int
    spec: ProblemSpec
    allreduce: tuple[str, ...] = ()  # outputs all-reduced (summed) across ranks after the kernel
    units: str = "bytes"  # what ``work`` counts: "bytes" (HBM) or "flops" (tensor)
    work: int = 0  # algorithmic bytes or flops of one rank's step


def _bytes(c: int) -> int:
    return c


SIZES = {"c1_vector_add": 1 << 24, "c2_gelu_chain": (8192, 8192), "c3_row_softmax": (16384, 4096),
         "c4_full_sum": 1 << 30, "c5_matmul": (8192, 8192, 8192),
         "c5b_matmul_splitk": (1024, 1024, 65536)}


def _check_split(total: int, world: int, what: str) -> int:
    if total % world:
        raise ValueError(f"{what} of {total} does not split over {world} ranks")
    return total // world


BUILDERS: dict[str, Callable[[int], Plan]] = {}


def _register(name: str) -> Callable[[Callable[[int], Plan]], Callable[[int], Plan]]:
    def deco(fn: Callable[[int], Plan]) -> Callable[[int], Plan]:
        BUILDERS[name] = fn
        return fn
    return deco


@_register("c1_vector_add")
def _c1(world: int) -> Plan:
    n = _check_split(SIZES["c1_vector_add"], world, "elements")
    return Plan("c1_vector_add", world, problems.pointwise_add(n), work=12 * n)


@_register("c2_gelu_chain")
def _c2(world: int) -> Plan:
    rows, cols = SIZES["c2_gelu_chain"]
    r = _check_split(rows, world, "rows")
    return Plan("c2_gelu_chain", world, problems.gelu_chain(r, cols),
                work=4 * r * cols + 4 * r + 8)


@_register("c3_row_softmax")
def _c3(world: int) -> Plan:
    rows, cols = SIZES["c3_row_softmax"]
    r = _check_split(rows, world, "rows")
    return Plan("c3_row_softmax", world, problems.row_softmax(r, cols), work=8 * r * cols)


@_register("c4_full_sum")
def _c4(world: int) -> Plan:
    n = _check_split(SIZES["c4_full_sum"], world, "elements")
    return Plan("c4_full_sum", world, problems.full_sum(n), allreduce=("sum_1",), work=4 * n + 4)


@_register("c5_matmul")
def _c5(world: int) -> Plan:
    m, n, k = SIZES["c5_matmul"]
    ml = _check_split(m, world, "rows of A")
    return Plan("c5_matmul", world, problems.matmul(ml, n, k), units="flops",
                work=2 * ml * n * k)


@_register("c5b_matmul_splitk")
def _c5b(world: int) -> Plan:
    m, n, k = SIZES["c5b_matmul_splitk"]
    ml = _check_split(m, world, "rows of A")
    split = 4 * (m // ml) if (m // ml) * 4 * 64 <= k else 4
    return Plan("c5b_matmul_splitk", world,
                problems.matmul(ml, n, k, split_k=split, raster_group=None),
                units="flops", work=2 * ml * n * k)


def local_problem(name: str, world: int = 1) -> Plan:
    """The problem one of ``world`` ranks runs for configuration ``name``."""
    if name not in BUILDERS:
        raise KeyError(f"unknown configuration {name!r} (have {', '.join(BUILDERS)})")
    return BUILDERS[name](world)

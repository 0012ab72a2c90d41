"""The compiler's entry points: ``compile_module`` (reference ``ptxgen/compiler.py:82-93``) and
``to_ptx`` (reference ``compile.py:24-55``), with the same arguments and error behaviour.

A kernel first meets the template matchers (``templates``): a matmul-shaped nest over bf16/f16
operands becomes the TMA + tcgen05 kernel. Everything else, and everything with a flag that asks
for the plain lowering, goes through the generic lowering (``lower``).
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence
from typing import Any

from .ir import Graph, KernelOp
from .lower import Buffer, Lowering

__all__ = ["Buffer", "compile_module", "to_ptx", "kernel_for_meta"]


def compile_module(op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str],
                   block_threads: int, *, no_unroll: bool = False, no_fusion: bool = False,
                   no_cse: bool = False, smem_bytes: int = 0, templates: bool = True,
                   exchange: str | None = None) -> str:
    """The sm_100a PTX module for ``op``, launched with ``block_threads`` threads per block and
    ``smem_bytes`` of dynamic shared memory (meta.json's figure; templates size their pipelines
    to it). ``exchange`` names a one-element f32 output that the kernel, once every block has
    added into it, sums across ranks over peer memory (``templates.exchange``)."""
    if templates and exchange is None:
        from . import templates as tpl

        ptx = tpl.try_templates(op, buffers, arg_order, block_threads, smem_bytes)
        if ptx is not None:
            return ptx
    # sibling loops over one axis, trip by trip (``jam``); with unrolling off the jammed loop is
    # still a runtime loop with one body per trip. Then accumulators that hold equal values on
    # every trip become one (``congruence``), with common subexpression elimination. In the
    # default build, work a loop repeats across one thread axis is done once and shared
    # (``hoist``).
    from dataclasses import replace

    from .congruence import merge_equal
    from .hoist import share_invariant
    from .jam import jam

    stmts = jam(op.body.body)
    if not no_cse:
        stmts = merge_equal(stmts)
    tile = replace(op.body, body=stmts)
    if templates and exchange is None:
        tile = share_invariant(tile, block_threads)
    op = replace(op, body=tile)
    k = Lowering(op, buffers, arg_order, block_threads, no_unroll=no_unroll,
                 no_fusion=no_fusion, no_cse=no_cse, exchange=exchange).run()
    return k.render()


def as_graph(graph: Any) -> Graph:
    """This loader's Graph from a Graph, a graph JSON dict, or a live Emmy graph."""
    if isinstance(graph, Graph):
        return graph
    if isinstance(graph, dict):
        return Graph.from_dict(graph)
    return Graph.from_emmy(graph)


def kernel_for_meta(graph: Graph | Any, meta: dict[str, Any]) -> tuple[KernelOp, dict[str, Any]]:
    """The KernelOp whose name a meta.json kernel names, and that launch entry. ``graph`` may
    also be a graph JSON dict or a live Emmy graph (the reference's ``to_ptx`` argument)."""
    launches = {k["entry"]: k for k in meta["kernels"]}
    ops = as_graph(graph).kernel_ops()
    op = next((o for o in ops if o.name in launches), None)
    if op is None:
        raise ValueError(f"no KernelOp named like a meta.json kernel ({', '.join(launches)})")
    return op, launches[op.name]


def to_ptx(graph: Graph, meta: dict[str, Any], no_unroll: bool = False, no_fusion: bool = False,
           no_cse: bool = False, templates: bool = True) -> str:
    """The PTX module for the kernel meta.json names (same contract as the reference).
    ``templates=False`` keeps every kernel on the generic lowering."""
    op, launch = kernel_for_meta(graph, meta)
    if list(launch["block"][1:]) != [1, 1] or list(launch["grid"][1:]) != [1, 1]:
        raise NotImplementedError("only 1-D launches")
    if any(a.get("scalar") for a in launch["args"]):
        raise NotImplementedError("by-value scalar arguments")
    buffers = {
        a["name"]: Buffer(tuple(a["shape"]), a["dtype"],
                          bool(a.get("output")) or a["name"] in op.outputs)
        for a in launch["args"]
    }
    exchange = launch.get("exchange", {}).get("output")  # a sharded plan's own meta only
    return compile_module(op, buffers, launch["arg_order"], launch["block"][0],
                          no_unroll=no_unroll, no_fusion=no_fusion, no_cse=no_cse,
                          smem_bytes=int(launch.get("smem_bytes", 0)),
                          templates=templates and not (no_unroll or no_fusion or no_cse),
                          exchange=exchange)

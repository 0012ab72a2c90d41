"""Hand-written sm_100a kernel templates that replace whole Kernel IR nests.

``try_templates`` offers a kernel to each matcher in turn; the first that recognises it returns
the finished PTX module, else the kernel takes the generic lowering.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

from ..ir import KernelOp
from ..lower import Buffer


def try_templates(op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str],
                  block: int, smem_bytes: int) -> str | None:
    from . import matmul

    plan = matmul.match(op, buffers, arg_order, block, smem_bytes)
    if plan is not None:
        return matmul.emit(plan)
    return None

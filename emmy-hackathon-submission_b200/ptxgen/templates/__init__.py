"""Hand-written sm_100a kernel templates that replace whole Kernel IR nests: the tcgen05 GEMM
for bf16/f16 matmul nests (``matmul``) and the register-blocked f32 GEMM (``simt``).

``try_templates`` offers a kernel to each matcher in turn; the first that recognises it returns
the finished PTX module, else the kernel takes the generic lowering.
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

from ..ir import KernelOp
from ..lower import Buffer


def try_templates(op: KernelOp, buffers: Mapping[str, Buffer], arg_order: Sequence[str],
                  block: int, smem_bytes: int) -> str | None:
    from . import matmul, simt

    plan = matmul.match(op, buffers, arg_order, block, smem_bytes)
    if plan is not None:
        return matmul.emit(plan)
    blocked = simt.match(op, buffers, arg_order, block, smem_bytes)
    if blocked is not None:
        return simt.emit(blocked)
    return None

"""Direct NumPy formulas of the benchmark configurations: the CPU path timed as the baseline.

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg (and its
``--impl reference`` arm) use this module.

The reference compiler has no CPU implementation of its kernels (its output is PTX), so the CPU
path of the same Kernel IR semantics is NumPy, as the reference's problem set states them
(``tools/expressions_open.py``, ``tools/expressions_closed.py``): elementwise formulas evaluated in
f32 (bf16 inputs widened exactly, bf16 outputs rounded once to nearest even), the sum in f64 over
f32 chunks, and the GEMM as an f32 ``np.matmul`` of the bf16-rounded operands (multi-threaded BLAS).
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import Any

import numpy as np

from .fp import bf16_bits_to_f32, f32_to_bf16_bits

GELU_C = np.float32(0.044715)
GELU_K = np.float32(math.sqrt(2.0 / math.pi))


def vector_add(ins: dict[str, np.ndarray], meta: dict[str, Any]) -> dict[str, np.ndarray]:
    return {"add": ins["x"] + ins["y"]}


def gelu_chain(ins: dict[str, np.ndarray], meta: dict[str, Any]) -> dict[str, np.ndarray]:
    args = {a["name"]: a for a in meta["kernels"][0]["args"]}
    a = np.float32(args["mul_c1"]["data"][0])
    b = np.float32(args["add_c1"]["data"][0])
    x = bf16_bits_to_f32(ins["x"])
    u = a * x + b
    t = np.tanh(GELU_K * (u + GELU_C * (u * u * u)))
    y = np.float32(0.5) * u * (np.float32(1.0) + t) * ins["s"].reshape(-1, 1)
    return {"mul_1": f32_to_bf16_bits(y)}


def row_softmax(ins: dict[str, np.ndarray], meta: dict[str, Any]) -> dict[str, np.ndarray]:
    x = ins["x"]
    e = np.exp(x - x.max(-1, keepdims=True))
    return {"softmax": e * (np.float32(1.0) / e.sum(-1, keepdims=True))}


def full_sum(ins: dict[str, np.ndarray], meta: dict[str, Any]) -> dict[str, np.ndarray]:
    x = ins["x"].reshape(-1)
    total = 0.0
    for lo in range(0, x.size, 1 << 22):
        total += float(x[lo:lo + (1 << 22)].sum(dtype=np.float64))
    return {"sum_1": np.array([total], np.float32)}


def matmul(ins: dict[str, np.ndarray], meta: dict[str, Any]) -> dict[str, np.ndarray]:
    a = ins["x0"]
    b = ins["x1"]
    if a.dtype == np.uint16:
        a, b = bf16_bits_to_f32(a), bf16_bits_to_f32(b)
    return {"matmul": np.matmul(a, b)}


FORMULAS: dict[str, Callable[[dict[str, np.ndarray], dict[str, Any]], dict[str, np.ndarray]]] = {
    "c1_vector_add": vector_add, "c2_gelu_chain": gelu_chain, "c3_row_softmax": row_softmax,
    "c4_full_sum": full_sum, "c5_matmul": matmul, "c5b_matmul_splitk": matmul,
}

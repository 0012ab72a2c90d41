"""``pg_grid_sum_f32_noalloc``: the grid-kernel sum for callers that cannot allocate device
memory (a plug-in without an allocator of its own, or a process whose device memory is reserved
up front). ptxgen's two-kernel sum (the ``r17_grid_kernel`` problem) keeps its per-block partials
in a buffer the caller allocates; this entry point keeps them in a fixed 16 KiB device array
inside the library and allocates nothing.

The GPU test calls it through the C ABI twice in a row and checks each result against the
two-kernel sum launched through the existing entry points (``pg_module_load`` /
``pg_kernel_launch`` via ``ProblemSet``) on the same input. The two add in the same order (each
thread's grid-stride share in index order, the warp butterfly of strides 16..1, the halving tree
over the block's warp slots, then the same over the partials), so the results must be equal bit
for bit; each must also be within rel 1e-5 of the f64 sum of the data, the bar of the problem's
own formula. The second call uses fewer blocks on other data, so partials the first call left in
the shared array must not leak into it. The argument checks run before any CUDA call, so they
are tested on the CPU.

This file is named to be collected last: it passes alone in a fresh process and after every
other test."""

from __future__ import annotations

import numpy as np
import pytest

from ptxgen.build import build_library
from ptxgen.runtime import library

PG_ERR_ARGUMENT = -2
MAX_BLOCKS = 4096  # PG_GRID_SUM_MAX_BLOCKS in include/ptxgen_b200.h
RTOL = 1e-5  # r17_grid_kernel's tolerance


def test_noalloc_sum_rejects_bad_arguments_before_any_cuda_call() -> None:
    build_library()
    lib = library()
    aligned = 1 << 20  # never dereferenced: every case fails its argument check first
    for x, n, out, blocks in [(aligned, 16, aligned, 0),               # no blocks
                              (aligned, 16, aligned, MAX_BLOCKS + 1),  # beyond the array
                              (aligned, 16, 0, 128),                   # null out
                              (0, 16, aligned, 128),                   # null x with n > 0
                              (aligned + 2, 16, aligned, 128)]:        # misaligned x
        assert lib.pg_grid_sum_f32_noalloc(x, n, out, blocks, 0) == PG_ERR_ARGUMENT
    lib.pg_grid_sum_f32_noalloc(aligned, 16, aligned, MAX_BLOCKS + 1, 0)
    assert b"4096" in lib.pg_last_error()


@pytest.mark.gpu
def test_noalloc_sum_matches_the_two_kernel_sum(cuda) -> None:
    import torch

    from ptxgen.runtime import ProblemSet
    from ptxgen.suite import grid_kernel_sum

    lib = library()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    results = []
    for call, (n, blocks) in enumerate([(1 << 20, 128), ((1 << 20) + 12345, 64)]):
        x = np.random.default_rng(call).random(n, dtype=np.float32)
        spec = grid_kernel_sum(n=n, blocks=blocks)
        ps = ProblemSet(spec.graphs, spec.meta)
        tensors = ps.allocate()
        tensors["x"].copy_(torch.from_numpy(x))
        ps.launch(tensors, stream=stream, check_status=True)
        torch.cuda.synchronize()
        want = float(tensors["out"].cpu()[0])

        out = torch.full((1,), float("nan"), dtype=torch.float32, device=cuda)
        rc = lib.pg_grid_sum_f32_noalloc(tensors["x"].data_ptr(), n, out.data_ptr(), blocks,
                                         stream)
        assert rc == 0, lib.pg_last_error().decode(errors="replace")
        torch.cuda.synchronize()
        got = float(out.cpu()[0])
        exact = float(x.astype(np.float64).sum())
        assert got == want, (call, got, want)  # same summation order, same bits
        assert abs(got - exact) <= RTOL * abs(exact), (call, got, exact)
        results.append((got, want, exact))
    print("noalloc sum (got, two-kernel, f64):", results)

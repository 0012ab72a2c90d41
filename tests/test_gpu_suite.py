"""The op/dtype suite (``ptxgen.suite``) on a B200: each case's kernel, under each compiler flag
set, launched through the C-ABI launcher, against the oracle's run of the same Kernel IR on the
same seeded inputs, to the bar the case states: bit-exact for IEEE round-to-nearest arithmetic
(pointwise, casts, selects, f64, single-block reductions, the SIMT matmul); a few f32 ulp, one
bf16 ulp, or rel 2e-5 of the output's scale where fast-math approximations enter; rel 1e-6
where atomics add in the order the hardware picks. With fusion off, ptxas may fuse a product
into an add, so the bar holds against the oracle with products rounded or fused
(``check_flags``). Outputs carry 64 canary elements past
their end."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import gpu_run, oracle_once, reference_inputs
from test_gpu_parity import check, check_flags

from ptxgen.suite import MULTI, SUITE

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(SUITE))
@pytest.mark.parametrize("flags", [{}, {"no_unroll": True}, {"no_fusion": True},
                                   {"no_cse": True}],
                         ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_suite_parity(cuda, name: str, flags: dict) -> None:
    case = SUITE[name]()
    ins = reference_inputs(case.spec.meta)
    got = gpu_run(case.spec.graph, case.spec.meta, ins, guard=64, **flags)[case.out]

    def run(nf: bool) -> np.ndarray:
        return oracle_once(f"suite/{name}", case.spec.graph, case.spec.meta, ins, nf)[case.out]

    kind, bound = case.bar
    want = run(False)
    check_flags(kind, got.reshape(want.shape), lambda nf: run(nf).reshape(want.shape),
                case.out_dtype, bound, flags)


@pytest.mark.parametrize("name", sorted(MULTI))
def test_multi_kernel_parity(cuda, name: str) -> None:
    """A chained problem through ``ProblemSet``: the kernels in meta.json order on one stream,
    the intermediates one writes read by the next, against the oracle's chained run."""
    import torch
    from test_suite import multi_inputs

    from oracle.interp import run_problem
    from ptxgen.runtime import ProblemSet

    case = MULTI[name]()
    ins = multi_inputs(case.spec.meta)
    ps = ProblemSet(case.spec.graphs, case.spec.meta)
    tensors = ps.allocate()
    for n, t in tensors.items():
        if n in ins:
            t.copy_(torch.from_numpy(np.ascontiguousarray(ins[n]).reshape(-1)))
        else:
            t.fill_(float("nan"))
    ps.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    want = run_problem(case.spec.graphs, case.spec.meta, ins)
    for out in case.spec.meta["graph_outputs"]:
        got = tensors[out].cpu().numpy()
        kind, bound = case.bar
        check(kind, got, want[out].reshape(-1), "f32", bound)


@pytest.mark.parametrize("name", ["r17_grid_kernel", "f13_softmax_two_pass"])
def test_multi_kernel_graph_replay(cuda, name: str) -> None:
    """A chained problem captured once as a CUDA graph and replayed gives the eager launches'
    outputs bit for bit, and replays faster than launching each kernel through the launcher."""
    import time

    import numpy as np
    import torch
    from test_suite import multi_inputs

    from ptxgen.runtime import ProblemSet

    case = MULTI[name]()
    ins = multi_inputs(case.spec.meta)
    ps = ProblemSet(case.spec.graphs, case.spec.meta)
    tensors = ps.allocate()
    for n, t in tensors.items():
        if n in ins:
            t.copy_(torch.from_numpy(np.ascontiguousarray(ins[n]).reshape(-1)))
    ps.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    out = case.spec.meta["graph_outputs"][0]
    eager = tensors[out].clone()
    graph = ps.capture(tensors)
    tensors[out].fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(tensors[out], eager)

    def wall(fn, n: int = 200) -> float:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / n

    eager_s, graph_s = wall(lambda: ps.launch(tensors)), wall(graph.replay)
    print(f"{name}: eager {eager_s * 1e6:.1f} us, graph {graph_s * 1e6:.1f} us per step")
    assert graph_s < eager_s

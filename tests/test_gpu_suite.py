"""The op/dtype suite (``ptxgen.suite``) on a B200: each case's kernel, under each compiler flag
set, launched through the C-ABI launcher, against the oracle's run of the same Kernel IR on the
same seeded inputs, to the bar the case states: bit-exact for IEEE round-to-nearest arithmetic
(pointwise, casts, selects, f64, single-block reductions, the SIMT matmul); a few f32 ulp, one
bf16 ulp, or rel 2e-5 of the output's scale where fast-math approximations enter; rel 1e-6
where atomics add in the order the hardware picks. Outputs carry 64 canary elements past
their end."""

from __future__ import annotations

import pytest
from conftest import gpu_run, oracle_run, reference_inputs
from test_gpu_parity import check

from ptxgen.suite import SUITE

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(SUITE))
@pytest.mark.parametrize("flags", [{}, {"no_unroll": True}, {"no_fusion": True},
                                   {"no_cse": True}],
                         ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_suite_parity(cuda, name: str, flags: dict) -> None:
    case = SUITE[name]()
    ins = reference_inputs(case.spec.meta)
    got = gpu_run(case.spec.graph, case.spec.meta, ins, guard=64, **flags)[case.out]
    want = oracle_run(case.spec.graph, case.spec.meta, ins,
                      no_fusion=flags.get("no_fusion", False))[case.out]
    kind, bound = case.bar
    check(kind, got.reshape(want.shape), want, case.out_dtype, bound)

"""The tcgen05 GEMM template on a B200: parity against the f64 product of the same bf16/f16
operands (and against the oracle's run of the SIMT IR it replaces), split-K, odd tile counts,
and the bounded-wait give-up path.

Bar: the tensor cores accumulate in f32 in their own order, so results are not bit-equal to the
SIMT nest; the bound is rel 1e-2 on each element (the north-star bound for bf16 GEMM with f32
accumulation) with an absolute floor of 1e-4 of the largest |C|, for elements near zero, whose
relative error an f32 sum of K products does not bound. Measured on a B200, the largest error is
1e-7..1.3e-6 of max |C| for these cases and about 9e-6 at K = 8192 and 65536; it is printed.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import gpu_run, oracle_run, reference_inputs

from oracle.fp import bf16_bits_to_f32
from ptxgen import problems
from ptxgen.compiler import to_ptx
from ptxgen.ir import Graph

pytestmark = pytest.mark.gpu


def operands(spec: problems.ProblemSpec, ins: dict[str, np.ndarray]) -> tuple[np.ndarray, ...]:
    a, b = ins["x0"], ins["x1"]
    if a.dtype == np.uint16:
        a, b = bf16_bits_to_f32(a), bf16_bits_to_f32(b)
    else:
        a, b = a.astype(np.float32), b.astype(np.float32)
    return a.astype(np.float64), b.astype(np.float64)


def assert_gemm_close(got: np.ndarray, want: np.ndarray) -> float:
    err = np.abs(got.astype(np.float64) - want)
    scale = np.abs(want).max()
    bad = err > 1e-2 * np.abs(want) + 1e-4 * scale
    assert not bad.any(), f"{bad.sum()} elements off; max err {err.max():.3e} (|C| max {scale:.3e})"
    return float(err.max() / scale)


CASES = {
    "256_bn256": lambda: problems.matmul(256, 256, 256),
    "512x768x1024": lambda: problems.matmul(512, 768, 1024),
    "rect_bn128_k128": lambda: problems.matmul(256, 512, 128, bn=128),
    "bn64_odd_tiles": lambda: problems.matmul(384, 256, 512, bn=64),
    "f16": lambda: problems.matmul(256, 256, 256, dtype="f16"),
    "raster_ragged": lambda: problems.matmul(1280, 512, 256, raster_group=4),
    "splitk4": lambda: problems.matmul(256, 256, 1024, split_k=4, raster_group=None),
    "splitk_odd": lambda: problems.matmul(384, 512, 768, split_k=3, raster_group=None),
    # the mbarrier ring at its edges: one K block, and one more K block than stages (6 on a
    # pair, 4 on one SM) so the ring wraps once
    "k64_one_block": lambda: problems.matmul(256, 256, 64),
    "k448_ring_wraps_pair": lambda: problems.matmul(256, 512, 448),
    "k320_ring_wraps_1sm": lambda: problems.matmul(128, 256, 320),
    # 8 tiles x 256 K blocks: the template's own 18 uneven splits (14 or 15 K blocks), 144 CTAs
    "splitk_uneven": lambda: problems.matmul(512, 512, 16384, split_k=8, raster_group=None),
}


def template_ptx(spec: problems.ProblemSpec, staged: bool, mixed: bool = True) -> str:
    """The GEMM template's module for ``spec`` with the chosen epilogue: staged (each warp's
    32 x 32 blocks through shared memory, one TMA store or reduce-add per block; the default)
    or per thread (``st.global.v4`` / ``red.global.add.v4`` from registers). ``mixed=False``
    keeps whole 256-column tiles where the template would cut some narrower."""
    import dataclasses

    from ptxgen.compiler import kernel_for_meta
    from ptxgen.lower import Buffer
    from ptxgen.templates import matmul

    op, launch = kernel_for_meta(Graph.from_dict(spec.graph), spec.meta)
    bufs = {a["name"]: Buffer(tuple(a["shape"]), a["dtype"],
                              bool(a.get("output")) or a["name"] in op.outputs)
            for a in launch["args"]}
    plan = matmul.match(op, bufs, launch["arg_order"], launch["block"][0],
                        int(launch.get("smem_bytes", 0)))
    assert plan is not None
    return matmul.emit(dataclasses.replace(plan, staged=staged, mixed=mixed))


@pytest.mark.parametrize("staged", [True, False], ids=["staged", "per_thread"])
@pytest.mark.parametrize("key", sorted(CASES))
def test_tcgen05_gemm(cuda, key: str, staged: bool) -> None:
    spec = CASES[key]()
    ptx = template_ptx(spec, staged)
    assert "tcgen05.mma" in ptx and ("_tmap_c" in ptx) == staged
    if staged:
        assert ptx == to_ptx(Graph.from_dict(spec.graph), spec.meta)  # the default form
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64, ptx=ptx)["matmul"]
    a, b = operands(spec, ins)
    worst = assert_gemm_close(got, a @ b)
    print(f"{key} ({'staged' if staged else 'per thread'}): max |err| / max |C| = {worst:.3e}")


MIXED = {
    # (problem, cost model): the planner's own choice with the measured K-block times, or a
    # width-proportional model that cuts the part-full last wave into mixed widths
    "64_wide": (lambda: problems.matmul(256, 256, 256), False),  # four 64-column tiles
    "64_wide_1024": (lambda: problems.matmul(1024, 1024, 1024), False),
    # config 5's 1/8 share layout (one 256- and one 192-column tile per pair) and its 1/4 share
    # layout (two of each), at K = 1024
    "share8_256_192": (lambda: problems.matmul(1024, 8192, 1024), True),
    "share4_256_192": (lambda: problems.matmul(2048, 8192, 1024), True),
    "128_wide_raster": (lambda: problems.matmul(1280, 512, 256, raster_group=4), True),
}


@pytest.mark.parametrize("key", sorted(MIXED))
def test_mixed_widths_match_whole_tiles(cuda, key: str, monkeypatch) -> None:
    """The mixed-width table against whole 256-column tiles on the same operands: bit for bit
    (every element is one tile's whole K loop in the same K order either way), and at the GEMM
    bar against the f64 product."""
    from ptxgen.templates import matmul

    build, scaled = MIXED[key]
    spec = build()
    if scaled:
        monkeypatch.setattr(matmul, "K_BLOCK_TIME", {w: w / 256 for w in matmul.K_BLOCK_TIME})
    mixed, whole = template_ptx(spec, True), template_ptx(spec, True, mixed=False)
    assert "widths=mixed" in mixed and "widths=mixed" not in whole
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins, guard=64, ptx=mixed)["matmul"]
    ref = gpu_run(spec.graph, spec.meta, ins, guard=64, ptx=whole)["matmul"]
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    a, b = operands(spec, ins)
    worst = assert_gemm_close(got, a @ b)
    print(f"{key}: bit-equal to whole tiles; max |err| / max |C| = {worst:.3e}")


def simt_cases() -> dict[str, tuple[dict, dict]]:
    """(graph, meta) of each f32 nest the register-blocked template takes: the shipped m01 and
    the generated ones of ``test_simt.CASES``."""
    import json
    from pathlib import Path

    from test_simt import CASES, case

    d = Path(__file__).parent / "golden" / "shipped" / "m01_matmul_512"
    out = {"m01_shipped": (json.loads(next(d.glob("*.ir.json")).read_text()),
                           json.loads((d / "meta.json").read_text()))}
    for key in CASES:
        spec = case(key)
        out[key] = (spec.graph, spec.meta)
    return out


@pytest.mark.parametrize("key", ["m01_shipped", "one_k_step", "rect", "tile_32x32",
                                 "tile_64x64", "tile_64x128"])
def test_simt_gemm_bit_equal(cuda, key: str) -> None:
    """The register-blocked f32 template against the generic lowering of the same nest and
    against the oracle, bit for bit: every element of C is the same fma chain over k in order.
    The canaries past C must survive."""
    graph, meta = simt_cases()[key]
    g = Graph.from_dict(graph)
    ptx = to_ptx(g, meta)
    assert "@ptxgen simt" in ptx
    ins = reference_inputs(meta)
    out = meta["graph_outputs"][0]
    got = gpu_run(graph, meta, ins, guard=64, ptx=ptx)[out]
    generic = gpu_run(graph, meta, ins, guard=64, ptx=to_ptx(g, meta, templates=False))[out]
    want = oracle_run(graph, meta, ins)[out]
    assert np.array_equal(got.view(np.uint32), generic.view(np.uint32))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_tcgen05_matches_oracle_small(cuda) -> None:
    """The template against the oracle's run of the very SIMT nest it replaces."""
    spec = problems.matmul(256, 256, 128)
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins)["matmul"]
    want = oracle_run(spec.graph, spec.meta, ins)["matmul"].astype(np.float64)
    assert_gemm_close(got, want)


def test_tcgen05_full_k_rows(cuda) -> None:
    """A full-K (8192) slab of config 5: 128 rows of A against all of B."""
    spec = problems.matmul(128, 8192, 8192)
    ins = reference_inputs(spec.meta)
    got = gpu_run(spec.graph, spec.meta, ins)["matmul"]
    a, b = operands(spec, ins)
    assert_gemm_close(got, a @ b)


@pytest.mark.parametrize("warp", [False, True], ids=["one_thread", "warp_uniform"])
@pytest.mark.parametrize("arrive", [False, True], ids=["gives_up", "completes"])
def test_bounded_wait(cuda, warp: bool, arrive: bool) -> None:
    """Both exits of both wait forms. On an mbarrier nothing arrives at, the wait returns after
    its limit and sets its status bit, and the context stays usable; on one that lane 0 arrives
    at first, it succeeds without touching the status word. The warp-uniform form (the
    epilogue's, before ``tcgen05.ld``) runs on all 32 lanes and ends at a full-warp
    ``bar.warp.sync``, which only a converged warp passes."""
    import time

    import torch

    from ptxgen.runtime import Module
    from ptxgen.templates.matmul import wait_probe_ptx

    mod = Module(wait_probe_ptx(20_000_000, code=7, warp=warp, arrive=arrive))
    k = mod.kernel("wait_probe")
    dummy = torch.zeros(1, device="cuda")
    t0 = time.perf_counter()
    k.launch(1, 32, 0, [dummy.data_ptr()])
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert mod.status() == (0 if arrive else 1 << 7)
    assert mod.status() == 0  # taking the status clears it
    dummy += 1  # the context still runs work
    torch.cuda.synchronize()
    assert dummy.item() == 1.0


def test_short_shared_memory_launch_reports_and_returns(cuda) -> None:
    """A GEMM launched with less dynamic shared memory than its layout needs (here meta.json's
    figure, which is what every launch got before the runtime read the module's own) leaves at
    entry with status bit ``SMEM_SHORT``, before any barrier, TMEM or shared access exists; the
    context stays usable and the same module then runs correctly with its full figure."""
    import torch

    from ptxgen.runtime import Problem, library
    from ptxgen.templates.matmul import SMEM_SHORT

    spec = problems.matmul(256, 256, 256)
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    ins = reference_inputs(spec.meta)
    for name, arr in ins.items():
        tensors[name].copy_(torch.from_numpy(arr.reshape(-1).view(np.int16)).view(torch.bfloat16))
    tensors["matmul"].fill_(float("nan"))
    kernel, module = prob.load(), prob.module
    need = module.dynamic_smem
    short = int(spec.kernel["smem_bytes"])
    assert short < need
    module.fill_tensormaps({n: t.data_ptr() for n, t in tensors.items()})
    launch = prob.launch_entry
    ptrs = [tensors[n].data_ptr() for n in launch["arg_order"]]
    import ctypes

    arr = (ctypes.c_uint64 * len(ptrs))(*ptrs)
    stream = torch.cuda.current_stream().cuda_stream
    rc = library().pg_kernel_launch(kernel.handle, prob.grid(), launch["block"][0], short,
                                    stream, arr, len(ptrs))
    assert rc == 0
    torch.cuda.synchronize()
    assert module.status() == 1 << SMEM_SHORT
    assert torch.isnan(tensors["matmul"]).all()  # nothing was written
    prob.launch(tensors, check_status=True)  # the module's own figure: runs and is right
    torch.cuda.synchronize()
    got = tensors["matmul"].cpu().numpy().reshape(256, 256)
    a, b = operands(spec, ins)
    assert_gemm_close(got, a @ b)


def test_launcher_times_launches(cuda) -> None:
    """``pg_kernel_time`` (CUDA events around each launch) agrees with PyTorch's events on the
    same back-to-back launches of the config-5 template, within a factor of 1.5. The GEMM is
    large enough (4096 x 4096 x 2048, tens of microseconds) that the GPU, not the host's
    enqueueing, sets the pace of the PyTorch-timed loop."""
    import torch

    from ptxgen.runtime import Problem

    spec = problems.matmul(4096, 4096, 2048)
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    for t in tensors.values():
        t.zero_()
    ms = prob.time(tensors, warmup=3, reps=10)
    assert len(ms) == 10 and all(0 < t < 100 for t in ms), ms
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(10):
        prob.launch(tensors)
    stop.record()
    torch.cuda.synchronize()
    theirs = start.elapsed_time(stop) / 10
    ours = sorted(ms)[5]
    assert theirs / 1.5 < ours < theirs * 1.5, (ours, theirs)


@pytest.mark.parametrize("staged", [True, False], ids=["staged", "per_thread"])
def test_stream_k_tail(cuda, staged: bool) -> None:
    """A 4096^3 GEMM (256 pair tiles: three waves of 74 and 34 more) with its 34 tail tiles in
    two K pieces each: the last piece of each tile to finish sums both partials. C is filled
    with NaN before each of two launches of one module; they must agree bit for bit (the sum's
    order does not depend on which piece ends last, and the counters clear themselves), meet
    the GEMM bar against the f64 product on sampled rows, and stay within it of the whole-tile
    build."""
    import dataclasses

    import torch

    from ptxgen.compiler import kernel_for_meta
    from ptxgen.lower import Buffer
    from ptxgen.runtime import Problem
    from ptxgen.templates import matmul

    spec = problems.matmul(4096, 4096, 4096)
    op, launch = kernel_for_meta(Graph.from_dict(spec.graph), spec.meta)
    bufs = {a["name"]: Buffer(tuple(a["shape"]), a["dtype"],
                              bool(a.get("output")) or a["name"] in op.outputs)
            for a in launch["args"]}
    plan = matmul.match(op, bufs, launch["arg_order"], launch["block"][0],
                        int(launch.get("smem_bytes", 0)))
    plan = dataclasses.replace(plan, staged=staged)
    assert plan.tail() == (222, 2)
    ins = reference_inputs(spec.meta)
    outs = {}
    for name, p in (("tail", plan), ("whole", dataclasses.replace(plan, stream_k=False))):
        ptx = matmul.emit(p)
        assert ("tail=" in ptx) == (name == "tail")
        prob = Problem(spec.graph, spec.meta, ptx=ptx)
        t = prob.allocate()
        for k, arr in ins.items():
            host = np.ascontiguousarray(arr).reshape(-1)
            t[k].copy_(torch.from_numpy(host.view(np.int16)).view(t[k].dtype))
        runs = []
        for _ in range(2):
            t["matmul"].fill_(float("nan"))
            prob.launch(t, check_status=True)
            torch.cuda.synchronize()
            runs.append(t["matmul"].clone())
        assert torch.equal(runs[0].view(torch.int32), runs[1].view(torch.int32)), name
        outs[name] = runs[0].cpu().numpy().reshape(4096, 4096)
    rows = np.array(sorted({0, 4095, *range(7, 4096, 131)}))
    a, b = operands(spec, {"x0": ins["x0"].reshape(4096, 4096)[rows], "x1": ins["x1"]})
    worst = assert_gemm_close(outs["tail"][rows], a @ b)
    assert_gemm_close(outs["tail"], outs["whole"].astype(np.float64))
    print(f"stream-K tail ({'staged' if staged else 'per thread'}): max |err| / max |C| = "
          f"{worst:.3e}")


def test_splitk_zero_kernel_and_early_launch(cuda) -> None:
    """A split-K GEMM runs as its module's zero kernel followed by the GEMM launched early
    (programmatic stream serialization), eagerly and captured in a CUDA graph. C is filled with
    NaN before each run, so a GEMM that added into it before the zero kernel's stores landed, or
    a graph without the zeroing, leaves NaN behind; both runs must meet the GEMM bar against
    the f64 product (the reduce-add order may differ between runs, so not bit for bit)."""
    import numpy as np
    import torch

    from ptxgen.runtime import Problem

    spec = problems.matmul(512, 512, 16384, split_k=8, raster_group=None)
    ins = reference_inputs(spec.meta)
    prob = Problem(spec.graph, spec.meta)
    assert "matmul" in prob.module.zeroers
    tensors = prob.allocate()
    for name, arr in ins.items():
        tensors[name].copy_(torch.from_numpy(arr.reshape(-1).view(np.int16)).view(torch.bfloat16))
    a, b = operands(spec, ins)
    want = a @ b
    tensors["matmul"].fill_(float("nan"))
    prob.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    assert_gemm_close(tensors["matmul"].cpu().numpy().reshape(512, 512), want)
    graph = prob.capture(tensors)
    tensors["matmul"].fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert_gemm_close(tensors["matmul"].cpu().numpy().reshape(512, 512), want)
    assert prob.module.status() == 0


def test_gemm_graph_replay(cuda) -> None:
    """The tcgen05 template (tensor maps in module globals, a paired persistent grid) captured
    as a CUDA graph replays to the eager launch's result bit for bit."""
    import numpy as np
    import torch

    from ptxgen.runtime import Problem

    spec = problems.matmul(512, 512, 512)
    ins = reference_inputs(spec.meta)
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    for name, arr in ins.items():
        tensors[name].copy_(torch.from_numpy(arr.reshape(-1).view(np.int16)).view(torch.bfloat16))
    prob.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    eager = tensors["matmul"].clone()
    graph = prob.capture(tensors)
    tensors["matmul"].fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(tensors["matmul"], eager)
    assert prob.module.status() == 0

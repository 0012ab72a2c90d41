"""Benchmark of the B200 ptxgen backend: kernel throughput against the HBM / tensor roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

For N > 1 launch one process per GPU with torchrun (``--nproc-per-node N``); ranks share each
configuration's Tile axis (``ptxgen.shard``), and only the full sum all-reduces its partials.

A step is one launch of the workload's kernel over its whole (per-rank) input, compiled from
Kernel IR by this repository's compiler and launched through its C-ABI launcher, with the inputs
already resident in HBM. L2 is flushed before every timed step, outside the kernel's CUDA
events: a 256 MiB write, then a 256 MiB read, so no input line is in L2 and the flush's own dirty
lines are written back before the step starts (``--l2``). The printed ``value`` is the whole job's algorithmic bytes (or flops) per
second over the slowest rank's mean kernel time; ``e2e`` is the same metric through the one-call
host-buffer path (``pg_run_host``: page-locked inputs copied in, launch, result copied out;
two steps in flight on two streams).
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path
from typing import Any

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "emmy-hackathon-submission_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

DEFAULT_WORKLOAD = "c2_gelu_chain"  # the configuration BASELINE.json's metric is quoted on
EXTRA_WORKLOADS = ("c1_vector_add", "c3_row_softmax", "c4_full_sum", "c5_matmul",
                   "c5b_matmul_splitk")
FLUSH_BYTES = 256 << 20
IDLE_BETWEEN_S = 1.0  # idle time before each of the other configurations is measured


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--workload", default=DEFAULT_WORKLOAD)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-extras", action="store_true", help="skip the other configurations")
    p.add_argument("--scaling", choices=("strong", "weak"), default="strong",
                   help="strong (default): the N GPUs split the configuration's fixed size "
                        "(BASELINE's problem at every N); weak: each GPU keeps a full "
                        "benchmark-sized share of an N-times larger problem (a different, larger "
                        "configuration at N > 1)")
    p.add_argument("--share", type=int, default=1,
                   help="on one GPU, run one share of a K-way strong split of the workload (a "
                        "smaller case of the same kernel, e.g. for a profiler capture)")
    p.add_argument("--l2", choices=("clean", "write", "none"), default="clean",
                   help="clean (default): flush L2 before each timed step with a 256 MiB write "
                        "followed by a 256 MiB read, so no input line is in L2 and the flush's "
                        "own dirty lines are written back before the step starts; write: the "
                        "write alone, which leaves L2 full of dirty lines that the timed kernel "
                        "then writes back (up to 126 MB charged to it); none: no flush, steps "
                        "back to back over inputs larger than L2 (each step writes back the "
                        "previous step's dirty lines, the steady state)")
    p.add_argument("--ablation", action="store_true",
                   help="instead of the benchmark: time the reference's shipped example kernels "
                        "under each compiler flag (its published ablation tables), one JSON line")
    p.add_argument("--collective", choices=("fused", "peer", "nccl"), default="fused",
                   help="how the sharded sum's partials are summed across ranks: inside the sum "
                        "kernel (its last block exchanges over NVLink peer memory), by a "
                        "separate one-warp kernel over peer memory, or by NCCL")
    p.add_argument("--splitk-shard", choices=("m", "k"), default="m",
                   help="how the split-K GEMM divides across ranks: along M (default: rows of A "
                        "and C, B replicated, no collective) or along K (each rank 1/N of A and "
                        "B, the partial C reduce-scattered by rows over NCCL)")
    p.add_argument("--e2e-lanes", type=int, default=2,
                   help="steps of the host-buffer (e2e) path in flight at once, one stream each")
    p.add_argument("--only", default=None,
                   help="with --ablation: time only this shipped example (e.g. m01_matmul_512)")
    p.add_argument("--flags", default=None, choices=("default", "no_loop_unroll", "no_fusion",
                                                     "no_cse"),
                   help="with --ablation: time only this flag set")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="target seconds of CPU work for the CPU baseline sample")
    return p.parse_args()


# --- distributed plumbing ----------------------------------------------------------------------


_T0 = time.perf_counter()


def log(msg: str) -> None:
    """Progress on stderr (stdout carries only the JSON line)."""
    rank = os.environ.get("RANK", "0")
    print(f"[bench r{rank} {time.perf_counter() - _T0:7.1f}s] {msg}", file=sys.stderr, flush=True)


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def init_dist(world: int, local_rank: int) -> Any:
    import torch
    import torch.distributed as dist

    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    return dist


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --- peaks, clocks, profiles -------------------------------------------------------------------


def peaks() -> tuple[dict[str, float], str]:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tensor": float(d["bf16_tflops"]),
                "tensor_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))}, \
            "measured"
    return {"hbm": 6650.0, "tensor": 1590.0, "tensor_sustained": 1400.0}, "fallback"


def ptx_sha16(ptx: str) -> str:
    import hashlib

    return hashlib.sha256(ptx.encode()).hexdigest()[:16]


def traffic_of(workload: str, ptx: str) -> tuple[float | None, dict[str, Any]]:
    """DRAM bytes (read + write) of one launch of the workload's kernel from the committed ncu
    summary ``profiles/traffic.json``, and where the figure comes from. Each entry names the
    sha-256 (first 16 hex digits) of the PTX module it was captured on; if the kernel compiled
    now differs, the figure no longer describes it and no traffic is reported."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None, {"file": None}
    entry = json.loads(f.read_text()).get(workload)
    if not isinstance(entry, dict):
        return None, {"file": "profiles/traffic.json", "entry": None}
    now = ptx_sha16(ptx)
    src = {"file": "profiles/traffic.json", "profile": entry.get("profile"),
           "captured_on_ptx_sha16": entry.get("ptx_sha16"), "kernel_ptx_sha16": now,
           "how": entry.get("how")}
    if entry.get("ptx_sha16") != now:
        src["stale"] = True
        return None, src
    return float(entry["bytes"]), src


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML while the timed region runs."""

    REASONS = {0x2: "applications_clocks", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clocks"}

    def __init__(self, index: int):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz: int | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - no NVML: report no clocks
            self.nvml = None

    # NVML's cumulative violation counters: time spent held below the requested clocks, by cause
    POLICIES = {"power": 0, "thermal": 1, "sync_boost": 2, "board_limit": 3, "reliability": 5}

    def _violations(self) -> dict[str, int]:
        out = {}
        for name, policy in self.POLICIES.items():
            try:
                out[name] = int(self.nvml.nvmlDeviceGetViolationStatus(self.h, policy)
                                .violationTime)
            except Exception:  # noqa: BLE001 - a policy this device does not report
                pass
        return out

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h,
                                                                     self.nvml.NVML_CLOCK_SM))
                bits = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.reasons |= {n for b, n in self.REASONS.items() if bits & b}
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.0002)

    def __enter__(self) -> ClockSampler:
        self.violation_ns: dict[str, int] = {}
        if self.nvml is not None:
            self._v0 = self._violations()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
            v1 = self._violations()
            self.violation_ns = {n: v1[n] - self._v0[n] for n in v1 if n in self._v0}

    def summary(self) -> dict[str, Any]:
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples),
                "violation_us": {n: round(v / 1e3, 1) for n, v in self.violation_ns.items()}}


# --- inputs ------------------------------------------------------------------------------------


def device_tensors(prob: Any, seed: int) -> dict[str, Any]:
    """Every argument of the problem on the GPU; inputs drawn on the device from their
    configured distribution (bf16 rounded to nearest even), outputs left for the kernel."""
    import torch

    tensors = prob.allocate()
    gen = torch.Generator(device="cuda").manual_seed(seed)
    for i, a in enumerate(prob.launch_entry["args"]):
        t = tensors[a["name"]]
        if a.get("output"):
            continue
        if "data" in a:
            t.copy_(torch.tensor(a["data"], dtype=torch.float32).to(t.dtype))
            continue
        dist = a.get("dist", ["normal", 0.0, 1.0])
        f = torch.empty(t.numel(), dtype=torch.float32, device=t.device)
        if dist[0] == "uniform":
            f.uniform_(dist[1], dist[2], generator=gen)
        else:
            f.normal_(dist[1], dist[2], generator=gen)
        t.copy_(f.to(t.dtype))
        del f
    return tensors


# --- result checks -------------------------------------------------------------------------------

CHECK_ROWS = 16  # sampled rows of C per rank for the full-K GEMM (all rows for split-K)

CHECK_BARS = {
    "c1_vector_add": "bit-exact against torch x + y",
    "c2_gelu_chain": "|y - ref| <= 2^-7 |ref| + 1e-5 against torch's f32 gelu(a*x+b, tanh) * s",
    "c3_row_softmax": "|y - ref| <= 1e-4 |ref| + 1e-9 against torch.softmax, and every row sums "
                      "to 1 within 1e-4",
    "c4_full_sum": "the total within rel 1e-5 of the f64 sum of every rank's data",
    "c5_matmul": f"{CHECK_ROWS} rows of C (first, last, seeded picks) of every rank: "
                 "|C - ref| <= 1e-2 |ref| + 1e-4 max|ref| against the f64 product",
    "c5b_matmul_splitk": "every row of C of every rank: |C - ref| <= 1e-2 |ref| + 1e-4 max|ref| "
                         "against the f64 product",
}


def check_output(name: str, plan: Any, tensors: dict[str, Any], world: int) -> dict[str, Any]:
    """Check one rank's result after the timed steps against a torch evaluation of the same
    configuration on the same device data (the rank's own shard; the sum's total against the
    f64 sum over every rank's data), and agree on the outcome across ranks: the check passes
    only if it passes on every rank. Works on CPU tensors too (a gloo group)."""
    import torch

    args = {a["name"]: a for a in plan.spec.kernel["args"]}

    def view(n: str) -> Any:
        return tensors[n][: int(np.prod(args[n]["shape"]))].view(*args[n]["shape"])

    dev = tensors[next(iter(tensors))].device
    total = None
    if name == "c1_vector_add":
        ok = bool(torch.equal(view("add"), view("x") + view("y")))
        err = 0.0 if ok else float((view("add") - (view("x") + view("y"))).abs().max())
    elif name == "c2_gelu_chain":
        a, b = view("mul_c1").float()[0], view("add_c1").float()[0]
        u = view("x").float() * a + b
        ref = torch.nn.functional.gelu(u, approximate="tanh") * view("s").float()[:, None]
        diff = (view("mul_1").float() - ref).abs()
        ok = bool((diff <= 2.0 ** -7 * ref.abs() + 1e-5).all())
        err = float(diff.max())
    elif name == "c3_row_softmax":
        got = view("softmax")
        ref = torch.softmax(view("x"), dim=-1)
        diff = (got - ref).abs()
        rows = (got.sum(dim=-1, dtype=torch.float64) - 1.0).abs()
        ok = bool((diff <= 1e-4 * ref.abs() + 1e-9).all()) and bool((rows <= 1e-4).all())
        err = float(diff.max())
    elif name == "c4_full_sum":
        part = torch.sum(view("x"), dtype=torch.float64).reshape(1)
        if world > 1:
            import torch.distributed as tdist

            tdist.all_reduce(part)
        total = float(part.item())
        got = float(view("sum_1").double()[0])
        err = abs(got - total) / max(abs(total), 1e-30)
        ok = err <= 1e-5
    elif name == "c5b_matmul_splitk" and plan.reduce_scatter and world > 1:
        # each rank holds a K slice of A and B: the product is the sum over ranks of the f64
        # products of the slices; this rank's rows of it against the rows it was left with
        import torch.distributed as tdist

        part = view("x0").double() @ view("x1").double()
        tdist.all_reduce(part)
        rank = tdist.get_rank()
        got = tensors["matmul@rows"]
        ref = part[rank * got.shape[0]:(rank + 1) * got.shape[0]]
        diff = (got.double() - ref).abs()
        ok = bool((diff <= 1e-2 * ref.abs() + 1e-4 * ref.abs().max()).all())
        err = float(diff.max() / ref.abs().max())
    elif name in ("c5_matmul", "c5b_matmul_splitk"):
        a, b, c = view("x0"), view("x1"), view("matmul")
        m = a.shape[0]
        if name == "c5_matmul" and m > CHECK_ROWS:
            g = torch.Generator().manual_seed(7)
            picks = torch.randperm(m - 2, generator=g)[: CHECK_ROWS - 2] + 1
            rows = torch.cat([torch.tensor([0, m - 1]), picks]).to(dev)
        else:
            rows = torch.arange(m, device=dev)
        bd = b.double()
        ref = a.index_select(0, rows).double() @ bd
        del bd
        diff = (c.index_select(0, rows).double() - ref).abs()
        ok = bool((diff <= 1e-2 * ref.abs() + 1e-4 * ref.abs().max()).all())
        err = float(diff.max() / ref.abs().max())
    else:
        raise KeyError(name)
    flag = torch.tensor([1.0 if ok else 0.0], dtype=torch.float64, device=dev)
    worst = torch.tensor([err], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as tdist

        tdist.all_reduce(flag, op=tdist.ReduceOp.MIN)
        tdist.all_reduce(worst, op=tdist.ReduceOp.MAX)
    res = {"result": "pass" if flag.item() == 1.0 else "fail", "bar": CHECK_BARS[name],
           "max_err": float(worst.item()), "ranks": world}
    if total is not None:
        res["f64_total"] = total
    return res


# --- measurement ---------------------------------------------------------------------------------


L2_MODES = {
    "clean": "flushed before every timed step: a 256 MiB write, then a 256 MiB read (no input "
             "line in L2, and the flush's dirty lines written back before the step)",
    "write": "flushed (256 MiB write) before every timed step; the timed kernel writes back the "
             "flush's dirty lines",
    "none": "not flushed: inputs larger than L2 (126 MB), steps back to back in steady state",
}


def measure_kernel(plan: Any, steps: int, warmup: int, world: int, l2: str = "clean",
                   via: str = "peer") -> dict[str, Any]:
    """Mean kernel time over ``steps`` timed launches (each after an L2 flush), the slowest
    rank's, with the launch count and NVML clocks of the timed region."""
    import torch

    from ptxgen.runtime import Problem

    rank = int(os.environ.get("RANK", 0))
    prob = Problem(plan.spec.graph, plan.spec.meta)
    prob.load()
    tensors = device_tensors(prob, seed=1000 + rank)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    reread = torch.zeros(FLUSH_BYTES if l2 == "clean" else 8, dtype=torch.uint8, device="cuda")
    sink = torch.empty((), dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()

    def flush_l2() -> None:
        if l2 == "none":
            return
        flush.zero_()
        if l2 == "clean":
            torch.sum(reread.view(torch.int64), dim=(0,), out=sink)

    collective = bool(plan.allreduce or plan.reduce_scatter) and world > 1
    # the kernel sums its (scalar) partial across ranks itself
    fused = collective and via == "fused" and bool(plan.allreduce)
    mids: list[Any] = []
    peer = slots = None
    if collective and via == "peer" and plan.allreduce:
        from ptxgen.peer import PeerSum

        peer = PeerSum()
    if fused:
        from ptxgen.peer import PeerSlots, bind_exchange

        slots = PeerSlots()
        bind_exchange(prob.module, slots)

    def combine(t: Any, s: Any) -> None:
        """The path's collective: this rank's partial summed over the ranks, in place."""
        if peer is not None:
            peer(t.data_ptr(), stream=s.cuda_stream)
        else:
            import torch.distributed as tdist

            with torch.cuda.stream(s):
                tdist.all_reduce(t)

    # reduce-scattered outputs: this rank's rows of the summed partials
    shapes = {a["name"]: a["shape"] for a in plan.spec.kernel["args"]}
    rows_out = {}
    if collective:
        for name in plan.reduce_scatter:
            m, n = shapes[name]
            rows_out[name] = torch.empty(m // world, n, dtype=tensors[name].dtype,
                                         device=tensors[name].device)

    def step(mid: Any = None) -> None:
        prob.launch(tensors, stream=stream.cuda_stream)
        if collective and not fused:
            if mid is not None:
                mid.record(stream)
            for name in plan.allreduce:
                combine(tensors[name], stream)
            for name, out in rows_out.items():
                import torch.distributed as tdist

                with torch.cuda.stream(stream):
                    tdist.reduce_scatter_tensor(out, tensors[name][:out.numel() * world]
                                                .view(-1, out.shape[1]))

    align = torch.zeros(1, dtype=torch.float32, device="cuda")
    # where the path's collective is over peer memory, the ranks realign over peer memory too:
    # a one-warp exchange kernel releases every rank within NVLink latency of the last one to
    # arrive, where ranks leave a one-element NCCL all-reduce microseconds apart, and a rank that
    # starts its step early is charged the others' lag by the step's own exchange
    aligner = None
    if collective and via in ("fused", "peer") and plan.allreduce:
        from ptxgen.peer import PeerSum

        aligner = PeerSum()

    def realign() -> None:
        """Ranks leave one step's collective together; the L2 flush before the next (not part
        of the workload) takes each rank a different time, so a one-element exchange after it,
        outside the step's events, lines them up again as the previous collective would."""
        if aligner is not None:
            aligner(align.data_ptr(), stream=stream.cuda_stream)
        elif collective:
            import torch.distributed as tdist

            tdist.all_reduce(align)

    for _ in range(warmup):
        flush_l2()
        realign()
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as tdist

        tdist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    sampler = ClockSampler(torch.cuda.current_device())
    if collective and not fused:
        mids = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with sampler:
        for i in range(steps):
            flush_l2()
            realign()
            starts[i].record(stream)
            step(mids[i] if mids else None)
            stops[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as tdist

        tdist.barrier()
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) for s, e in zip(starts, stops, strict=True)]
    mean_ms = statistics.fmean(times)
    if mids:  # this rank's split of its step: its own kernel, then the collective's wait
        kern = statistics.fmean(s.elapsed_time(m) for s, m in zip(starts, mids, strict=True))
        log(f"{plan.name}: kernel {kern * 1e3:.1f} us, collective {(mean_ms - kern) * 1e3:.1f} us "
            "(this rank)")
    status = prob.module.status()
    if status:
        raise RuntimeError(f"kernel status word 0x{status:08x}")
    if peer is not None:
        peer.check()
    if aligner is not None:
        aligner.check()
    out = {"mean_ms": max_over_ranks(mean_ms, world),
           "median_ms": max_over_ranks(statistics.median(times), world),
           "min_ms": max_over_ranks(min(times), world),
           # this backend's kernels per step: the workload's own, and a zero kernel of its
           # module for each zero_outputs buffer it clears in place of a memset
           "launches": steps * (1 + sum(n in prob.module.zeroers
                                        for n in prob.launch_entry.get("zero_outputs", []))),
           "clocks": sampler.summary(),
           "tensors": {**tensors, **{f"{n}@rows": t for n, t in rows_out.items()}},
           "prob": prob, "peer": peer, "slots": slots, "aligner": aligner}
    return out


def _host_lane(prob: Any, tensors: dict[str, Any], stream: int) -> dict[str, Any]:
    """One lane of the host-buffer path: page-locked copies of the inputs and room for the
    outputs, and the ``pg_run_host`` arguments over ``prob``'s device buffers on ``stream``."""
    import torch

    launch = prob.launch_entry
    host, dev, nbytes, flags, keep = [], [], [], [], []
    h2d = d2h = 0
    zero = set(launch.get("zero_outputs", []))
    for name in launch["arg_order"]:
        a = next(x for x in launch["args"] if x["name"] == name)
        t = tensors[name]
        size = t.numel() * t.element_size()
        pinned = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
        f = 0
        if not a.get("output"):
            pinned.copy_(t)
            f |= 1
            h2d += size
        if name in zero:
            f |= 2
        if a.get("output"):
            f |= 4
            d2h += size
        keep.append(pinned)
        host.append(pinned.data_ptr())
        dev.append(t.data_ptr())
        nbytes.append(size)
        flags.append(f)
    prob.module.fill_tensormaps({n: tensors[n].data_ptr() for n in tensors})
    args = (prob.grid(), launch["block"][0], int(launch.get("smem_bytes", 0)), stream,
            dev, host, nbytes, flags)
    cols = {a["name"]: a["shape"][-1] for a in launch["args"]}
    return {"kernel": prob.load(), "args": args, "keep": keep, "tensors": tensors, "cols": cols,
            "h2d": h2d, "d2h": d2h}


def measure_e2e(plan: Any, prob: Any, tensors: dict[str, Any], steps: int, world: int,
                in_flight: int = 2, peer: Any = None, fused: bool = False) -> dict[str, Any]:
    """The same metric through ``pg_run_host``, the one-call host-buffer API: every step copies
    its page-locked inputs in, zeroes its zero_outputs, launches, copies its outputs back and
    waits. ``in_flight`` steps run at a time, each lane with its own module, buffers and
    stream, so one step's upload overlaps another's download on the full-duplex link (a
    workload with a collective keeps one lane, its partial summed over the ranks after each
    step by ``peer`` when given, else by NCCL, or inside the kernel when ``fused``). The value is
    all steps' work over the wall time from the first call to the last return."""
    import torch

    from ptxgen.runtime import Problem

    lanes = [_host_lane(prob, tensors, torch.cuda.Stream().cuda_stream)]
    collective = bool(plan.allreduce or plan.reduce_scatter) and world > 1
    while len(lanes) < in_flight and not collective:
        other = Problem(plan.spec.graph, plan.spec.meta)
        other.load()
        lanes.append(_host_lane(other, {n: t.clone() for n, t in tensors.items()},
                                torch.cuda.Stream().cuda_stream))
    for lane in lanes:  # warm each path once
        lane["kernel"].run_host(*lane["args"])
    torch.cuda.synchronize()

    def run(lane: dict[str, Any], count: int) -> None:
        for _ in range(count):
            lane["kernel"].run_host(*lane["args"])
            if plan.reduce_scatter and world > 1:
                import torch.distributed as tdist

                for name in plan.reduce_scatter:
                    full = lane["tensors"][name]
                    rows = torch.empty(full.numel() // world // lane["cols"][name],
                                       lane["cols"][name], dtype=full.dtype, device=full.device)
                    tdist.reduce_scatter_tensor(rows, full.view(-1, lane["cols"][name]))
                torch.cuda.synchronize()
            if plan.allreduce and world > 1 and not fused:
                import torch.distributed as tdist

                for name in plan.allreduce:
                    if peer is not None:
                        peer(lane["tensors"][name].data_ptr(), stream=lane["args"][3])
                    else:
                        tdist.all_reduce(lane["tensors"][name])
                torch.cuda.synchronize()

    shares = [steps // len(lanes) + (i < steps % len(lanes)) for i in range(len(lanes))]
    workers = [threading.Thread(target=run, args=(lane, n)) for lane, n in zip(lanes, shares)]
    t0 = time.perf_counter()
    for w in workers:
        w.start()
    for w in workers:
        w.join()
    total = time.perf_counter() - t0
    mean_s = max_over_ranks(total / steps, world)
    return {"mean_s": mean_s, "h2d": lanes[0]["h2d"], "d2h": lanes[0]["d2h"],
            "in_flight": len(lanes)}


def pcie_bandwidth(nbytes: int = 256 << 20, reps: int = 3) -> dict[str, float]:
    """Measured page-locked copy bandwidth of this GPU's host link, the bound of the e2e path:
    host-to-device alone, device-to-host alone, and both at once on two streams (total bytes of
    both directions over the time both take). Best of ``reps``, CUDA events, GB/s."""
    import torch

    host_in = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_out = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev_in = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dev_out = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    up, down = torch.cuda.Stream(), torch.cuda.Stream()

    def timed(h2d: bool, d2h: bool) -> float:
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            ends = []
            start.record(up)
            down.wait_event(start)
            for on, go, stream in ((h2d, lambda: dev_in.copy_(host_in, non_blocking=True), up),
                                   (d2h, lambda: host_out.copy_(dev_out, non_blocking=True),
                                    down)):
                if on:
                    with torch.cuda.stream(stream):
                        go()
                        ev = torch.cuda.Event(enable_timing=True)
                        ev.record(stream)
                        ends.append(ev)
            torch.cuda.synchronize()
            best = min(best, max(start.elapsed_time(e) for e in ends) / 1e3)
        return best

    h2d, d2h, both = timed(True, False), timed(False, True), timed(True, True)
    return {"h2d_gbs": nbytes / h2d / 1e9, "d2h_gbs": nbytes / d2h / 1e9,
            "bidirectional_gbs": 2 * nbytes / both / 1e9, "bytes": nbytes}


def e2e_floor_s(h2d_bytes: int, d2h_bytes: int, pcie: dict[str, float]) -> float:
    """The shortest time a step's copies can take on the measured link: each direction at its
    own rate, and both together at the measured two-way rate."""
    return max(h2d_bytes / (pcie["h2d_gbs"] * 1e9), d2h_bytes / (pcie["d2h_gbs"] * 1e9),
               (h2d_bytes + d2h_bytes) / (pcie["bidirectional_gbs"] * 1e9))


# inputs the CPU path splits across threads: contiguous rows / elements of each
_SPLIT = {"c1_vector_add": ("x", "y"), "c2_gelu_chain": ("x", "s"), "c3_row_softmax": ("x",),
          "c4_full_sum": ("x",)}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # not Linux
        return os.cpu_count() or 1


class CpuPath:
    """The NumPy path of one configuration (the oracle's direct formulas of its semantics) on
    this host's cores. The inputs are made once; ``run`` times repetitions. The elementwise and
    reduction configurations cut their rows (elements) into one contiguous chunk per thread,
    each evaluated by one thread (NumPy releases the GIL in its array loops); the GEMMs use the
    BLAS's own threads.

    The size is the configuration's full size whenever ``reps`` full-size repetitions are
    estimated (from a small first sample) to fit in ``budget_s`` seconds; otherwise it is the
    largest sample (a whole number of rows) that fits, and ``fraction`` says which share of the
    full size that is. ``value`` figures are scaled by that fraction to the full size's work."""

    def __init__(self, name: str, budget_s: float, reps: int, threads: int = 1):
        from ptxgen import shard

        self.name = name
        split = _SPLIT.get(name)
        self.threads = max(1, threads) if split else 1
        self.work = shard.local_problem(name, 1).work
        self._prepare(min(1 / 4, self.threads / 64))
        probe = min(self.run_once() for _ in range(2))
        want = budget_s / max(1, reps)
        frac = 1.0 if probe / self.fraction <= want else max(self.fraction,
                                                               want / probe * self.fraction)
        if frac != self.fraction:
            self._prepare(frac)
        self.cores = host_threads() if name.startswith("c5") else self.threads

    def _prepare(self, frac: float) -> None:
        from oracle.semantics import FORMULAS
        from ptxgen import problems

        samples = {
            "c1_vector_add": lambda f: problems.pointwise_add(
                max(1 << 12, int((1 << 24) * f) // 256 * 256)),
            "c2_gelu_chain": lambda f: problems.gelu_chain(max(8, int(8192 * f)), 8192),
            "c3_row_softmax": lambda f: problems.row_softmax(max(8, int(16384 * f)), 4096),
            "c4_full_sum": lambda f: problems.full_sum(
                max(1 << 16, int((1 << 30) * f) // 256 * 256)),
            "c5_matmul": lambda f: problems.matmul(max(128, int(8192 * f) // 128 * 128), 8192,
                                                   8192),
            "c5b_matmul_splitk": lambda f: problems.matmul(
                max(128, int(1024 * f) // 128 * 128), 1024, 65536, split_k=4,
                raster_group=None),
        }
        self.fn = FORMULAS[self.name]
        self.parts = []  # free the previous sample's arrays first
        spec = samples[self.name](frac)
        ins = {a["name"]: problems.seeded_input(a) for a in spec.kernel["args"]
               if not a.get("output")}
        split = _SPLIT.get(self.name)
        self.parts = [[ins]]
        if split:
            # each thread's contiguous share, cut again into blocks of about 2^20 elements so a
            # block's temporaries stay in cache and are reused instead of freshly faulted in
            first = ins[split[0]]
            per_row = int(np.prod(first.shape[1:])) if first.ndim > 1 else 1
            rows = first.shape[0]
            nblocks = max(self.threads, -(-rows * per_row // (1 << 20)))
            nblocks = min(rows, -(-nblocks // self.threads) * self.threads)
            cut = {n: np.array_split(ins[n], nblocks) for n in split}
            blocks = [{**ins, **{n: cut[n][i] for n in split}} for i in range(nblocks)]
            share = nblocks // self.threads
            self.parts = [blocks[i * share:(i + 1) * share] for i in range(self.threads)]
        self.spec = spec
        full = problems.CONFIGS[self.name]().kernel["args"]
        self.elements = _elements(spec.kernel["args"])
        self.fraction = self.elements / _elements(full)

    def run_once(self) -> float:
        """Seconds of one repetition over the whole sample."""
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(self.threads) as pool:
            t0 = time.perf_counter()
            list(pool.map(lambda part: [self.fn(b, self.spec.meta) for b in part], self.parts))
            return time.perf_counter() - t0

    def value(self, seconds: float) -> float:
        """The metric's work per second (bytes or flops, not yet in the unit's scale) for one
        repetition that took ``seconds``."""
        return self.work * self.fraction / seconds

    def sample(self, reps: int) -> str:
        size = ("the full size" if self.fraction == 1.0
                else f"{self.fraction:.4f} of the full size")
        return (f"{self.spec.meta['id']} at {size} ({self.elements} input elements), "
                f"{reps} repetitions"
                + (f", split over {self.threads} threads" if self.threads > 1 else ""))


def cpu_baseline(name: str, plan: Any, seconds: float, threads: int = 1) -> dict[str, Any]:
    """The NumPy path of the same configuration timed on this host for about ``seconds``
    (``CpuPath``): the mean over repetitions, at the full size where two repetitions fit."""
    path = CpuPath(name, seconds, 2, threads)
    reps, el = 0, 0.0
    while True:
        el += path.run_once()
        reps += 1
        if el >= seconds or reps >= 1000:
            break
    per_rep = el / reps
    return {"value": path.value(per_rep), "per_rep_s": per_rep, "reps": reps,
            "cores": path.cores, "fraction": path.fraction, "sample": path.sample(reps)}


def _elements(args: list[dict[str, Any]]) -> int:
    return int(sum(np.prod(a["shape"]) for a in args if not a.get("output")))


# --- the two arms --------------------------------------------------------------------------------


def unit_of(plan: Any) -> tuple[str, str, float]:
    if plan.units == "flops":
        return "TFLOP/s", "tensor", 1e12
    return "GB/s", "hbm", 1e9


def run_ours(args: argparse.Namespace) -> None:
    import torch

    from ptxgen import shard
    from ptxgen.build import build_library
    from ptxgen.runtime import init

    rank, world, local_rank = dist_env()
    log(f"start: world {world}, local rank {local_rank}, --gpus {args.gpus}")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}: launch with torchrun")
    torch.cuda.set_device(local_rank)
    init_dist(world, local_rank)
    if rank == 0:
        build_library()
    if world > 1:
        import torch.distributed as tdist

        tdist.barrier()
    init(local_rank)
    pk, pk_kind = peaks()
    if args.share > 1 and world > 1:
        raise SystemExit("--share runs a share of the workload on one GPU; use it without torchrun")

    def plan_for(name: str) -> Any:
        if args.share > 1:
            return shard.local_problem(name, args.share)
        plan = shard.local_problem(name, world, weak=args.scaling == "weak",
                                   ksplit=args.splitk_shard == "k")
        if args.collective == "fused" and plan.allreduce and world > 1:
            import dataclasses

            from ptxgen.peer import with_exchange

            plan = dataclasses.replace(plan, spec=with_exchange(plan.spec, plan.allreduce[0]))
        return plan

    pcie = None

    def one(name: str, steps: int, warmup: int, with_e2e: bool) -> dict[str, Any]:
        nonlocal pcie
        log(f"{name}: compile and inputs")
        plan = plan_for(name)
        unit, bound, scale = unit_of(plan)
        m = measure_kernel(plan, steps, warmup, world, args.l2, args.collective)
        per_rank = plan.work / (m["mean_ms"] / 1e3) / scale
        res: dict[str, Any] = {"workload": name, "value": per_rank * world, "unit": unit,
                               "ms_per_step": m["mean_ms"], "median_ms": m["median_ms"],
                               "min_ms": m["min_ms"], "clocks": m["clocks"],
                               "launches": m["launches"]}
        peak = pk[bound]
        traffic, traffic_src = traffic_of(name, m["prob"].compile())
        res["roofline"] = {"bound": bound, "achieved": per_rank, "peak": peak,
                           "unit": unit, "frac": per_rank / peak,
                           "traffic": traffic, "traffic_source": traffic_src,
                           "peak_source": pk_kind, "algorithmic_per_launch": plan.work}
        log(f"{name}: {res['ms_per_step']:.4f} ms per step, {res['value']:.1f} {unit}")
        res["check"] = check_output(name, plan, m["tensors"], world)
        log(f"{name}: check {res['check']['result']} (max err {res['check']['max_err']:.3g})")
        if with_e2e:
            e = measure_e2e(plan, m["prob"], m["tensors"], max(3, min(steps, 20)), world,
                            args.e2e_lanes, m["peer"], fused=m["slots"] is not None)
            value = plan.work * world / e["mean_s"] / scale
            if pcie is None:
                pcie = pcie_bandwidth()
            floor = e2e_floor_s(e["h2d"], e["d2h"], pcie)
            bound_value = plan.work * world / floor / scale
            res["e2e"] = {"value": value, "unit": unit,
                          "h2d_bytes_per_step": e["h2d"], "d2h_bytes_per_step": e["d2h"],
                          "steps_in_flight": e["in_flight"],
                          "pcie": {k: round(v, 2) for k, v in pcie.items() if k != "bytes"},
                          "pcie_bound": bound_value, "frac_of_pcie": value / bound_value}
        if m["peer"] is not None or m["slots"] is not None:  # all ranks done before unmapping
            import torch.distributed as tdist

            if m["peer"] is not None:
                m["peer"].check()
            tdist.barrier()
            (m["peer"] or m["slots"]).close()
            if m["aligner"] is not None:
                m["aligner"].close()
        del m
        torch.cuda.empty_cache()
        return res

    head = one(args.workload, args.steps, args.warmup, with_e2e=True)
    extras = []
    if not args.no_extras:
        for name in EXTRA_WORKLOADS:
            if name == args.workload:
                continue
            # each configuration starts from an idle GPU: a long GEMM before it holds the power
            # cap, and the clocks it leaves behind would be charged to the next one
            time.sleep(IDLE_BETWEEN_S)
            try:
                r = one(name, min(args.steps, 20), min(args.warmup, 3), with_e2e=False)
                extras.append({k: r[k] for k in ("workload", "value", "unit", "ms_per_step",
                                                 "roofline", "check", "clocks")})
            except Exception as e:  # noqa: BLE001 - report and continue
                extras.append({"workload": name, "error": f"{type(e).__name__}: {e}"[:300]})
    log("measurements done")
    failed = [head["workload"]] if head["check"]["result"] != "pass" else []
    failed += [x["workload"] for x in extras
               if "error" in x or x.get("check", {}).get("result") != "pass"]
    if rank != 0:
        if failed:
            raise SystemExit(f"result check failed: {', '.join(failed)}")
        return
    plan = plan_for(args.workload)
    cpu = None
    if world == 1:
        cpu = cpu_baseline(args.workload, plan, args.cpu_seconds, host_threads())
    line = {
        "metric": METRIC,
        "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": _dtype(args.workload),
        "data": "synthetic (seeded, the configuration's distributions, generated on the GPU)",
        "config": config_of(args.workload, world, args.scaling, args.share),
        "setup": {"per_rank": plan.spec.meta["id"],
                  "parallelism": f"tile-axis x{world}" if world > 1 else "single GPU",
                  "l2": L2_MODES[args.l2],
                  "allreduce": list(plan.allreduce),
                  "reduce_scatter": list(plan.reduce_scatter),
                  "collective": ({"fused": "inside the sum kernel: its last block exchanges "
                                           "the partials over NVLink peer memory",
                                  "peer": "a separate one-warp kernel over NVLink peer memory",
                                  "nccl": "NCCL all-reduce"}[args.collective]
                                 if plan.allreduce and world > 1 else
                                 "NCCL reduce-scatter of the partial C by rows"
                                 if plan.reduce_scatter and world > 1 else None)},
        "check": head["check"]["result"] if not failed else "fail",
        "checks": {head["workload"]: head["check"],
                   **{x["workload"]: x.get("check", {"result": "error"}) for x in extras}},
        "roofline": head["roofline"], "e2e": head["e2e"], "clocks": head["clocks"],
        "gpu_launches": head["launches"],
        "cpu_baseline": cpu and {"value": cpu["value"] / unit_of(plan)[2], "unit": head["unit"],
                                 "cores": cpu["cores"], "kind": "port", "sample": cpu["sample"]},
        "workloads": extras,
    }
    print(json.dumps(line), flush=True)
    if failed:
        raise SystemExit(f"result check failed: {', '.join(failed)}")


METRIC = "Kernel time: HBM GB/s (% of ~8 TB/s), GEMM TFLOPS (% peak) at 1/2/4/8 B200"


def config_of(name: str, world: int, scaling: str, share: int = 1) -> dict[str, Any]:
    """The workload both arms report: the configuration, the whole problem's size, and how
    many ranks share it. The reference arm prints the same dictionary for the same flags."""
    from ptxgen import shard

    size = list(shard.SIZES[name])
    if scaling == "weak":
        size[0] *= world
    cfg = {"workload": name, "size": size, "scaling": scaling, "ranks": world,
           "split": shard.SPLIT_AXIS[name]}
    if share > 1:
        cfg["share"] = f"1/{share} of the workload on one GPU"
    return cfg


def _dtype(name: str) -> str:
    return {"c1_vector_add": "f32", "c2_gelu_chain": "bf16 (f32 compute)",
            "c3_row_softmax": "f32", "c4_full_sum": "f32", "c5_matmul": "bf16 (f32 accumulate)",
            "c5b_matmul_splitk": "bf16 (f32 accumulate)"}[name]


def run_reference(args: argparse.Namespace) -> None:
    """The CPU path of the same configuration (the NumPy port of its semantics, the oracle's
    formulas) on this host's cores, one repetition per step: the full problem at every N (the
    strong-scaling configuration's whole size), or a stated fraction of it when the steps would
    not fit in a few minutes. Under torchrun rank 0 alone runs it; the others exit."""
    from ptxgen import shard

    rank, world, _ = dist_env()
    if rank != 0:
        return
    plan = shard.local_problem(args.workload, 1)
    unit, _, scale = unit_of(plan)
    reps = args.steps + args.warmup
    path = CpuPath(args.workload, max(args.cpu_seconds, 120.0), reps, host_threads())
    times = [path.run_once() for _ in range(reps)][args.warmup:]
    mean_s = statistics.fmean(times)
    value = path.value(mean_s) / scale
    line = {
        "metric": METRIC,
        "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_s * 1e3, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": _dtype(args.workload),
        "data": "synthetic (seeded NumPy inputs)", "impl": "reference",
        "config": config_of(args.workload, world, args.scaling, args.share),
        "setup": {"parallelism": "host CPU", "sample_fraction": path.fraction},
        "cpu_baseline": {"value": value, "unit": unit, "cores": path.cores, "kind": "port",
                         "sample": path.sample(len(times))},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


GRAPH_LAUNCHES = 20
ABLATION_FLAGS = {"default": {}, "no_loop_unroll": {"no_unroll": True},
                  "no_fusion": {"no_fusion": True}, "no_cse": {"no_cse": True}}


def run_ablation(args: argparse.Namespace) -> None:
    """The reference's published numbers are flag ablations of its shipped example kernels
    (median kernel time with and without loop unrolling, fusion and CSE). This times the same
    kernels, compiled here for sm_100a. Two timings per kernel: the median of per-launch
    CUDA-event times (``pg_kernel_time``, launches enqueued one by one from the host), and the
    median over replays of a CUDA graph of ``GRAPH_LAUNCHES`` back-to-back launches divided by
    that count -- for a kernel of a few microseconds the host enqueues slower than the GPU runs,
    and only the graph keeps the GPU busy from one launch to the next."""
    import torch

    from ptxgen.build import build_library
    from ptxgen.problems import seeded_input
    from ptxgen.runtime import Problem, capture_launches, init

    build_library()
    init(0)
    shipped = ROOT / "tests" / "golden" / "shipped"
    table = []
    for d in sorted(p for p in shipped.iterdir() if p.is_dir()):
        if args.only and d.name != args.only:
            continue
        graph = json.loads(next(d.glob("*.ir.json")).read_text())
        meta = json.loads((d / "meta.json").read_text())
        row: dict[str, Any] = {"problem": d.name}
        for label, flags in ABLATION_FLAGS.items():
            if args.flags and label != args.flags:
                continue
            prob = Problem(graph, meta, flags=flags)
            tensors = prob.allocate()
            for i, a in enumerate(prob.launch_entry["args"]):
                if a.get("output"):
                    tensors[a["name"]].zero_()
                    continue
                arg = dict(a)
                if "seed" in arg:
                    arg["seed"] = meta["graph_inputs"].index(a["name"])
                tensors[a["name"]].copy_(torch.from_numpy(seeded_input(arg).reshape(-1)))
            ms = prob.time(tensors, warmup=10, reps=max(20, args.steps))
            row[f"{label}_us"] = statistics.median(ms) * 1e3
            replayed = capture_launches([prob] * GRAPH_LAUNCHES, tensors)
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            per = []
            for _ in range(max(10, args.steps // 2)):
                start.record()
                replayed.replay()
                stop.record()
                stop.synchronize()
                per.append(start.elapsed_time(stop) / GRAPH_LAUNCHES)
            row[f"{label}_graph_us"] = statistics.median(per) * 1e3
            del replayed
        table.append(row)
        log(f"{d.name}: " + ", ".join(f"{k} {v:.2f}" for k, v in row.items() if k != "problem"))
    print(json.dumps({"ablation": table, "unit": "us (median kernel time)",
                      "timing": "*_us: pg_kernel_time, one event pair per host-enqueued launch; "
                                f"*_graph_us: a CUDA graph of {GRAPH_LAUNCHES} back-to-back "
                                "launches per replay, divided; L2 warm",
                      "gpu": torch.cuda.get_device_name(0)}))


def main() -> None:
    args = parse_args()
    if args.ablation:
        run_ablation(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    run_ours(args)
    rank, world, _ = dist_env()
    if world > 1:
        import torch.distributed as tdist

        tdist.destroy_process_group()


if __name__ == "__main__":
    main()

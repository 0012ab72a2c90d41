"""Multi-rank host logic on CPU: gloo ranks (world size 2) run the per-rank problems of
``ptxgen.shard`` through the oracle on their slices of one seeded input, combine them, and the
result must be the unsharded problem's. A second test makes one rank fail before the collective
and checks that the other rank errors out within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import pickle
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]

SMALL = {"c1_vector_add": (4096,), "c2_gelu_chain": (16, 256), "c3_row_softmax": (8, 512),
         "c4_full_sum": (1 << 18,), "c5_matmul": (256, 256, 128),
         "c5b_matmul_splitk": (256, 256, 1024)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    for p in (str(ROOT), str(ROOT / "emmy-hackathon-submission_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _sharded_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _setup(rank, world, port)
    import torch.distributed as dist

    from oracle.interp import run_kernel
    from ptxgen import problems, shard

    results = {}
    for name, size in SMALL.items():
        full = shard.local_problem(name, 1, size)
        ins = {a["name"]: problems.seeded_input(a) for a in full.spec.kernel["args"]
               if not a.get("output")}
        plan = shard.local_problem(name, world, size, ksplit=True)
        local = plan.slice_inputs(ins, rank)
        out = run_kernel(plan.spec.graph, plan.spec.meta, local)
        out = plan.combine(out)
        gathered: list = [None] * world
        dist.all_gather_object(gathered, out)
        results[name] = gathered
    dist.barrier()
    if rank == 0:
        Path(out_dir, "sharded.pkl").write_bytes(pickle.dumps(results))
    dist.destroy_process_group()


def test_sharded_plans_equal_unsharded(tmp_path) -> None:
    import torch.multiprocessing as mp

    from oracle.interp import run_kernel
    from ptxgen import problems, shard

    world = 2
    mp.spawn(_sharded_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    results = pickle.loads((tmp_path / "sharded.pkl").read_bytes())
    for name, size in SMALL.items():
        full = shard.local_problem(name, 1, size)
        ins = {a["name"]: problems.seeded_input(a) for a in full.spec.kernel["args"]
               if not a.get("output")}
        want = run_kernel(full.spec.graph, full.spec.meta, ins)
        plan = shard.local_problem(name, world, size, ksplit=True)
        for out, ref in want.items():
            parts = [r[out] for r in results[name]]
            if out in plan.reduce_scatter:  # K-split partials summed: f32 order differs
                got = np.concatenate(parts, axis=0)
                np.testing.assert_allclose(got.astype(np.float64), ref.astype(np.float64),
                                           rtol=1e-5, atol=1e-5 * np.abs(ref).max())
            elif out in plan.allreduce:
                for p in parts:  # every rank holds the all-reduced total
                    np.testing.assert_allclose(p.astype(np.float64), ref.astype(np.float64),
                                               rtol=1e-6)
            else:
                got = np.concatenate(parts, axis=0)
                assert np.array_equal(got, ref), f"{name}.{out}: sharded result differs"


def _failing_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    _setup(rank, world, port, timeout_s=5.0)
    import time

    import torch
    import torch.distributed as dist

    if rank == 1:
        os._exit(0)  # a rank that leaves between steps, before the collective
    t0 = time.perf_counter()
    try:
        dist.all_reduce(torch.ones(1))
        outcome = "completed"
    except Exception as e:  # noqa: BLE001 - the error is the expected outcome
        outcome = f"raised {type(e).__name__}"
    Path(out_dir, "rank0.txt").write_text(f"{outcome} after {time.perf_counter() - t0:.1f}s")
    os._exit(0)


def test_lost_rank_raises_instead_of_hanging(tmp_path) -> None:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung past the process-group timeout"
    text = (tmp_path / "rank0.txt").read_text()
    assert text.startswith("raised"), text

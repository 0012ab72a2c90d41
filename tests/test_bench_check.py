"""``bench.py``'s result check on the CPU, over two gloo ranks: each rank holds its shard of a
small configuration with outputs from the oracle's formulas (standing in for the kernel's), and
``check_output`` must pass on both; a mistake planted in one rank's output must fail the check
on both ranks (they agree through the collective). The sum checks the combined total."""

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
         "c4_full_sum": (1 << 16,), "c5_matmul": (256, 256, 128),
         "c5b_matmul_splitk": (256, 256, 1024)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tensors(plan, ins: dict[str, np.ndarray], outs: dict[str, np.ndarray]) -> dict:
    """Flat torch tensors as the bench holds them on the device (bf16 as torch.bfloat16)."""
    import torch

    args = {a["name"]: a for a in plan.spec.kernel["args"]}
    out = {}
    for name, arr in {**ins, **outs}.items():
        flat = np.ascontiguousarray(arr).reshape(-1)
        if args[name]["dtype"] == "bf16":
            out[name] = torch.from_numpy(flat.view(np.int16).copy()).view(torch.bfloat16)
        else:
            out[name] = torch.from_numpy(flat.astype(np.float32, copy=True))
    return out


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "emmy-hackathon-submission_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bench
    from oracle.semantics import FORMULAS
    from ptxgen import problems, shard

    results = {}
    for name, size in SMALL.items():
        full = shard.local_problem(name, 1, size)
        ins = {a["name"]: problems.seeded_input(a) for a in full.spec.kernel["args"]
               if not a.get("output")}
        plan = shard.local_problem(name, world, size, ksplit=True)
        local = plan.slice_inputs(ins, rank)
        outs = FORMULAS[name](local, plan.spec.meta)
        if name == "c4_full_sum":  # every rank holds the combined total, as the exchange leaves it
            outs = plan.combine(outs)
        rows = {}
        if plan.reduce_scatter:  # the K-split GEMM: this rank's rows of the summed partials
            combined = plan.combine(outs)
            import torch
            rows = {f"{n}@rows": torch.from_numpy(np.ascontiguousarray(combined[n]))
                    for n in plan.reduce_scatter}
        good = bench.check_output(name, plan, {**_tensors(plan, local, outs), **rows}, world)
        if plan.reduce_scatter:  # the planted mistake goes into the rows the check reads
            outs = {f"{n}@rows": combined[n] for n in plan.reduce_scatter}
        bad_outs = {k: v.copy() for k, v in outs.items()}
        if rank == 1:  # one wrong element on one rank only
            key = next(iter(bad_outs))
            flat = bad_outs[key].reshape(-1)
            if flat.dtype == np.uint16:
                flat[-1] ^= 0x4000  # flip a high exponent bit of the bf16 value
            else:
                flat[-1] = flat[-1] * 1.01 + 0.5
        if plan.reduce_scatter:
            import torch
            bad_t = {**_tensors(plan, local, FORMULAS[name](local, plan.spec.meta)),
                     **{k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in bad_outs.items()}}
        else:
            bad_t = _tensors(plan, local, bad_outs)
        bad = bench.check_output(name, plan, bad_t, world)
        results[name] = (good, bad)
    dist.barrier()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(results))
    dist.destroy_process_group()


def test_check_passes_and_catches_a_planted_mistake(tmp_path) -> None:
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    per_rank = [pickle.loads((tmp_path / f"rank{r}.pkl").read_bytes()) for r in range(world)]
    for name in SMALL:
        for r in range(world):
            good, bad = per_rank[r][name]
            assert good["result"] == "pass", (name, r, good)
            assert bad["result"] == "fail", (name, r, bad)
            assert good["ranks"] == world and good["bar"]
    total = per_rank[0]["c4_full_sum"][0]["f64_total"]
    assert total == per_rank[1]["c4_full_sum"][0]["f64_total"]


def test_config_is_the_same_for_both_arms() -> None:
    """The GPU arm and the reference arm build ``config`` from the same function: the whole
    problem's size at every rank count under strong scaling."""
    import bench

    one = bench.config_of("c2_gelu_chain", 1, "strong")
    eight = bench.config_of("c2_gelu_chain", 8, "strong")
    assert one["size"] == eight["size"] == [8192, 8192]
    assert eight["ranks"] == 8 and eight["scaling"] == "strong"
    assert bench.config_of("c2_gelu_chain", 8, "weak")["size"] == [8 * 8192, 8192]

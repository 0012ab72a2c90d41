"""The cross-rank sum over peer memory (``ptxgen.peer``, ``templates/exchange.py``).

On the CPU: the kernel assembles for sm_100a, publishes and collects with 64-bit stores and
loads at system scope, bounds its wait by %globaltimer, and loads nothing with cluster
multicast.

On one GPU, three single-kernel cases, none of which waits on another kernel:
1. one rank sums its own partial;
2. two ranks are emulated, the host writing rank 1's word into this rank's slot before the
   launch, so the kernel reads it as if rank 1 had stored it over NVLink;
3. a slot nothing ever fills: the wait gives up after its limit, sets the status bit, and the
   result stays untouched.

On two GPUs (skipped with fewer): two processes, one per GPU, sum 50 rounds of partials and
must both hold the rank-order f32 sum bit for bit.
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from ptxgen.templates.exchange import ENTRY, STATUS_TIMEOUT, peer_sum_ptx

ROOT = Path(__file__).resolve().parents[1]


def test_peer_sum_ptx_assembles(tmp_path) -> None:
    ptx = peer_sum_ptx()
    assert "st.relaxed.sys.global.u64" in ptx and "ld.relaxed.sys.global.u64" in ptx
    assert "%globaltimer" in ptx and "red.global.or.b32 [ptxgen_status]" in ptx
    assert "multicast" not in ptx and "multimem" not in ptx
    if shutil.which("ptxas") is None:
        pytest.skip("no ptxas")
    f = tmp_path / "peer.ptx"
    f.write_text(ptx)
    subprocess.run(["ptxas", "-arch=sm_100a", str(f), "-o", str(tmp_path / "peer.cubin")],
                   check=True, capture_output=True)


def _word(seq: int, value: np.float32) -> np.int64:
    bits = int(np.float32(value).view(np.uint32))
    return np.int64(np.uint64((seq << 32) | bits).view(np.int64))


def _run(cuda, world: int, prefill: dict[int, float], limit_ns: int, seq: int = 1):
    """One launch as rank 0 of ``world`` on this GPU: every peer's slot array is a local
    buffer, and ``prefill`` maps rank -> partial already present in rank 0's slots."""
    import torch

    from ptxgen.runtime import Module

    dev = "cuda:0"
    src = torch.tensor([1.25], dtype=torch.float32, device=dev)
    dst = torch.tensor([-7.0], dtype=torch.float32, device=dev)
    slots = [torch.zeros(2 * world, dtype=torch.int64, device=dev) for _ in range(world)]
    half = (seq & 1) * world
    for p, v in prefill.items():
        slots[0][half + p] = int(_word(seq, np.float32(v)))
    peers = torch.tensor([s.data_ptr() for s in slots], dtype=torch.int64, device=dev)
    mod = Module(peer_sum_ptx())
    mod.kernel(ENTRY).launch(1, 32, 0, [src.data_ptr(), dst.data_ptr(), peers.data_ptr(),
                                        slots[0].data_ptr(), 0, world, seq, limit_ns])
    torch.cuda.synchronize()
    return mod.status(), float(dst.item()), [s.cpu().numpy() for s in slots]


@pytest.mark.gpu
def test_one_rank_sums_its_own_partial(cuda) -> None:
    status, total, slots = _run(cuda, 1, {}, 1_000_000_000)
    assert status == 0 and total == 1.25
    assert slots[0][1] == _word(1, np.float32(1.25))  # seq 1: half (1 & 1) * world, rank 0


@pytest.mark.gpu
def test_emulated_peer_partial_is_summed_in_rank_order(cuda) -> None:
    v1 = np.float32(3.0e-8)
    status, total, slots = _run(cuda, 2, {1: float(v1)}, 1_000_000_000)
    assert status == 0
    assert np.float32(total) == np.float32(np.float32(1.25) + v1)
    # rank 0's partial went into "rank 1's" slots at index (seq & 1) * world + 0
    assert slots[1][2 + 0] == _word(1, np.float32(1.25))


@pytest.mark.gpu
def test_missing_peer_partial_gives_up_and_reports(cuda) -> None:
    status, total, _ = _run(cuda, 2, {}, 10_000_000)  # 10 ms: nothing fills rank 1's slot
    assert status == 1 << STATUS_TIMEOUT
    assert total == -7.0  # the result is left untouched


_WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path[:0] = [sys.argv[1], os.path.join(sys.argv[1], "emmy-hackathon-submission_b200")]
rank, world = int(sys.argv[2]), int(sys.argv[3])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:" + sys.argv[4], rank=rank,
                        world_size=world)
from ptxgen.runtime import init
from ptxgen.peer import PeerSum
init(rank)
ps = PeerSum(device=rank)
x = torch.zeros(1, dtype=torch.float32, device="cuda")
out = []
for i in range(50):
    x.fill_(float(np.float32((rank + 1) * 0.1 + i * 1e-3)))
    ps(x.data_ptr())
    torch.cuda.synchronize()
    out.append(float(x.item()))
ps.check()
dist.barrier()
ps.close()
dist.destroy_process_group()
print("RESULT", " ".join(repr(v) for v in out), flush=True)
"""


@pytest.mark.gpu
def test_two_gpus_agree_on_the_rank_order_sum(cuda, tmp_path) -> None:
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, str(29600 + os.getpid() % 300)
    script = tmp_path / "worker.py"
    script.write_text(_WORKER)
    procs = [subprocess.Popen([sys.executable, str(script), str(ROOT), str(r), str(world), port],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            so, se = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        assert p.returncode == 0, se[-2000:]
        outs.append([float(v) for v in so.split("RESULT", 1)[1].split()])
    for i in range(50):
        parts = [np.float32((r + 1) * 0.1 + i * 1e-3) for r in range(world)]
        want = parts[0]
        for v in parts[1:]:
            want = np.float32(want + v)
        for r in range(world):
            assert np.float32(outs[r][i]) == want, (i, r, outs[r][i], want)


# --- the exchange as the epilogue of the sum kernel itself ----------------------------------------


def _fused_sum(n: int = 1 << 16, blocks: int = 8):
    from ptxgen import problems
    from ptxgen.peer import with_exchange

    return with_exchange(problems.full_sum(n, blocks=blocks), "sum_1")


def test_fused_sum_keeps_the_meta_parameters_and_assembles(tmp_path) -> None:
    from ptxgen.compiler import to_ptx
    from ptxgen.ir import Graph

    spec = _fused_sum()
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    params = re.findall(r"\.param \.u64 (\w+)", ptx)
    assert params == [f"k_sum_1_reduce_param_{a}" for a in spec.meta["kernels"][0]["arg_order"]]
    assert ptx.count("atom.add.acq_rel.gpu.global.u32") == 1
    assert ptx.count("st.relaxed.sys.global.u64") == 1 and "multicast" not in ptx
    if shutil.which("ptxas") is None:
        pytest.skip("no ptxas")
    f = tmp_path / "fused.ptx"
    f.write_text(ptx)
    subprocess.run(["ptxas", "-arch=sm_100a", str(f), "-o", str(tmp_path / "fused.cubin")],
                   check=True, capture_output=True)


class _Slots:
    """A stand-in for ``PeerSlots`` on one GPU: every rank's slot array is a local buffer."""

    def __init__(self, world: int):
        import torch

        self.rank, self.world = 0, world
        self.arrays = [torch.zeros(2 * world, dtype=torch.int64, device="cuda")
                       for _ in range(world)]
        self.slots = self.arrays[0]
        self.peers = torch.tensor([a.data_ptr() for a in self.arrays], dtype=torch.int64,
                                  device="cuda")


def _fused_run(world: int, prefill: dict[int, float], limit_ns: int, launches: int = 1):
    """``launches`` launches of the fused sum of 2^16 ones as rank 0 of ``world``; ``prefill``
    maps rank -> partial already present in rank 0's slots for every launch's sequence number."""
    import torch

    from ptxgen.peer import bind_exchange
    from ptxgen.runtime import Problem

    spec = _fused_sum()
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    tensors["x"].fill_(1.0)
    fake = _Slots(world)
    bind_exchange(prob.module, fake, limit_ns)
    out = []
    for seq in range(1, launches + 1):
        for p, v in prefill.items():
            fake.slots[(seq & 1) * world + p] = int(_word(seq, np.float32(v)))
        prob.launch(tensors)
        torch.cuda.synchronize()
        out.append(float(tensors["sum_1"].item()))
    return prob.module.status(), out, [a.cpu().numpy() for a in fake.arrays]


@pytest.mark.gpu
def test_fused_sum_one_rank(cuda) -> None:
    status, out, _ = _fused_run(1, {}, 1_000_000_000, launches=3)
    assert status == 0 and out == [65536.0] * 3  # the block counter resets between launches


@pytest.mark.gpu
def test_fused_sum_emulated_peer(cuda) -> None:
    status, out, arrays = _fused_run(2, {1: 0.5}, 1_000_000_000, launches=2)
    assert status == 0 and out == [65536.5, 65536.5]
    assert arrays[1][0] == _word(2, np.float32(65536.0))  # seq 2's word to "rank 1", slot 0


@pytest.mark.gpu
def test_fused_sum_missing_peer_gives_up(cuda) -> None:
    status, out, _ = _fused_run(2, {}, 10_000_000)
    assert status == 1 << STATUS_TIMEOUT
    assert out == [65536.0]  # the rank's own partial, not a total


_FUSED_WORKER = r"""
import os, sys, torch, torch.distributed as dist
sys.path[:0] = [sys.argv[1], os.path.join(sys.argv[1], "emmy-hackathon-submission_b200")]
rank, world = int(sys.argv[2]), int(sys.argv[3])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:" + sys.argv[4], rank=rank,
                        world_size=world)
from ptxgen import problems
from ptxgen.peer import PeerSlots, bind_exchange, check_exchange, with_exchange
from ptxgen.runtime import Problem, init
init(rank)
spec = with_exchange(problems.full_sum(1 << 20, blocks=64), "sum_1")
prob = Problem(spec.graph, spec.meta, device=rank)
t = prob.allocate()
t["x"].fill_(float(rank + 1))
slots = PeerSlots(device=rank)
bind_exchange(prob.module, slots)
out = []
for i in range(20):
    prob.launch(t)
    torch.cuda.synchronize()
    out.append(float(t["sum_1"].item()))
check_exchange(prob.module)
dist.barrier()
slots.close()
dist.destroy_process_group()
print("RESULT", " ".join(repr(v) for v in out), flush=True)
"""


@pytest.mark.gpu
def test_two_gpus_fused_sum(cuda, tmp_path) -> None:
    """Rank r sums 2^20 copies of r + 1 (exact in f32): both ranks must hold 3 * 2^20."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, str(29900 + os.getpid() % 90)
    script = tmp_path / "fused_worker.py"
    script.write_text(_FUSED_WORKER)
    procs = [subprocess.Popen([sys.executable, str(script), str(ROOT), str(r), str(world), port],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in range(world)]
    for p in procs:
        try:
            so, se = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        assert p.returncode == 0, se[-2000:]
        got = [float(v) for v in so.split("RESULT", 1)[1].split()]
        assert got == [3.0 * (1 << 20)] * 20


@pytest.mark.gpu
def test_fused_sum_never_bound_exchanges_nothing(cuda) -> None:
    """A fused kernel launched before ``bind_exchange`` leaves its partial and reports."""
    import torch

    from ptxgen.runtime import Problem
    from ptxgen.templates.exchange import STATUS_UNBOUND

    spec = _fused_sum()
    prob = Problem(spec.graph, spec.meta)
    tensors = prob.allocate()
    tensors["x"].fill_(1.0)
    prob.launch(tensors)
    torch.cuda.synchronize()
    assert prob.module.status() == 1 << STATUS_UNBOUND
    assert float(tensors["sum_1"].item()) == 65536.0

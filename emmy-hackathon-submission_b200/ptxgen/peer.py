"""Cross-rank sums over NVLink peer memory, for the path's one collective step: the sharded full
sum's partials (one f32 per rank) summed into the job's result on every rank.

``PeerSum`` maps each rank's slot array into every other rank's process with CUDA IPC
(``pg_ipc_handle``/``pg_ipc_open``, handles exchanged once through the process group) and runs
``templates/exchange.py``'s one-warp kernel per call: each rank stores its partial straight into
every peer's memory and waits, bounded, for theirs. Nothing goes through NCCL, and every rank
adds the partials in rank order, so all ranks hold the same bits.

Every rank must make the same calls in the same order, as with any collective. The kernel's
waits give up after ``limit_ns`` and set the module's status word; ``check()`` raises then.
"""

from __future__ import annotations

import ctypes
from typing import Any

from .runtime import KernelStatusError, Module, _check, library
from .templates.exchange import ENTRY, MAX_RANKS, peer_sum_ptx

HANDLE_BYTES = 64


def _signed(x: int) -> int:
    return x - (1 << 64) if x >= 1 << 63 else x


class PeerSum:
    """One f32 summed across the ranks of ``group`` (default: the whole job) through peer
    memory. Construction is collective: every rank of the group builds one at the same time."""

    def __init__(self, group: Any = None, device: int | None = None,
                 limit_ns: int = 2_000_000_000):
        import torch
        import torch.distributed as dist

        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 1 <= self.world <= MAX_RANKS:
            raise ValueError(f"PeerSum: {self.world} ranks (1 to {MAX_RANKS})")
        dev = torch.cuda.current_device() if device is None else device
        self.limit_ns = int(limit_ns)
        self.seq = 0
        self.slots = torch.zeros(2 * self.world, dtype=torch.int64, device=f"cuda:{dev}")
        self.module = Module(peer_sum_ptx(), device=dev)
        self.kernel = self.module.kernel(ENTRY)
        lib = library()
        handle = (ctypes.c_ubyte * HANDLE_BYTES)()
        offset = ctypes.c_uint64()
        _check(lib.pg_ipc_handle(self.slots.data_ptr(), handle, ctypes.byref(offset)),
               "pg_ipc_handle")
        table: list[Any] = [None] * self.world
        dist.all_gather_object(table, (bytes(handle), offset.value), group=group)
        self.opened: list[int] = []
        addrs = []
        for p, (h, off) in enumerate(table):
            if p == self.rank:
                addrs.append(self.slots.data_ptr())
                continue
            base = ctypes.c_uint64()
            buf = (ctypes.c_ubyte * HANDLE_BYTES).from_buffer_copy(h)
            _check(lib.pg_ipc_open(buf, ctypes.byref(base)), f"pg_ipc_open(rank {p})")
            self.opened.append(base.value)
            addrs.append(base.value + off)
        self.peers = torch.tensor([_signed(a) for a in addrs], dtype=torch.int64,
                                  device=f"cuda:{dev}")
        torch.cuda.synchronize(dev)
        dist.barrier(group)  # every rank has mapped its peers before any rank stores into them

    def __call__(self, src: int, dst: int | None = None, stream: int = 0) -> None:
        """Sum the f32 at device address ``src`` over the ranks into ``dst`` (default: in
        place), stream-ordered on ``stream``."""
        self.seq += 1
        args = [src, src if dst is None else dst, self.peers.data_ptr(),
                self.slots.data_ptr(), self.rank, self.world, self.seq, self.limit_ns]
        self.kernel.launch(1, 32, 0, args, stream=stream)

    def check(self) -> None:
        """Raise ``KernelStatusError`` if a call's wait for a peer gave up (synchronous)."""
        status = self.module.status()
        if status:
            raise KernelStatusError(f"PeerSum: a rank's partial did not arrive within "
                                    f"{self.limit_ns} ns (status 0x{status:08x})")

    def close(self) -> None:
        """Unmap the peers' slot arrays. Every rank should be past its last call."""
        lib = library()
        while self.opened:
            _check(lib.pg_ipc_close(self.opened.pop()), "pg_ipc_close")

"""Cross-rank sums over NVLink peer memory, for the path's one collective step: the sharded full
sum's partials (one f32 per rank) summed into the job's result on every rank.

``PeerSlots`` gives each rank a slot array and maps every rank's array into every other rank's
process with CUDA IPC (``pg_ipc_handle``/``pg_ipc_open``; the handles go round the process group
once). Two kernels use it, both from ``templates/exchange.py``:

* ``PeerSum``: the exchange as its own one-warp kernel, launched after the kernel that made the
  partial.
* ``bind_exchange``: the exchange as the epilogue of the kernel that makes the partial. The
  last block to add its share stores the rank's partial into every peer's slots, collects theirs
  and writes the total, so one launch does both the sum and the collective. ``with_exchange``
  marks a problem's meta.json for that form.

Every rank must make the same calls in the same order, as with any collective. The kernels'
waits give up after ``limit_ns`` and set their module's status word; ``check`` raises then.
"""

from __future__ import annotations

import copy
import ctypes
import struct
from typing import Any

from .problems import ProblemSpec
from .runtime import KernelStatusError, Module, _check, library
from .templates.exchange import ENTRY, MAX_RANKS, peer_sum_ptx

HANDLE_BYTES = 64
DEFAULT_LIMIT_NS = 2_000_000_000


def _signed(x: int) -> int:
    return x - (1 << 64) if x >= 1 << 63 else x


class PeerSlots:
    """This rank's slot array (2 x world 64-bit words) and the device table of every rank's
    array as mapped into this process. Construction is collective over ``group``."""

    def __init__(self, group: Any = None, device: int | None = None):
        import torch
        import torch.distributed as dist

        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 1 <= self.world <= MAX_RANKS:
            raise ValueError(f"peer slots: {self.world} ranks (1 to {MAX_RANKS})")
        self.device = torch.cuda.current_device() if device is None else device
        self.slots = torch.zeros(2 * self.world, dtype=torch.int64, device=f"cuda:{self.device}")
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
                                  device=f"cuda:{self.device}")
        torch.cuda.synchronize(self.device)
        dist.barrier(group)  # every rank has mapped its peers before any rank stores into them

    def close(self) -> None:
        """Unmap the peers' slot arrays. Every rank should be past its last exchange."""
        lib = library()
        while self.opened:
            _check(lib.pg_ipc_close(self.opened.pop()), "pg_ipc_close")


def _check_status(module: Module, limit_ns: int, what: str) -> None:
    status = module.status()
    if status:
        raise KernelStatusError(f"{what}: a rank's partial did not arrive within {limit_ns} ns "
                                f"(status 0x{status:08x})")


class PeerSum:
    """One f32 summed across the ranks of ``group`` (default: the whole job) by the exchange
    kernel. Construction is collective: every rank of the group builds one at the same time."""

    def __init__(self, group: Any = None, device: int | None = None,
                 limit_ns: int = DEFAULT_LIMIT_NS):
        self.peer = PeerSlots(group, device)
        self.rank, self.world = self.peer.rank, self.peer.world
        self.limit_ns = int(limit_ns)
        self.seq = 0
        self.module = Module(peer_sum_ptx(), device=self.peer.device)
        self.kernel = self.module.kernel(ENTRY)

    def __call__(self, src: int, dst: int | None = None, stream: int = 0) -> None:
        """Sum the f32 at device address ``src`` over the ranks into ``dst`` (default: in
        place), stream-ordered on ``stream``."""
        self.seq += 1
        args = [src, src if dst is None else dst, self.peer.peers.data_ptr(),
                self.peer.slots.data_ptr(), self.rank, self.world, self.seq, self.limit_ns]
        self.kernel.launch(1, 32, 0, args, stream=stream)

    def check(self) -> None:
        """Raise ``KernelStatusError`` if a call's wait for a peer gave up (synchronous)."""
        _check_status(self.module, self.limit_ns, "PeerSum")

    def close(self) -> None:
        self.peer.close()


def with_exchange(spec: ProblemSpec, output: str) -> ProblemSpec:
    """``spec`` with its kernel marked to sum ``output`` across ranks in its own epilogue (the
    ``exchange`` key of the launch entry, which only sharded problems carry)."""
    meta = copy.deepcopy(spec.meta)
    meta["kernels"][0]["exchange"] = {"output": output}
    return ProblemSpec(graph=spec.graph, meta=meta)


def bind_exchange(module: Module, peer: PeerSlots, limit_ns: int = DEFAULT_LIMIT_NS) -> None:
    """Point a ``with_exchange`` kernel's module at ``peer``'s slot arrays (its module globals;
    once, before its first launch)."""
    module.write_global("xch_peers", struct.pack("<Q", peer.peers.data_ptr()))
    module.write_global("xch_slots", struct.pack("<Q", peer.slots.data_ptr()))
    module.write_global("xch_limit", struct.pack("<Q", int(limit_ns)))
    module.write_global("xch_rank", struct.pack("<I", peer.rank))
    module.write_global("xch_world", struct.pack("<I", peer.world))


def check_exchange(module: Module, limit_ns: int = DEFAULT_LIMIT_NS) -> None:
    """Raise ``KernelStatusError`` if a ``with_exchange`` kernel's wait gave up."""
    _check_status(module, limit_ns, "exchange epilogue")

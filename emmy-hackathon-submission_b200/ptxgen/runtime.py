"""Running emitted PTX on a GPU through the C-ABI launcher (``include/ptxgen_b200.h``).

``Module`` loads a PTX module, ``Module.kernel`` finds an entry, and ``Kernel.launch`` starts it
on device pointers. ``Problem`` is one meta.json kernel end to end: compile the IR, allocate the
buffers (PyTorch is used for device memory only), fill its inputs, zero ``zero_outputs``, launch
with meta.json's geometry, and read the status word. ``ProblemSet`` runs a meta.json problem of
several kernels in order, chaining the intermediates one kernel writes into the next.

The emitted module states the launch it was compiled for in ``// @ptxgen`` header lines
(``launch grid=G block=B``, ``dynamic_smem=N``, ``tensormap ...``); a launch that disagrees is
refused here, because the kernel's index arithmetic relies on it (a tail guard proven
unnecessary for G blocks is not there for more).
"""

from __future__ import annotations

import ctypes
import json
import re
import threading
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np

from .build import LIB

# "// @ptxgen <key> <fields>" or "// @ptxgen <key>=<value>" (dynamic_smem=N)
_NOTE = re.compile(r"^// @ptxgen (\w+)[ =](.*)$", re.M)
_DTYPE_CODE = {"u8": 0, "f16": 1, "bf16": 2, "f32": 3}


class LaunchError(RuntimeError):
    """A launcher call failed; the message carries the driver's error and any JIT log."""


class KernelStatusError(LaunchError):
    """A kernel reported a failure through its status word (a bounded wait gave up)."""


_lib: ctypes.CDLL | None = None
_lock = threading.Lock()
_initialised: set[int] = set()


def library() -> ctypes.CDLL:
    """The loaded launcher library (it must have been built: ``ptxgen.build``)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB.exists():
                raise LaunchError(f"launcher library {LIB} is not built (run ptxgen.build)")
            lib = ctypes.CDLL(str(LIB))
            u64, i32, u32, vp, cp = (ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32,
                                     ctypes.c_void_p, ctypes.c_char_p)
            pu64, pu32, psz = (ctypes.POINTER(u64), ctypes.POINTER(u32),
                               ctypes.POINTER(ctypes.c_size_t))
            sig = {
                "pg_init": [i32],
                "pg_last_error": [],
                "pg_module_load": [cp, ctypes.POINTER(vp)],
                "pg_module_unload": [vp],
                "pg_kernel_get": [vp, cp, ctypes.POINTER(vp)],
                "pg_kernel_launch": [vp, u32, u32, u32, u64, pu64, i32],
                "pg_kernel_launch_ex": [vp, u32, u32, u32, u64, pu64, i32, u32],
                "pg_kernel_max_clusters": [vp, u32, u32, u32, ctypes.POINTER(i32)],
                "pg_kernel_time": [vp, u32, u32, u32, u64, pu64, i32, i32, i32,
                                   ctypes.POINTER(ctypes.c_float)],
                "pg_tensormap_fill": [vp, cp, i32, i32, u64, pu64, pu64, pu32, i32],
                "pg_status_take": [vp, pu32],
                "pg_global_write": [vp, cp, vp, ctypes.c_size_t],
                "pg_memset_async": [u64, ctypes.c_size_t, u64],
                "pg_memcpy_htod_async": [u64, vp, ctypes.c_size_t, u64],
                "pg_memcpy_dtoh_async": [vp, u64, ctypes.c_size_t, u64],
                "pg_stream_synchronize": [u64],
                "pg_run_host": [vp, u32, u32, u32, u64, i32, pu64, ctypes.POINTER(vp), psz,
                                pu32],
                "pg_ipc_handle": [u64, vp, pu64],
                "pg_ipc_open": [vp, pu64],
                "pg_ipc_close": [u64],
                "pg_grid_sum_f32_noalloc": [u64, u64, u64, u32, u64],
            }
            for name, args in sig.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_char_p if name == "pg_last_error" else ctypes.c_int
            _lib = lib
        return _lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = library().pg_last_error().decode(errors="replace")
        cls = KernelStatusError if rc == -4 else LaunchError
        raise cls(f"{what} failed ({rc}): {msg}")


def init(device: int = 0) -> None:
    """Make ``device``'s primary context current for the launcher (idempotent per device)."""
    lib = library()
    _check(lib.pg_init(device), f"pg_init({device})")
    _initialised.add(device)


def header_notes(ptx: str) -> dict[str, list[str]]:
    notes: dict[str, list[str]] = {}
    for key, rest in _NOTE.findall(ptx):
        notes.setdefault(key, []).append(rest.strip())
    return notes


def _kv(text: str) -> dict[str, str]:
    return dict(part.split("=", 1) for part in text.split() if "=" in part)


@dataclass
class TensorMapNote:
    """A ``// @ptxgen tensormap`` line: which .global symbol holds a map over which buffer."""

    symbol: str
    buffer: str
    dtype: str
    dims: tuple[int, ...]
    strides: tuple[int, ...]
    box: tuple[int, ...]
    swizzle: int

    @classmethod
    def parse(cls, text: str) -> TensorMapNote:
        kv = _kv(text)
        ints = lambda s: tuple(int(x) for x in s.split(",") if x)  # noqa: E731
        return cls(kv["symbol"], kv["buffer"], kv["dtype"], ints(kv["dims"]),
                   ints(kv.get("strides", "")), ints(kv["box"]), int(kv.get("swizzle", "0")))


class Module:
    def __init__(self, ptx: str, device: int = 0):
        if device not in _initialised:
            init(device)
        self.ptx = ptx
        self.notes = header_notes(ptx)
        handle = ctypes.c_void_p()
        _check(library().pg_module_load(ptx.encode(), ctypes.byref(handle)), "pg_module_load")
        self.handle = handle
        self.tensormaps = [TensorMapNote.parse(t) for t in self.notes.get("tensormap", [])]
        self._filled: tuple[int, ...] | None = None  # the buffer addresses the maps describe
        launch = _kv(self.notes["launch"][0]) if "launch" in self.notes else {}
        self.grid = int(launch["grid"]) if "grid" in launch else None
        self.block = int(launch["block"]) if "block" in launch else None
        # a persistent kernel loops over its tiles (tile = ctaid + i * nctaid): any grid works,
        # and one CTA per SM is the right one
        self.persistent = launch.get("persistent") == "1"
        # CTAs per cluster (the kernel's .reqnctapercluster): the grid is a multiple of it
        self.cluster = int(launch.get("cluster", "1"))
        dyn = self.notes.get("dynamic_smem")
        self.dynamic_smem = int(dyn[0]) if dyn else 0
        # output buffer -> (entry, grid, block) of a kernel in the module that zeroes it, to run
        # in place of a memset right before the main entry (``// @ptxgen zero``)
        self.zeroers = {}
        for z in self.notes.get("zero", []):
            kv = _kv(z)
            self.zeroers[kv["buffer"]] = (kv["entry"], int(kv["grid"]), int(kv["block"]))

    def kernel(self, entry: str) -> Kernel:
        handle = ctypes.c_void_p()
        _check(library().pg_kernel_get(self.handle, entry.encode(), ctypes.byref(handle)),
               f"pg_kernel_get({entry})")
        return Kernel(self, handle, entry)

    def fill_tensormaps(self, pointers: dict[str, int]) -> None:
        """Write every tensor map the module names, over the buffers at ``pointers``. The
        maps are written only when an address differs from the last call's, so a launch on the
        same buffers costs no call into the library (a rewrite waits for the device to idle)."""
        if not self.tensormaps:
            return
        now = tuple(pointers[t.buffer] for t in self.tensormaps)
        if now == self._filled:
            return
        lib = library()
        for t in self.tensormaps:
            rank = len(t.dims)
            dims = (ctypes.c_uint64 * rank)(*t.dims)
            strides = (ctypes.c_uint64 * max(1, rank - 1))(*(t.strides or (0,)))
            box = (ctypes.c_uint32 * rank)(*t.box)
            _check(lib.pg_tensormap_fill(self.handle, t.symbol.encode(), _DTYPE_CODE[t.dtype],
                                         rank, pointers[t.buffer], dims, strides, box,
                                         t.swizzle), f"pg_tensormap_fill({t.symbol})")
        self._filled = now

    def write_global(self, symbol: str, data: bytes) -> None:
        """Copy ``data`` into the module's ``.global`` symbol (at most its size)."""
        buf = ctypes.create_string_buffer(data, len(data))
        _check(library().pg_global_write(self.handle, symbol.encode(), buf, len(data)),
               f"pg_global_write({symbol})")

    def status(self) -> int:
        out = ctypes.c_uint32()
        _check(library().pg_status_take(self.handle, ctypes.byref(out)), "pg_status_take")
        return out.value

    def __del__(self) -> None:
        h = getattr(self, "handle", None)
        if h is not None and _lib is not None:
            try:
                _lib.pg_module_unload(h)
            except Exception:  # noqa: BLE001 - interpreter shutdown
                pass


@dataclass
class Kernel:
    module: Module
    handle: ctypes.c_void_p
    entry: str

    def launch(self, grid: int, block: int, smem: int, pointers: list[int],
               stream: int = 0, early: bool = False) -> None:
        """Launch the module's main entry. ``early``: programmatic stream serialization
        (``PG_LAUNCH_EARLY``), for a kernel that waits (``griddepcontrol.wait``) before it
        touches what the kernel ahead of it writes."""
        m = self.module
        if m.persistent:
            if block != m.block:
                raise LaunchError(f"{self.entry}: compiled for block {m.block}, asked {block}")
        elif m.grid is not None and (grid, block) != (m.grid, m.block):
            raise LaunchError(f"{self.entry}: compiled for grid {m.grid} x block {m.block}, "
                              f"asked to launch {grid} x {block}")
        if grid % m.cluster:
            raise LaunchError(f"{self.entry}: grid {grid} is not a multiple of its cluster "
                              f"size {m.cluster}")
        smem = max(smem, m.dynamic_smem)
        ptrs = (ctypes.c_uint64 * len(pointers))(*pointers)
        _check(library().pg_kernel_launch_ex(self.handle, grid, block, smem, stream, ptrs,
                                             len(pointers), 1 if early else 0),
               f"pg_kernel_launch({self.entry})")

    def launch_plain(self, grid: int, block: int, pointers: list[int], stream: int = 0) -> None:
        """Launch this entry as it is, with no dynamic shared memory and none of the main
        entry's launch notes (a helper kernel of the module, such as its zero kernel)."""
        ptrs = (ctypes.c_uint64 * len(pointers))(*pointers)
        _check(library().pg_kernel_launch(self.handle, grid, block, 0, stream, ptrs,
                                          len(pointers)), f"pg_kernel_launch({self.entry})")

    def time(self, grid: int, block: int, smem: int, pointers: list[int], warmup: int = 3,
             reps: int = 20, stream: int = 0) -> list[float]:
        """Device milliseconds of each of ``reps`` back-to-back launches after ``warmup``
        untimed ones (``pg_kernel_time``: CUDA events around every launch)."""
        out = (ctypes.c_float * reps)()
        ptrs = (ctypes.c_uint64 * len(pointers))(*pointers)
        _check(library().pg_kernel_time(self.handle, grid, block,
                                        max(smem, self.module.dynamic_smem), stream, ptrs,
                                        len(pointers), warmup, reps, out),
               f"pg_kernel_time({self.entry})")
        return list(out)

    def max_clusters(self, block: int, smem: int) -> int:
        """Clusters of this kernel that fit on the device at once."""
        out = ctypes.c_int()
        _check(library().pg_kernel_max_clusters(
            self.handle, block, max(smem, self.module.dynamic_smem), self.module.cluster,
            ctypes.byref(out)), f"pg_kernel_max_clusters({self.entry})")
        return out.value

    def run_host(self, grid: int, block: int, smem: int, stream: int, dev: list[int],
                 host: list[int | None], nbytes: list[int], flags: list[int]) -> None:
        """The one-call host-buffer path (``pg_run_host``)."""
        n = len(dev)
        _check(library().pg_run_host(
            self.handle, grid, block, max(smem, self.module.dynamic_smem), stream, n,
            (ctypes.c_uint64 * n)(*dev), (ctypes.c_void_p * n)(*host),
            (ctypes.c_size_t * n)(*nbytes), (ctypes.c_uint32 * n)(*flags)),
            f"pg_run_host({self.entry})")


# --- problems: one meta.json kernel, end to end ----------------------------------------------

_TORCH_DTYPE = {"f32": "float32", "f64": "float64", "f16": "float16", "bf16": "bfloat16",
                "i32": "int32", "i64": "int64", "u8": "uint8", "i16": "int16", "bool": "bool",
                "u32": "int32", "u64": "int64", "u16": "int16"}


def torch_dtype(dtype: str) -> Any:
    import torch

    return getattr(torch, _TORCH_DTYPE[dtype])


@dataclass
class Problem:
    """A compiled meta.json kernel: its IR, launch entry and module."""

    graph_json: dict[str, Any]
    meta: dict[str, Any]
    ptx: str = ""
    flags: dict[str, bool] = field(default_factory=dict)
    device: int | None = None  # None: the current CUDA device when first used
    _module: Module | None = None
    _kernel: Kernel | None = None
    _launch: dict[str, Any] | None = None
    _max_clusters: int | None = None
    _helpers: dict[str, Kernel] = field(default_factory=dict)  # other entries of the module

    @classmethod
    def from_dir(cls, path: str | Path, **flags: bool) -> Problem:
        path = Path(path)
        ir = next(path.glob("*.ir.json"))
        return cls(json.loads(ir.read_text()), json.loads((path / "meta.json").read_text()),
                   flags=flags)

    @property
    def launch_entry(self) -> dict[str, Any]:
        if self._launch is None:
            from .compiler import kernel_for_meta
            from .ir import Graph

            self._launch = kernel_for_meta(Graph.from_dict(self.graph_json), self.meta)[1]
        return self._launch

    def compile(self) -> str:
        from .compiler import to_ptx
        from .ir import Graph

        if not self.ptx:
            self.ptx = to_ptx(Graph.from_dict(self.graph_json), self.meta,
                              self.flags.get("no_unroll", False),
                              self.flags.get("no_fusion", False),
                              self.flags.get("no_cse", False),
                              templates=not self.flags.get("no_templates", False))
        return self.ptx

    def _dev(self) -> int:
        if self.device is None:
            import torch

            self.device = torch.cuda.current_device()
        return self.device

    def load(self) -> Kernel:
        if self._kernel is None:
            self._dev()
            self._module = Module(self.compile(), self.device)
            self._kernel = self._module.kernel(self.launch_entry["entry"])
        return self._kernel

    @property
    def module(self) -> Module:
        self.load()
        assert self._module is not None
        return self._module

    def _helper(self, entry: str) -> Kernel:
        """Another entry of this problem's module (looked up once)."""
        if entry not in self._helpers:
            self._helpers[entry] = self.module.kernel(entry)
        return self._helpers[entry]

    def grid(self) -> int:
        """meta.json's grid, or for a persistent kernel one CTA per SM (at most one per tile),
        in whole clusters that can all be resident at once."""
        m = self.module
        if m.persistent and m.grid is not None:
            import torch

            sms = torch.cuda.get_device_properties(self._dev()).multi_processor_count
            if m.cluster > 1:
                if self._max_clusters is None:
                    launch = self.launch_entry
                    self._max_clusters = self.load().max_clusters(
                        launch["block"][0], int(launch.get("smem_bytes", 0)))
                sms = min(sms, self._max_clusters * m.cluster)
            return max(m.cluster, min(m.grid, sms) // m.cluster * m.cluster)
        return int(self.launch_entry["grid"][0])

    def allocate(self, extra_guard: int = 0) -> dict[str, Any]:
        """Device tensors for every argument (uninitialised)."""
        import torch

        out = {}
        for a in self.launch_entry["args"]:
            n = int(np.prod(a["shape"]))
            out[a["name"]] = torch.empty(n + extra_guard, dtype=torch_dtype(a["dtype"]),
                                         device=f"cuda:{self._dev()}")
        return out

    def launch(self, tensors: dict[str, Any], stream: int | None = None, zero: bool = True,
               check_status: bool = False) -> None:
        import torch

        launch = self.launch_entry
        kernel = self.load()
        if stream is None:
            stream = torch.cuda.current_stream(self._dev()).cuda_stream
        ptrs = {name: t.data_ptr() for name, t in tensors.items()}
        self.module.fill_tensormaps(ptrs)
        early = False
        if zero:
            shapes = {a["name"]: a["shape"] for a in launch["args"]}
            for name in launch.get("zero_outputs", []):
                t = tensors[name]
                zeroer = self.module.zeroers.get(name)
                if zeroer is not None:
                    # the module's own kernel clears the buffer and lets the main kernel start
                    # at once; the main kernel waits for it before it adds into the buffer
                    entry, grid, block = zeroer
                    self._helper(entry).launch_plain(grid, block, [t.data_ptr()], stream)
                    early = True
                    continue
                n = int(np.prod(shapes[name])) if shapes[name] else 1
                _check(library().pg_memset_async(t.data_ptr(), n * t.element_size(), stream),
                       "pg_memset_async")
        kernel.launch(self.grid(), launch["block"][0], int(launch.get("smem_bytes", 0)),
                      [ptrs[n] for n in launch["arg_order"]], stream, early=early)
        if check_status:
            torch.cuda.synchronize(self._dev())
            status = self.module.status()
            if status:
                raise KernelStatusError(f"{launch['entry']}: status word 0x{status:08x}")

    def capture(self, tensors: dict[str, Any]) -> Any:
        """A CUDA graph of one launch on ``tensors`` (zero_outputs cleared, kernel launched),
        for replay with ``.replay()`` when the launch itself is the cost. One eager launch first
        JIT-loads the module and writes its tensor maps, so nothing synchronises during the
        capture; the graph keeps the buffers' addresses, so replay it only with these tensors."""
        return capture_launches([self], tensors)

    def time(self, tensors: dict[str, Any], warmup: int = 3, reps: int = 20,
             stream: int | None = None) -> list[float]:
        """Device milliseconds of ``reps`` back-to-back launches (after ``warmup``) on the
        buffers in ``tensors``; zero_outputs are cleared once, before the warm-up."""
        import torch

        if stream is None:
            stream = torch.cuda.current_stream(self._dev()).cuda_stream
        self.launch(tensors, stream)  # tensor maps filled, zero_outputs cleared
        launch = self.launch_entry
        ptrs = {name: t.data_ptr() for name, t in tensors.items()}
        return self.load().time(self.grid(), launch["block"][0],
                                int(launch.get("smem_bytes", 0)),
                                [ptrs[n] for n in launch["arg_order"]], warmup, reps, stream)


# --- problems of several kernels -----------------------------------------------------------------


def problem_args(meta: dict[str, Any]) -> dict[str, dict[str, Any]]:
    """Every buffer a meta.json problem names, once, checked for chaining: an ``intermediate``
    argument (reference ``tools/generate.py:142-144``: neither written by its kernel nor an
    input or a constant) must be an output of an earlier kernel, of the same dtype and size."""
    out: dict[str, dict[str, Any]] = {}
    written: set[str] = set()
    for k in meta["kernels"]:
        for a in k["args"]:
            seen = out.get(a["name"])
            if a.get("intermediate") and a["name"] not in written:
                raise ValueError(f"{k['entry']}: intermediate {a['name']!r} is not written by "
                                 "an earlier kernel")
            if seen is not None and (seen["dtype"] != a["dtype"] or
                                     int(np.prod(seen["shape"] or [1])) !=
                                     int(np.prod(a["shape"] or [1]))):
                raise ValueError(f"{k['entry']}: {a['name']!r} disagrees with an earlier kernel")
            out.setdefault(a["name"], a)
        written |= {a["name"] for a in k["args"] if a.get("output")}
    return out


class ProblemSet:
    """A meta.json problem of one or more kernels: each kernel has its own ``<entry>.ir.json``
    (reference ``tools/generate.py:180-199``) and they run in meta.json order on one stream,
    each after its own zero_outputs are cleared, every buffer shared by name, so an
    intermediate one kernel writes is what the next one reads."""

    def __init__(self, graphs: dict[str, dict[str, Any]], meta: dict[str, Any],
                 flags: dict[str, bool] | None = None, device: int | None = None):
        self.meta = meta
        self.args = problem_args(meta)
        self.problems = [Problem(graphs[k["entry"]], meta, flags=dict(flags or {}),
                                 device=device) for k in meta["kernels"]]

    @classmethod
    def from_dir(cls, path: str | Path, **flags: bool) -> ProblemSet:
        path = Path(path)
        meta = json.loads((path / "meta.json").read_text())
        graphs = {k["entry"]: json.loads((path / f"{k['entry']}.ir.json").read_text())
                  for k in meta["kernels"]}
        return cls(graphs, meta, flags)

    def allocate(self, extra_guard: int = 0) -> dict[str, Any]:
        """Device tensors for every buffer of every kernel (uninitialised)."""
        import torch

        dev = self.problems[0]._dev()
        return {name: torch.empty(int(np.prod(a["shape"] or [1])) + extra_guard,
                                  dtype=torch_dtype(a["dtype"]), device=f"cuda:{dev}")
                for name, a in self.args.items()}

    def launch(self, tensors: dict[str, Any], stream: int | None = None,
               check_status: bool = False) -> None:
        for p in self.problems:
            p.launch(tensors, stream, check_status=check_status)

    def capture(self, tensors: dict[str, Any]) -> Any:
        """A CUDA graph of every kernel of the problem in order (see ``Problem.capture``)."""
        return capture_launches(self.problems, tensors)


def capture_launches(problems: list[Problem], tensors: dict[str, Any]) -> Any:
    """Record ``problems``' launches (each clearing its zero_outputs first) on a capture stream
    into a ``torch.cuda.CUDAGraph``; one eager pass first loads every module and fills its
    tensor maps, so the captured calls are only memsets and kernel launches."""
    import torch

    for p in problems:
        p.launch(tensors, check_status=True)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.graph(graph, stream=side):
        for p in problems:
            p.launch(tensors, side.cuda_stream)
    return graph

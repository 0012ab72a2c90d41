"""The C-ABI launcher library: it builds without a GPU, loads, and exports every function the
public header declares (no compute calls: those need a GPU)."""

from __future__ import annotations

import ctypes
import re

from conftest import ROOT

from ptxgen.build import build_library


def declared() -> list[str]:
    text = (ROOT / "include" / "ptxgen_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|const char \*)\s*(pg_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_launcher() -> None:
    names = declared()
    for want in ("pg_init", "pg_module_load", "pg_kernel_get", "pg_kernel_launch",
                 "pg_tensormap_fill", "pg_status_take", "pg_run_host", "pg_last_error"):
        assert want in names


def test_library_exports_every_declared_symbol() -> None:
    lib = ctypes.CDLL(str(build_library()))
    for name in declared():
        assert hasattr(lib, name), name


def test_calls_before_init_fail_cleanly() -> None:
    """Without pg_init every call returns PG_ERR_NOT_INITIALISED (-5) instead of crashing."""
    lib = ctypes.CDLL(str(build_library()))
    lib.pg_last_error.restype = ctypes.c_char_p
    lib.pg_stream_synchronize.argtypes = [ctypes.c_uint64]
    rc = lib.pg_stream_synchronize(0)
    assert rc in (-5, 0) or rc > 0
    assert isinstance(lib.pg_last_error(), bytes)
    lib.pg_module_load.argtypes = [ctypes.c_char_p, ctypes.c_void_p]
    assert lib.pg_module_load(None, None) == -2


def test_python_binding_types_every_declared_symbol() -> None:
    """``ptxgen.runtime.library()`` gives every header function its argument types, so no
    call goes through ctypes' default int conversion of 64-bit pointers."""
    from ptxgen.runtime import library

    lib = library()
    for name in declared():
        if name == "pg_last_error":
            continue
        assert getattr(lib, name).argtypes is not None, name

"""ptxgen for B200: Emmy Kernel IR -> sm_100a PTX, plus the launcher that runs it.

The public surface mirrors the reference compiler (``compile_module``, ``Buffer``, ``to_ptx``);
``runtime`` holds the C-ABI launcher binding and ``problems`` the Kernel IR generator for the
benchmark configurations.
"""

from .compiler import Buffer, compile_module, kernel_for_meta, to_ptx

__all__ = ["Buffer", "compile_module", "kernel_for_meta", "to_ptx"]

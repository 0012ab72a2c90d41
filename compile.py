"""Emmy Kernel IR -> PTX for B200 (sm_100a).

    python compile.py <kernel>.ir.json [--no_loop_unroll] [--no_fusion] [--no_cse] > out.ptx

The same command-line contract as the reference compiler (reference ``compile.py:1-73``): it reads
the IR and the ``meta.json`` beside it (the contract for the parameter order, the block size and
the buffers' shapes, dtypes and outputs) and writes one PTX module to stdout. An IR it cannot
lower raises (``NotImplementedError``/``ValueError``/``KeyError``) and exits non-zero.
``--no_loop_unroll`` turns every loop into a runtime loop with one copy of the body per trip.
``--no_fusion`` never fuses a float multiply and add into one ``fma`` (ptxas still may: the
multiply and the add are written without a rounding modifier, as the reference writes them).
``--no_cse`` turns off common subexpression elimination.
Any of the three flags also turns off the hand-written kernel templates, so the generic lowering
the flag describes is what runs.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from typing import Any

sys.path.insert(0, str(Path(__file__).resolve().parent / "emmy-hackathon-submission_b200"))

from ptxgen.compiler import compile_module  # noqa: E402
from ptxgen.compiler import to_ptx as _to_ptx  # noqa: E402
from ptxgen.ir import Graph  # noqa: E402
from ptxgen.lower import Buffer  # noqa: E402

__all__ = ["Buffer", "compile_module", "main", "to_ptx"]


def to_ptx(graph: Graph, meta: dict[str, Any], no_unroll: bool = False, no_fusion: bool = False,
           no_cse: bool = False) -> str:
    return _to_ptx(graph, meta, no_unroll, no_fusion, no_cse)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawTextHelpFormatter)
    parser.add_argument("json_path", type=Path, help="Kernel IR json (<kernel>.ir.json)")
    parser.add_argument("--no_loop_unroll", action="store_true", help="never unroll loops")
    parser.add_argument("--no_fusion", action="store_true", help="never fuse a multiply and an add")
    parser.add_argument("--no_cse", action="store_true", help="never reuse an identical result")
    args = parser.parse_args()
    graph = Graph.from_dict(json.loads(args.json_path.read_text()))
    meta = json.loads(args.json_path.with_name("meta.json").read_text())
    sys.stdout.write(to_ptx(graph, meta, args.no_loop_unroll, args.no_fusion, args.no_cse))


if __name__ == "__main__":
    main()

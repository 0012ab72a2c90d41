"""Regenerates the golden fixtures in this directory from the reference checkout.

Run with the environment variable REFERENCE set to a checkout of the reference; the fixtures it
writes are committed, so tests never read the reference at run time.

* ``shipped/<problem>/`` -- the five distinct Kernel IR kernels the reference ships as examples
  (``examples/*/<problem>/<kernel>.ir.json`` + ``meta.json``), byte for byte: they are the
  reference's only Kernel IR fixtures and the inputs its compiler was tested on.
* ``literals.json`` -- PTX immediates of a set of values written by the reference's own literal
  encoder (``ptxgen/dtypes.py:60-76``, importable without Emmy), and bf16 roundings by its
  packaging rule (``tools/generate.py:57-60``).
* ``fastmath.json`` -- the instruction sequence each of the reference's fast-math functions
  (``ptxgen/fastmath.py:23-74``, importable without Emmy) writes into its PTX builder for one
  input register (two for pow): opcode and operands per instruction, registers renamed in
  order of first appearance.
"""

from __future__ import annotations

import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("REFERENCE", "reference"))
SHIPPED = {
    "p02_scale_shift": "examples/op_fusion/p02_scale_shift",
    "r02_big_sum": "examples/cse/r02_big_sum",
    "m01_matmul_512": "examples/cse/m01_matmul_512",
    "a01_attention": "examples/op_fusion/a01_attention",
    "a03_noscale": "examples/op_fusion/a03_noscale",
}
VALUES = [0.0, -0.0, 1.0, -1.0, 0.5, 2.0, 1e-5, 1e-6, 3.141592653589793, 0.044715,
          0.7978845608028654, 1.4426950408889634, 0.6931471805599453, -2.5, 65504.0, 1e30,
          float("inf"), float("-inf"), 1.0000001, 0.1, 0.2, 0.3, 1.0 / 3.0, 255.99, 3.0e-39]


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    sys.modules[name] = mod  # dataclasses look their module up while it loads
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    out = HERE / "shipped"
    for name, rel in SHIPPED.items():
        src = REFERENCE / rel
        dst = out / name
        dst.mkdir(parents=True, exist_ok=True)
        for f in [*src.glob("*.ir.json"), src / "meta.json"]:
            shutil.copyfile(f, dst / f.name)

    sys.path.insert(0, str(REFERENCE))
    dtypes = _load(REFERENCE / "ptxgen" / "dtypes.py", "ref_dtypes")
    lits = {typ: {repr(v): dtypes.lit(v, typ) for v in VALUES}
            for typ in ("f32", "f64", "f16", "bf16")}
    lits["int"] = {repr(v): dtypes.lit(v, "s32") for v in (0, 1, 7, -3, 4096)}
    xs = np.array([v for v in VALUES if np.isfinite(v)], np.float32)
    xs = np.concatenate([xs, np.random.default_rng(7).standard_normal(64).astype(np.float32)])
    # the reference's packaging rule, restated verbatim in numpy below
    b = xs.view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + (b >> 16 & 1)) >> 16 << 16).astype(np.uint32)
    (HERE / "literals.json").write_text(json.dumps({
        "literals": lits,
        "bf16_inputs_f32_bits": [int(x) for x in xs.view(np.uint32)],
        "bf16_rounded_f32_bits": [int(x) for x in rounded],
    }, indent=1))
    # the reference's fastmath imports ``ptxgen.builder`` and ``ptxgen.dtypes``: its own files
    sys.modules["ptxgen.dtypes"] = dtypes
    builder = _load(REFERENCE / "ptxgen" / "builder.py", "ptxgen.builder")
    fastmath = _load(REFERENCE / "ptxgen" / "fastmath.py", "ref_fastmath")
    seqs = {}
    for name, fn in fastmath.F32_FUNCS.items():
        k = builder.PTXKernel("t", [], 32)
        ins = ["%in0", "%in1"][:2 if name == "pow" else 1]
        out = fn(k, *ins)
        seqs[name] = {"body": [line.strip().rstrip(";") for line in k.body], "out": out}
    (HERE / "fastmath.json").write_text(json.dumps(seqs, indent=1))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()

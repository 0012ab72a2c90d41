"""The register-blocked f32 GEMM template (``ptxgen.templates.simt``) on the CPU: which nests it
takes, the launch it keeps, and that ptxas accepts what it writes. Its results are checked on the
GPU (``test_gpu_gemm.py``), bit for bit against the generic lowering and the oracle."""

from __future__ import annotations

import json
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from ptxgen import problems
from ptxgen.compiler import to_ptx
from ptxgen.ir import Graph
from ptxgen.suite import SUITE

SHIPPED = Path(__file__).parent / "golden" / "shipped" / "m01_matmul_512"

# nests in the shipped m01's form (each thread 2 x 2, 4 x 2 or 2 x 4 of C) at other shapes:
# ragged tile counts, one K step (fewer steps than the ring has stages), 64 x 64, 32 x 32 and
# 64 x 128 tiles
CASES = {
    "rect": dict(m=96, n=192, k=192, bm=32, bn=64, bk=64, stages=3, block=512),
    "one_k_step": dict(m=64, n=64, k=32, bm=32, bn=32, bk=32, stages=3, block=256),
    "tile_64x64": dict(m=128, n=128, k=256, bm=64, bn=64, bk=32, stages=3, block=512),
    "tile_32x32": dict(m=64, n=64, k=96, bm=32, bn=32, bk=32, stages=3, block=256),
    # 1024 threads, 512 owners, a 96 KiB ring in the nest's own dynamic shared memory
    "tile_64x128": dict(m=128, n=256, k=256, bm=64, bn=128, bk=64, stages=3, block=1024),
}


def case(key: str) -> problems.ProblemSpec:
    return problems.matmul(dtype="f32", raster_group=None, **CASES[key])


def shipped() -> tuple[dict, dict]:
    return (json.loads(next(SHIPPED.glob("*.ir.json")).read_text()),
            json.loads((SHIPPED / "meta.json").read_text()))


def ptxas_info(ptx: str, tmp_path: Path) -> str:
    exe = shutil.which("ptxas")
    if exe is None:
        pytest.skip("no ptxas")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run([exe, "-arch=sm_100a", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return r.stderr


def note(ptx: str, key: str) -> dict[str, str]:
    m = re.search(rf"^// @ptxgen {key} (.*)$", ptx, re.M)
    assert m, key
    return dict(kv.split("=") for kv in m.group(1).split())


def test_shipped_m01_takes_the_template(tmp_path: Path) -> None:
    """m01 keeps meta.json's launch (128 CTAs of 512 threads); its 32 x 64 tiles go to 128
    owners of 4 x 4 blocks, with no spills. Under any compiler flag the generic nest runs."""
    graph, meta = shipped()
    g = Graph.from_dict(graph)
    ptx = to_ptx(g, meta)
    launch = note(ptx, "launch")
    k = meta["kernels"][0]
    assert (int(launch["grid"]), int(launch["block"])) == (k["grid"][0], k["block"][0])
    assert note(ptx, "simt") == {"m": "512", "n": "512", "k": "512", "bm": "32", "bn": "64",
                                 "bk": "64", "stages": "2", "owners": "128"}
    # 16 accumulators in 8 pairs, 64 k per stage; per 4 k, 4 loads of A and 4 of B
    assert ptx.count("fma.rn.f32x2") == 8 * 64 and ptx.count("fma.rn.f32 ") == 0
    assert ptx.count("ld.shared.v4.f32") == ptx.count("ld.shared.v2.b64") == 4 * 16
    info = ptxas_info(ptx, tmp_path)
    assert "0 bytes spill stores" in info
    for flag in ("no_unroll", "no_fusion", "no_cse"):
        assert "@ptxgen simt" not in to_ptx(g, meta, **{flag: True})
    assert "@ptxgen simt" not in to_ptx(g, meta, templates=False)


@pytest.mark.parametrize("key", sorted(CASES))
def test_m01_form_nests_take_the_template(key: str, tmp_path: Path) -> None:
    spec = case(key)
    ptx = to_ptx(Graph.from_dict(spec.graph), spec.meta)
    n = note(ptx, "simt")
    kw = CASES[key]
    assert (int(n["bm"]), int(n["bn"])) == (kw["bm"], kw["bn"])
    assert int(n["owners"]) == kw["bm"] * kw["bn"] // 16
    k = spec.meta["kernels"][0]
    launch = note(ptx, "launch")
    assert (int(launch["grid"]), int(launch["block"])) == (k["grid"][0], k["block"][0])
    ptxas_info(ptx, tmp_path)


def test_threads_that_own_16_outputs_keep_the_generic_nest() -> None:
    """Where each thread already owns 16 or more elements of C (every f32 matmul of the suite),
    4 x 4 blocks would not read fewer bytes per FMA: the template declines."""
    for name in sorted(SUITE):
        spec = SUITE[name]().spec
        if spec.meta["kernels"][0]["args"][0]["dtype"] != "f32":
            continue
        assert "@ptxgen simt" not in to_ptx(Graph.from_dict(spec.graph), spec.meta), name


@pytest.mark.parametrize("key", ["shipped", *sorted(CASES)])
def test_ring_needs_nothing_meta_does_not_give(key: str) -> None:
    """The copy ring is a static array when it fits 48 KiB, else no larger than the dynamic
    shared memory meta.json gives the nest: a launcher that runs the IR's launch as it stands
    (grid, block, smem_bytes) runs the template too."""
    if key == "shipped":
        graph, meta = shipped()
    else:
        spec = case(key)
        graph, meta = spec.graph, spec.meta
    ptx = to_ptx(Graph.from_dict(graph), meta)
    assert "@ptxgen simt" in ptx
    dyn = re.search(r"^// @ptxgen dynamic_smem=(\d+)$", ptx, re.M)
    if dyn is None:
        assert ".shared .align 16 .b8 smem_ring[" in ptx
    else:
        assert int(dyn.group(1)) <= int(meta["kernels"][0]["smem_bytes"])

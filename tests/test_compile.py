"""Compilation on the CPU: every IR lowers, ptxas accepts the module for sm_100a, the CLI keeps
the reference's contract, and the emitted code has the shape the B200 design asks for."""

from __future__ import annotations

import json
import re
import shutil
import subprocess
import sys

import pytest
from conftest import ROOT, SHIPPED, shipped

from ptxgen import problems
from ptxgen.compiler import to_ptx
from ptxgen.ir import Graph

PTXAS = shutil.which("ptxas")


def ptxas(ptx: str, tmp_path) -> str:
    if PTXAS is None:
        pytest.skip("no ptxas")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run([PTXAS, "-arch=sm_100a", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return r.stderr


def compile_spec(spec: problems.ProblemSpec, **flags: bool) -> str:
    return to_ptx(Graph.from_dict(spec.graph), spec.meta, **flags)


FLAG_SETS = [{}, {"no_unroll": True}, {"no_fusion": True}, {"no_cse": True}]


@pytest.mark.parametrize("name", SHIPPED)
@pytest.mark.parametrize("flags", FLAG_SETS, ids=["default", "no_unroll", "no_fusion", "no_cse"])
def test_shipped_compiles_and_assembles(name: str, flags: dict, tmp_path) -> None:
    graph, meta = shipped(name)
    ptx = to_ptx(Graph.from_dict(graph), meta, **flags)
    assert ".target sm_100a" in ptx
    assert_plain_tma(ptx)
    ptxas(ptx, tmp_path)


# The two forms of TMA load the kernels may issue: each CTA fills its own shared memory, and in
# a CTA pair (cta_group::2) signals the pair leader's barrier. Neither form multicasts. A load
# may be predicated (a mixed-width GEMM skips a chunk of B that a narrow tile does not use).
TMA_LOAD = re.compile(r"^\s*(@%\w+ )?cp\.async\.bulk\.tensor\.2d\.(shared::cluster\.global\.tile|"
                      r"cta_group::2\.shared::cluster\.global)"
                      r"\.mbarrier::complete_tx::bytes \[%\w+\], \[%\w+, \{%\w+, %\w+\}\], "
                      r"\[%\w+\];$")


# The staged GEMM epilogue's TMA ops: one lane writes a block of this CTA's shared memory into
# C (a store, or a reduce-add for split-K), and waits for its own bulk groups.
TMA_OUT = re.compile(r"^\s*@%\w+ cp\.(reduce\.async\.bulk\.tensor\.2d\.global\.shared::cta\.add|"
                     r"async\.bulk\.tensor\.2d\.global\.shared::cta)\.tile\.bulk_group "
                     r"\[%\w+, \{%\w+, %\w+\}\], \[%\w+\];$")
BULK_GROUP = re.compile(r"^\s*(@%\w+ )?cp\.async\.bulk\.(commit_group|wait_group(\.read)? \d);$")


def assert_plain_tma(ptx: str) -> None:
    for line in ptx.splitlines():
        if "cp.async.bulk" in line or "cp.reduce.async.bulk" in line:
            assert TMA_LOAD.match(line) or TMA_OUT.match(line) or BULK_GROUP.match(line), \
                f"unexpected bulk-copy form: {line.strip()}"
        # the only multicast form allowed is tcgen05.commit's arrival on both CTAs of a pair
        assert "multicast" not in line or line.lstrip().startswith("tcgen05.commit"), \
            f"multicast outside tcgen05.commit: {line.strip()}"


SMALL = {
    "c1": lambda: problems.pointwise_add(3000),
    "c2": lambda: problems.gelu_chain(64, 256),
    "c3": lambda: problems.row_softmax(8, 1024),
    "c4": lambda: problems.full_sum(1 << 20, 256, 16),
    "c5": lambda: problems.matmul(256, 256, 256),
    "c5b": lambda: problems.matmul(256, 256, 512, split_k=2, raster_group=None),
}


@pytest.mark.parametrize("key", sorted(SMALL))
def test_configs_assemble(key: str, tmp_path) -> None:
    ptx = compile_spec(SMALL[key]())
    assert_plain_tma(ptx)
    info = ptxas(ptx, tmp_path)
    assert "spill" in info


def test_full_size_configs_assemble(tmp_path) -> None:
    for key in ("c1_vector_add", "c2_gelu_chain", "c3_row_softmax", "c4_full_sum"):
        ptxas(compile_spec(problems.CONFIGS[key]()), tmp_path)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_gemm_rank_shares_assemble(world: int, tmp_path) -> None:
    """The GEMM kernel one rank of ``world`` compiles for configs 5 and 5b (rows of A and C on
    SM pairs down to the 1/8 share's 128 rows on single SMs; 5b also along K), through the
    template, with plain TMA only; each module assembles."""
    from ptxgen import shard

    for name, ksplit in (("c5_matmul", False), ("c5b_matmul_splitk", False),
                         ("c5b_matmul_splitk", True)):
        ptx = compile_spec(shard.local_problem(name, world, ksplit=ksplit).spec)
        assert "tcgen05.mma" in ptx, (name, world)
        assert_plain_tma(ptx)
        ptxas(ptx, tmp_path)


def test_pointwise_is_vectorised() -> None:
    ptx = compile_spec(problems.pointwise_add(1 << 20))
    assert ptx.count("ld.global.nc.v4.f32") == 2
    assert ptx.count("st.global.v4.f32") == 1
    assert "add.rn.f32" in ptx and "bra" not in ptx  # no tail guard: every block is full


def test_tail_guard_only_when_needed() -> None:
    assert "bra" in compile_spec(problems.pointwise_add(3000))  # 750 cells, blocks of 256
    assert "bra" not in compile_spec(problems.pointwise_add(4096))


def test_gelu_packs_bf16_128_bit() -> None:
    ptx = compile_spec(problems.gelu_chain(64, 256, unroll=8))
    assert ptx.count("ld.global.nc.v4.b32") == 1 and ptx.count("st.global.v4.b32") == 1
    assert ptx.count("ld.global.nc.f32") == 3  # a, b and one s[row] for all eight elements
    assert "fma.rn.f32" in ptx and "ex2.approx.ftz.f32" in ptx


def test_gelu_no_fusion_flag() -> None:
    """Without fusion only tanh's own fma remains: one per element, against three with it
    (a*x + b and u + c*u^3 fuse)."""
    spec = problems.gelu_chain(64, 256, unroll=8)
    fused, plain = compile_spec(spec), compile_spec(spec, no_fusion=True)

    def fma_lanes(ptx: str) -> int:
        return 2 * ptx.count("fma.rn.f32x2") + len(re.findall(r"fma\.rn\.f32 ", ptx))

    assert fma_lanes(plain) == plain.count("rcp.approx") == 8
    assert fma_lanes(fused) == 3 * 8


def test_gelu_pairs_arithmetic_into_f32x2() -> None:
    ptx = compile_spec(problems.gelu_chain(64, 256, unroll=16))
    assert ptx.count(".f32x2") >= 16 * 10 // 2
    assert not re.search(r"\b(add|sub|mul|fma)\.rn\.f32 ", ptx)  # no scalar f32 arithmetic left


def test_softmax_reads_each_row_once() -> None:
    ptx = compile_spec(problems.row_softmax(8, 4096, 256))
    assert ptx.count("ld.global.nc.f32") == 4096 // 256  # passes 2 and 3 reuse pass 1's loads
    assert ptx.count("ex2.approx") == 4096 // 256
    assert "redux.sync.max.f32" in ptx


def test_no_cse_reloads() -> None:
    ptx = compile_spec(problems.row_softmax(8, 4096, 256), no_cse=True)
    assert ptx.count("ld.global.nc.f32") == 3 * 4096 // 256


def test_no_unroll_makes_runtime_loops() -> None:
    ptx = compile_spec(problems.row_softmax(8, 4096, 256), no_unroll=True)
    assert ptx.count("$L_loop_") >= 3 * 2


def test_sum_unrolls_grid_stride_loop() -> None:
    """Config 4's counted loop runs 16 copies of its body a trip. The trip's 16 rows of 128
    bytes a warp come in as 8 8-byte loads a lane, go through a warp-private shared area, and
    each lane adds its own 16 elements in their order (``stage.py``)."""
    ptx = compile_spec(problems.CONFIGS["c4_full_sum"]())
    loop = ptx[ptx.index("$L_loop_1:"):ptx.index("$L_loop_end_2:")]
    assert loop.count("ld.global.nc.v2.f32") == 8 and loop.count("st.shared.v2.f32") == 8
    assert loop.count("ld.shared.f32") == 16 and loop.count("bar.warp.sync") == 2
    assert "ld.global.nc.f32" not in loop
    assert "red.global.add.f32" in ptx
    # no immediate offset beyond 2^30 bytes
    offs = [int(m) for m in re.findall(r"\[%rd\d+\+(\d+)\]", ptx)]
    assert max(offs) < 2**30


def test_cli_contract(tmp_path) -> None:
    graph, meta = shipped("p02_scale_shift")
    d = tmp_path / "p02"
    d.mkdir()
    (d / "k.ir.json").write_text(json.dumps(graph))
    (d / "meta.json").write_text(json.dumps(meta))
    for flags in ([], ["--no_loop_unroll"], ["--no_fusion"], ["--no_cse"]):
        r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(d / "k.ir.json"),
                            *flags], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert r.stdout.startswith("//") and ".visible .entry k_add_pointwise(" in r.stdout


def test_cli_fails_loudly(tmp_path) -> None:
    graph, meta = shipped("p02_scale_shift")
    meta["kernels"][0]["grid"] = [4, 2, 1]  # a 2-D launch is not supported
    d = tmp_path / "bad"
    d.mkdir()
    (d / "k.ir.json").write_text(json.dumps(graph))
    (d / "meta.json").write_text(json.dumps(meta))
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(d / "k.ir.json")],
                       capture_output=True, text=True)
    assert r.returncode != 0 and "NotImplementedError" in r.stderr
    meta["kernels"][0]["grid"] = [4, 1, 1]
    meta["kernels"][0]["entry"] = "no_such_kernel"
    (d / "meta.json").write_text(json.dumps(meta))
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(d / "k.ir.json")],
                       capture_output=True, text=True)
    assert r.returncode != 0 and "ValueError" in r.stderr


def test_unsupported_node_raises() -> None:
    graph, meta = shipped("p02_scale_shift")
    body = graph["nodes"]["add"]["op_fields"]["body"][0]
    graph["nodes"]["add"]["op_fields"]["body"][0] = body.replace("swizzle='NONE'",
                                                                 "swizzle='XOR'")
    with pytest.raises(NotImplementedError):
        to_ptx(Graph.from_dict(graph), meta)


def test_gemm_uses_the_tcgen05_template() -> None:
    ptx = compile_spec(problems.CONFIGS["c5_matmul"]())
    # 256-row tiles on SM pairs: one A and two B loads (this CTA's half of B) a stage
    assert "tcgen05.mma.cta_group::2.kind::f16" in ptx and "tcgen05.alloc.cta_group::2" in ptx
    assert ".reqnctapercluster 2, 1, 1" in ptx and "cluster=2" in ptx
    loads = "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global"
    assert ptx.count(loads) == 1 + 128 // 64
    # an odd number of 128-row tiles keeps one SM per tile: one A and four B loads a stage
    single = compile_spec(problems.matmul(384, 512, 512))
    assert "tcgen05.mma.cta_group::1.kind::f16" in single and ".reqnctapercluster" not in single
    assert single.count("cp.async.bulk.tensor.2d.shared::cluster.global") == 1 + 256 // 64
    assert_plain_tma(single)
    assert "// @ptxgen tensormap symbol=" in ptx and "persistent=1" in ptx
    assert_plain_tma(ptx)
    generic = to_ptx(Graph.from_dict(problems.matmul(256, 256, 256).graph),
                     problems.matmul(256, 256, 256).meta, templates=False)
    assert "tcgen05" not in generic and "cp.async.cg.shared.global" in generic


def test_stream_k_tail_plan_and_table(tmp_path) -> None:
    """Config 5's 1/4 share (256 pair tiles: three waves of 74 and 34 more) cuts its 34 tail
    tiles along K into two pieces each; the full kernel, the 1/2 share and the 1/8 share keep
    whole tiles. The table covers every K block of every tile once: the whole tiles first in
    raster order, then the pieces split-major. The module carries the partials' workspace and
    one counter per tail tile and epilogue warp, adds to a counter with acquire-release order,
    reads partials through L2, and clears the counter; nothing in it waits on another CTA."""
    from collections import Counter

    from ptxgen import shard
    from ptxgen.templates import matmul
    from ptxgen.templates.matmul import BK, ROLE_PIECE, ROLE_WHOLE

    plans = {n: gemm_plan(shard.local_problem("c5_matmul", n).spec) for n in (1, 2, 4, 8)}
    assert [plans[n].tail() for n in (1, 2, 4, 8)] == [None, None, (222, 2), None]
    p = plans[4]
    table = p.tail_table()
    kbs = p.k // BK
    cover = Counter()
    for mt, nt, kb0, cnt, *_ in table:
        cover.update((mt, nt, kb) for kb in range(kb0, kb0 + cnt))
    assert set(cover.values()) == {1} and len(cover) == len(p.order()) * kbs
    whole = [e for e in table if e[4] == ROLE_WHOLE]
    pieces = [e for e in table if e[4] == ROLE_PIECE]
    assert [e[:4] for e in whole] == [(mt, nt, 0, kbs) for mt, nt in p.order()[:222]]
    tails = p.order()[222:]
    assert [(e[0], e[1], e[5], e[6], e[7]) for e in pieces] == \
        [(mt, nt, j, 2, u) for j in range(2) for u, (mt, nt) in enumerate(tails)]
    ptx = matmul.emit(p)
    name = p.entry
    assert "tail=222,2" in ptx
    assert f".global .align 16 .b8 {name}_ws[{34 * 2 * 8 * 32 * 256 * 4}];" in ptx
    assert f".global .align 4 .u32 {name}_cnt[{34 * 8}];" in ptx
    assert ptx.count("atom.acq_rel.gpu.global.add.u32") == 1
    assert "ld.global.cg.v4.f32" in ptx and "st.relaxed.gpu.global.u32" in ptx
    assert "ld.acquire" not in ptx and "griddepcontrol" not in ptx
    assert_plain_tma(ptx)
    ptxas(ptx, tmp_path)
    import dataclasses

    assert dataclasses.replace(p, stream_k=False).tail() is None


def test_splitk_module_zeroes_c_itself(tmp_path) -> None:
    """A split-K GEMM's module carries the kernel that zeroes C (named in a ``zero`` note the
    launcher reads), whose first instruction lets the next launch start, and whose stores
    cover exactly C's bytes; the GEMM waits (``griddepcontrol.wait``) at the top of its
    epilogue, before any reduce-add into C. A plain GEMM has neither. Both assemble."""
    import re

    from ptxgen.runtime import header_notes
    from ptxgen.templates.matmul import ZERO_BLOCK, ZERO_GRID

    spec = problems.CONFIGS["c5b_matmul_splitk"]()
    ptx = compile_spec(spec)
    note = header_notes(ptx)["zero"]
    entry = f"{spec.kernel['entry']}_zero"
    assert note == [f"entry={entry} buffer=matmul grid={ZERO_GRID} block={ZERO_BLOCK}"]
    zero = ptx[ptx.index(f".visible .entry {entry}("):]
    body = [ln.strip() for ln in zero.splitlines() if ln.startswith("\t")]
    first = next(ln for ln in body if not ln.startswith((".reg", ".param")))
    assert first == "griddepcontrol.launch_dependents;"
    assert re.search(rf"setp\.lt\.u32 %z_p, %z_i, {1024 * 1024 * 4 // 16};", zero)
    assert "st.global.v4.b32 [%z_a], {0, 0, 0, 0};" in zero
    main = ptx[:ptx.index(f".visible .entry {entry}(")]
    epi = main[main.index("$M_epilogue:"):]
    assert epi.index("griddepcontrol.wait;") < epi.index("cp.reduce.async.bulk.tensor")
    assert main.count("griddepcontrol") == 1
    plain = compile_spec(problems.CONFIGS["c5_matmul"]())
    assert "griddepcontrol" not in plain and "zero" not in header_notes(plain)
    ptxas(ptx, tmp_path)


def test_gemm_epilogue_wait_is_warp_uniform(tmp_path) -> None:
    """The epilogue's warps go from their accumulator wait to warp-collective ``tcgen05.ld``:
    that wait leaves only through warp votes (all lanes saw the phase, or no lane has time
    left) and uniform branches, so no lane reaches ``tcgen05.ld.sync.aligned`` alone. The
    single-thread waits (producer, MMA issuer) keep their per-lane form. The probe kernels of
    both forms assemble."""
    import re

    from ptxgen.templates.matmul import wait_probe_ptx

    for spec in (problems.CONFIGS["c5_matmul"](), problems.matmul(384, 512, 512)):
        ptx = compile_spec(spec)
        epi = ptx[ptx.index("$M_epilogue:"):ptx.index("tcgen05.ld.sync.aligned")]
        waits = re.findall(r"mbarrier\.try_wait[^\n]*\n\s*(\S+)[^\n]*\n\s*([^\n]*)", epi)
        assert len(waits) == 1, waits
        assert waits[0][0] == "vote.sync.all.pred" and "bra.uni" in waits[0][1]
        assert "vote.sync.any.pred" in epi and "%laneid" in epi
        assert not re.search(r"@%m_pw2 bra \$", epi)  # no per-lane retry branch
        head = ptx[:ptx.index("$M_epilogue:")]
        assert "vote.sync" not in head  # one-thread waits stay per lane
    for warp in (False, True):
        for arrive in (False, True):
            ptxas(wait_probe_ptx(1000, warp=warp, arrive=arrive), tmp_path)


def test_gemm_staged_epilogue_structure(tmp_path) -> None:
    """The staged epilogue: C's tensor map (f32, 32 x 32 box, 128-byte swizzle) beside A's and
    B's; per block, lane 0 waits for the buffer's previous TMA read, the warp stores and fences
    the generic stores to the async proxy before lane 0's TMA op (a reduce-add for split-K, a
    store otherwise); the teardown waits for every bulk group; shared memory fits the limit."""
    import re

    from ptxgen.templates.matmul import SMEM_LIMIT

    for key, op in (("c5b_matmul_splitk", "cp.reduce.async.bulk.tensor.2d.global.shared::cta"
                     ".add.tile.bulk_group"),
                    ("c5_matmul", "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group")):
        ptx = compile_spec(problems.CONFIGS[key]())
        note = next(ln for ln in ptx.splitlines() if "_tmap_c" in ln and "@ptxgen" in ln)
        assert "dtype=f32" in note and "box=32,32" in note and "swizzle=128" in note
        epi = ptx[ptx.index("$M_epilogue:"):ptx.index("$M_teardown:")]
        assert epi.count(op) == 8 and "red.global.add" not in epi and "st.global" not in epi
        first = epi.index("cp.async.bulk.wait_group.read 1")
        assert first < epi.index("st.shared.v4.b32") < epi.index("fence.proxy.async.shared::cta")
        assert epi.index("fence.proxy.async.shared::cta") < epi.index(op)
        tail = ptx[ptx.index("$M_teardown:"):]
        assert tail.index("cp.async.bulk.wait_group 0") < tail.index("tcgen05.dealloc")
        smem = int(re.search(r"dynamic_smem=(\d+)", ptx).group(1))
        assert smem <= SMEM_LIMIT
        assert_plain_tma(ptx)
        ptxas(ptx, tmp_path)


def test_launch_notes_give_the_module_its_shared_memory() -> None:
    """Every ``// @ptxgen`` note the runtime reads parses, ``dynamic_smem=N`` included: a
    launch asks for the larger of meta.json's ``smem_bytes`` and the module's own figure (the
    GEMM template's layout is larger than meta.json's 198,656 bytes), and the template checks
    at entry that it got what its layout needs."""
    import re

    from ptxgen.runtime import header_notes
    from ptxgen.templates.matmul import SMEM_SHORT

    spec = problems.CONFIGS["c5b_matmul_splitk"]()
    ptx = compile_spec(spec)
    notes = header_notes(ptx)
    want = int(re.search(r"// @ptxgen dynamic_smem=(\d+)", ptx).group(1))
    assert int(notes["dynamic_smem"][0]) == want > int(spec.kernel["smem_bytes"])
    assert {"launch", "tensormap", "matmul"} <= set(notes) and len(notes["tensormap"]) == 3
    assert "%dynamic_smem_size" in ptx and f"[ptxgen_status], {1 << SMEM_SHORT}" in ptx
    head = ptx[:ptx.index("mbarrier.init")]
    assert "ret;" in head  # a short launch leaves before any barrier exists


def test_single_wave_runtime_loops_copy_ahead(tmp_path) -> None:
    """The shipped r02 (one 128-thread block summing 65,536 floats) with unrolling off: its
    rolled loop takes each trip's value from a shared-memory ring that ``cp.async`` fills
    ``DEPTH - 1`` trips ahead, read into registers one trip ahead. In front of the loop, trips
    0 .. DEPTH-2 are copied (trip j > 0 only where it exists), one commit group each, and trip
    0's slot is read once its group has landed. Each trip takes the value read ahead, waits for
    trip t + 1's group (``wait_group DEPTH-3``) and reads its slot, copies trip t + DEPTH - 1
    (where it exists) through the same induction pointer into trip t - 1's slot, and adds one
    value, in trip order; the loop waits for every copy after it. The ring replaces the L1
    prefetch. The default build unrolls instead; a kernel of several waves gets neither."""
    import re

    from ptxgen.pipeline import DEPTH

    graph, meta = shipped("r02_big_sum")
    rolled = to_ptx(Graph.from_dict(graph), meta, no_unroll=True)
    loop = rolled[rolled.index("$L_loop_1:"):rolled.index("$L_loop_end")]
    head = rolled[:rolled.index("$L_loop_1:")]
    assert "prefetch" not in rolled and "ld.global" not in loop
    assert re.search(r"\.shared \.align 16 \.b8 k_sum_1_reduce_ring0\[(\d+)\];", rolled).group(1) \
        == str(DEPTH * 128 * 4)
    fills = re.findall(r"(@%p\d+ )?cp\.async\.ca\.shared\.global \[%r\d+\+(\d+)\], "
                       r"\[%rd\d+\+(\d+)\], 4;", head)
    assert [(bool(p), int(d), int(s)) for p, d, s in fills] == \
        [(j > 0, j * 512, j * 512) for j in range(DEPTH - 1)]
    assert head.count("cp.async.commit_group") == DEPTH - 1
    first = re.search(rf"cp\.async\.wait_group {DEPTH - 2};\n\tld\.shared\.f32 (%f\d+), "
                      r"\[%r\d+\];", head)
    assert first, head[-600:]
    ahead = first.group(1)
    # the trip's value is the one read ahead; then trip t + 1's slot is read into its place
    value = re.search(rf"mov\.f32 (%f\d+), {re.escape(ahead)};", loop).group(1)
    assert loop.index(f"mov.f32 {value}") < loop.index(f"cp.async.wait_group {DEPTH - 3};") < \
        loop.index(f"ld.shared.f32 {ahead}, ")
    refill = re.search(r"@(%p\d+) cp\.async\.ca\.shared\.global \[%r\d+\+0\], "
                       r"\[(%rd\d+)\+(\d+)\], 4;", loop)
    step = re.search(r"add\.s64 (%rd\d+), %rd\d+, 512;", loop)
    assert refill and refill.group(2) == step.group(1) and int(refill.group(3)) == (DEPTH - 1) * 512
    guard = re.search(rf"setp\.lt\.s32 {re.escape(refill.group(1))}, (%r\d+), 65536;", loop)
    assert guard and re.search(rf"add\.u32 {re.escape(guard.group(1))}, %r\d+, "
                               rf"{(DEPTH - 1) * 128};", loop)
    assert loop.count("cp.async.commit_group") == 1 and loop.count("add.rn.f32") == 1
    assert re.search(rf"add\.rn\.f32 (%f\d+), \1, {re.escape(value)};", loop)
    after = rolled[rolled.index("@%p1 bra $L_loop_1;"):rolled.index("$L_loop_end")]
    assert "cp.async.wait_all" in after
    default = to_ptx(Graph.from_dict(graph), meta)
    assert "cp.async" not in default and "$L_loop" not in default
    wide = compile_spec(problems.CONFIGS["c4_full_sum"]())  # 1184 blocks: several waves
    assert "cp.async" not in wide and "prefetch" not in wide
    ptxas(rolled, tmp_path)


def gemm_plan(spec: problems.ProblemSpec):
    from ptxgen.compiler import kernel_for_meta
    from ptxgen.lower import Buffer
    from ptxgen.templates import matmul

    op, launch = kernel_for_meta(Graph.from_dict(spec.graph), spec.meta)
    bufs = {a["name"]: Buffer(tuple(a["shape"]), a["dtype"],
                              bool(a.get("output")) or a["name"] in op.outputs)
            for a in launch["args"]}
    return matmul.match(op, bufs, launch["arg_order"], launch["block"][0],
                        int(launch.get("smem_bytes", 0)))


@pytest.mark.parametrize("shape", [(8192, 8192, 8192, 1), (1024, 1024, 65536, 4),
                                   (384, 512, 768, 3), (256, 256, 1024, 4),
                                   (128, 1024, 65536, 32), (640, 768, 4096, 2)])
def test_gemm_segments_cover_every_k_block_once(shape) -> None:
    """The template's work table: every K block of every output tile exactly once; a plain GEMM
    takes its tiles in the template's grouped raster (groups of isqrt(CTAs at once) tile rows,
    rows fastest); a split-K GEMM goes split-major over the IR's tiles, with splits of at least
    MIN_SEGMENT K blocks that differ by at most one, in as few waves of SM_COUNT CTAs as its
    split count needs."""
    from collections import Counter

    import math

    from ptxgen.templates.matmul import BK, MIN_SEGMENT, SM_COUNT, raster

    m, n, k, split = shape
    kw = {"split_k": split, "raster_group": None} if split > 1 else {}
    p = gemm_plan(problems.matmul(m, n, k, **kw))
    table, ctas = p.segments()
    rows = 2 if p.pair else 1  # a pair's table tiles are two of the IR's 128-row tiles
    assert p.pair == (m % 256 == 0)
    seen = Counter()
    for mt, nt, kb0, cnt in table:
        seen.update((mt * rows + r, nt, kb) for kb in range(kb0, kb0 + cnt) for r in range(rows))
    tiles = list(dict.fromkeys((mt, nt) for mt, nt, _ in p.schedule))
    kbs = k // BK
    assert set(seen) == {(mt, nt, kb) for mt, nt in tiles for kb in range(kbs)}
    assert set(seen.values()) == {1}
    order = list(dict.fromkeys((mt // rows, nt) for mt, nt, _ in p.schedule))
    if split == 1:
        want = raster(m // (128 * rows), n // p.bn, math.isqrt(SM_COUNT // rows))
        assert [(mt, nt) for mt, nt, _, _ in table] == want == p.order()
        assert sorted(want) == sorted(order) and ctas == len(table) * rows
        return
    splits = len(table) // len(order)
    assert [(mt, nt) for mt, nt, _, _ in table] == order * splits
    counts = {cnt for _, _, _, cnt in table}
    assert max(counts) - min(counts) <= 1 and min(counts) >= min(MIN_SEGMENT, kbs)
    assert ctas == min(SM_COUNT // rows, len(table)) * rows


def test_splitk_config_fills_the_sms() -> None:
    """Config 5b (16 pair tiles of 1024 K blocks): 9 splits, two full waves over 74 SM pairs."""
    table, ctas = gemm_plan(problems.CONFIGS["c5b_matmul_splitk"]()).segments()
    assert (len(table), ctas) == (144, 148)


def proportional(monkeypatch) -> None:
    """A cost model in which a tile's K block takes time in proportion to its width: the one
    that makes the planner cut a part-full last wave into mixed widths."""
    from ptxgen.templates import matmul

    monkeypatch.setattr(matmul, "K_BLOCK_TIME", {w: w / 256 for w in matmul.K_BLOCK_TIME})


@pytest.mark.parametrize("shape,scaled", [((512, 512, 512), False), ((1024, 1024, 1024), False),
                                          ((256, 256, 256), False), ((1024, 8192, 8192), True),
                                          ((2048, 8192, 8192), True), ((1280, 512, 256), True),
                                          ((4096, 4096, 2048), True)])
def test_gemm_mixed_widths_cover_c_once(shape, scaled, monkeypatch) -> None:
    """The mixed-width table (under the measured cost model, or a width-proportional one that
    cuts part-full last waves): every column of every 256-row band of C in exactly one tile;
    widths from 256 and ``NARROW``, each tile inside C and starting on a 32-column boundary (the
    table stores column / 32; TMA wants 16-byte starts); entry r * used + q is pair q's r-th
    tile, and the longest pair's work (in the planner's own cost) is below whole tiles' waves."""
    from collections import Counter

    from ptxgen.templates import matmul
    from ptxgen.templates.matmul import BK, MIXED_GAIN, NARROW, SEGMENT_COST, SM_COUNT

    if scaled:
        proportional(monkeypatch)
    m, n, k = shape
    p = gemm_plan(problems.matmul(m, n, k))
    table, ctas = p.columns()
    used = ctas // 2
    assert used <= SM_COUNT // 2 and len(table) % used == 0
    cover = Counter()
    work = [0.0] * used
    kbs = k // BK
    for i, (band, col, w) in enumerate(table):
        if not w:
            continue
        assert w in (256, *NARROW) and col % 32 == 0 and col + w <= n and band < m // 256
        cover.update((band, c) for c in range(col, col + w))
        work[i % used] += kbs * matmul.K_BLOCK_TIME[w] + SEGMENT_COST
    assert set(cover.values()) == {1} and len(cover) == (m // 256) * n
    whole = -(-(m // 256) * (n // 256) // (SM_COUNT // 2)) * (kbs + SEGMENT_COST)
    assert max(work) <= (1 - MIXED_GAIN) * whole


def test_config5_shares_tile_widths(monkeypatch) -> None:
    """Config 5's kernel and every share of it keep whole 256-column tiles: a narrower tile runs
    a K block in nearly a whole tile's time on a B200, so cutting the part-full last wave of the
    1/4 and 1/8 shares (256 and 128 tiles over 74 pairs) gains nothing (measured: 96.6 against
    96.4 us at 1/8). Under a width-proportional model the planner would give the longest pair
    3.5 and 1.75 tiles' worth instead of 4 and 2."""
    from ptxgen import shard

    def longest(share: int) -> float:
        table, ctas = gemm_plan(shard.local_problem("c5_matmul", share).spec).columns()
        cols = [0] * (ctas // 2)
        for i, (_, _, w) in enumerate(table):
            cols[i % len(cols)] += w
        return max(cols) / 256

    for share in (1, 2, 4, 8):
        assert gemm_plan(shard.local_problem("c5_matmul", share).spec).columns() is None
    proportional(monkeypatch)
    assert (longest(4), longest(8)) == (3.5, 1.75)


def _normalised(lines: list[str]) -> list[str]:
    """Instruction lines with registers renamed by first appearance (inputs kept), and the
    explicit ``.rn`` of an f32 mul/add dropped: a lone IEEE multiply or add rounds to nearest
    either way, the suffix only bars ptxas from contracting it with a neighbour."""
    names: dict[str, str] = {}

    def rename(m: re.Match) -> str:
        r = m.group(0)
        if r.startswith("%in"):
            return r
        return names.setdefault(r, f"%v{len(names)}")

    out = []
    for line in lines:
        line = line.strip().rstrip(";").replace("mul.rn.f32 ", "mul.f32 ").replace(
            "add.rn.f32 ", "add.f32 ")
        out.append(re.sub(r"%[a-z]+\d+", rename, line))
    return out


@pytest.mark.parametrize("name", ["exp", "log", "pow", "tanh", "erf", "sin", "cos", "sigmoid"])
def test_fastmath_matches_reference_sequence(name: str) -> None:
    """Each fast-math function emits the instruction sequence the reference's does (fixture
    ``tests/golden/fastmath.json``, written by the reference's own ``ptxgen/fastmath.py``), so a
    fast-math result is the reference's bit for bit on the same hardware."""
    from conftest import ROOT

    from ptxgen.fastmath import F32_FUNCS
    from ptxgen.ptx import Kernel

    golden = json.loads((ROOT / "tests" / "golden" / "fastmath.json").read_text())[name]
    k = Kernel("t", [], 32)
    out = F32_FUNCS[name](k, *["%in0", "%in1"][:2 if name == "pow" else 1])
    ours = _normalised([ins.render() for ins in k.body] + [f"result {out}"])
    want = _normalised(golden["body"] + [f"result {golden['out']}"])
    assert ours == want


def _shared_loads(between: str | None) -> list[str]:
    """Vectorize two f32 shared loads at [a+0] and [a+4] (a 16-byte aligned), with ``between``
    ("st": a shared store, "ld": another shared load, None) placed between them."""
    from ptxgen.ptx import Kernel

    k = Kernel("t", [], 128)
    a = k.reg("u32")
    k.align[a] = 16
    x, y, z = k.reg("f32"), k.reg("f32"), k.reg("f32")
    k.mem("ld", "shared", "f32", a, 0, (x,))
    if between == "st":
        k.mem("st", "shared", "f32", a, 4, (z,))
    elif between == "ld":
        k.mem("ld", "shared", "f32", a, 8, (z,))
    k.mem("ld", "shared", "f32", a, 4, (y,))
    k.vectorize()
    return [ins.render().strip() for ins in k.body]


def test_shared_loads_merge_unless_a_shared_store_sits_between() -> None:
    """Adjacent shared loads become one vector load; a shared store between them keeps them
    apart, since the second load must read what the store wrote."""
    assert any(line.startswith("ld.shared.v2.f32") for line in _shared_loads(None))
    assert any(line.startswith("ld.shared.v2.f32") for line in _shared_loads("ld"))
    kept = _shared_loads("st")
    assert sum(line.startswith("ld.shared.f32") for line in kept) == 2
    assert not any(".v2" in line or ".v4" in line for line in kept)


def test_simt_matmul_reads_shared_memory_in_vectors() -> None:
    """The shipped m01 nest on the generic lowering (the default build takes the register-blocked
    template): A's four consecutive k of one row in one v4 load, B's two columns of one thread
    in one v2 load; no scalar shared loads remain."""
    graph, meta = shipped("m01_matmul_512")
    ptx = to_ptx(Graph.from_dict(graph), meta, templates=False)
    assert ptx.count("ld.shared.v4.f32") == 64 and ptx.count("ld.shared.v2.f32") == 128
    assert "ld.shared.f32" not in ptx


def _loop_bodies(ptx: str) -> list[list[str]]:
    """The instruction mnemonics of each innermost runtime loop, in order."""
    out = []
    # a body that holds no other loop's label: from a loop's top to the first loop end after it
    for m in re.finditer(r"(\$L_loop_\d+):\n((?:(?!\$L_loop_\d+:).)*?)\n\$L_loop_end_\d+:", ptx,
                         re.S):
        lines = [ln.strip() for ln in m.group(2).splitlines()]
        out.append([ln.split()[0] for ln in lines if ln and not ln.startswith(("$", "//"))])
    return out


def test_flat_runtime_loops_step_induction_pointers() -> None:
    """A runtime loop with no loop inside or around it loads through a 64-bit pointer its latch
    steps: r02's loop with unrolling off (128 threads x 4 bytes a trip) and config 4's
    grid-stride sum (copies of 148 x 8 blocks x 256 threads x 4 bytes). A loop nested in another,
    like
    a01's dot products with unrolling off, keeps its index arithmetic: a pointer there stays
    live beside the outer loop's state, and ptxas spilled."""
    graph, meta = shipped("r02_big_sum")
    body = _loop_bodies(to_ptx(Graph.from_dict(graph), meta, no_unroll=True))[0]
    # the trip's value comes from the copy ring the pointer feeds (see the copy-ahead test)
    assert body.count("ld.shared.f32") == 1 and body.count("add.s64") == 1
    assert not {"mul.wide.u32", "mad.lo.u32"} & set(body)
    step = re.search(r"add\.s64 (%rd\d+), \1, (\d+);", compile_spec(problems.full_sum(1 << 30)))
    assert step and int(step.group(2)) % (148 * 8 * 256 * 4) == 0
    graph, meta = shipped("a01_attention")
    body = next(b for b in _loop_bodies(to_ptx(Graph.from_dict(graph), meta, no_unroll=True))
                if "fma.rn.f32" in b)
    assert "mul.wide.u32" in body
    # with CSE off every address is computed again on every trip
    graph, meta = shipped("r02_big_sum")
    body = _loop_bodies(to_ptx(Graph.from_dict(graph), meta, no_unroll=True, no_cse=True))[0]
    assert "mul.wide.u32" in body

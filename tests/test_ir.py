"""The Kernel IR loader against the reference's shipped IR fixtures, and the generator's IRs."""

from __future__ import annotations

import json

import pytest
from conftest import GOLDEN, SHIPPED, shipped

from ptxgen import problems
from ptxgen.compiler import kernel_for_meta
from ptxgen.ir import Graph, IRError, Tile, parse_body, walk


@pytest.mark.parametrize("name", SHIPPED)
def test_shipped_body_round_trips(name: str) -> None:
    """Loading a shipped KernelOp body and writing it back gives the same string."""
    graph, _ = shipped(name)
    bodies = [n["op_fields"]["body"][0] for n in graph["nodes"].values()
              if n["op"] == "KernelOp"]
    assert bodies
    for text in bodies:
        assert repr(parse_body(text)) == text


@pytest.mark.parametrize("name", SHIPPED)
def test_shipped_kernel_found_by_meta(name: str) -> None:
    graph, meta = shipped(name)
    op, launch = kernel_for_meta(Graph.from_dict(graph), meta)
    assert op.name == launch["entry"]
    assert isinstance(op.body, Tile)
    assert -(-op.body.n_elements // launch["block"][0]) == launch["grid"][0]


def test_tile_facts() -> None:
    graph, _ = shipped("m01_matmul_512")
    op = Graph.from_dict(graph).kernel_ops()[0]
    assert op.body.extents == (16, 8, 16, 32)
    assert op.body.n_elements == 65536
    assert set(op.smem_buffers) == {"_a_smem", "_b_smem"}


@pytest.mark.parametrize("bad", ["Tile(", "Foo(x=1)", "1 + 2", "Tile(axes=(), body=(), "
                                 "block_threads=1, bogus=3)"])
def test_loader_rejects(bad: str) -> None:
    with pytest.raises((IRError, NotImplementedError, TypeError)):
        parse_body(bad)


@pytest.mark.parametrize("make", [
    lambda: problems.pointwise_add(4096), lambda: problems.gelu_chain(16, 64),
    lambda: problems.row_softmax(4, 512), lambda: problems.full_sum(1 << 16, 64, 4),
    lambda: problems.matmul(256, 256, 128), lambda: problems.matmul(128, 256, 256, split_k=2),
])
def test_generated_round_trip(make, tmp_path) -> None:
    spec = make()
    d = spec.write(tmp_path / "p")
    graph = json.loads(next(d.glob("*.ir.json")).read_text())
    meta = json.loads((d / "meta.json").read_text())
    op, launch = kernel_for_meta(Graph.from_dict(graph), meta)
    assert repr(op.body) == graph["nodes"][launch["node"]]["op_fields"]["body"][0]
    assert -(-op.body.n_elements // launch["block"][0]) == launch["grid"][0]
    assert list(walk([op.body]))


def test_literal_golden() -> None:
    """Literal encodings match the reference's own encoder on the committed vectors."""
    from ptxgen.dtypes import literal

    data = json.loads((GOLDEN / "literals.json").read_text())
    for typ, table in data["literals"].items():
        for value, want in table.items():
            v = float(value) if typ != "int" else int(value)
            assert literal(v, typ if typ != "int" else "s32") == want, (typ, value)


def test_bf16_rounding_golden() -> None:
    import numpy as np

    from ptxgen.problems import bf16_bits

    data = json.loads((GOLDEN / "literals.json").read_text())
    x = np.array(data["bf16_inputs_f32_bits"], np.uint32).view(np.float32)
    want = np.array(data["bf16_rounded_f32_bits"], np.uint32) >> 16
    assert np.array_equal(bf16_bits(x).astype(np.uint32), want)


def test_to_ptx_takes_a_live_emmy_graph() -> None:
    """``to_ptx`` accepts the object the reference's ``to_ptx`` receives: an Emmy graph whose
    ``nodes`` hold Emmy op objects. Emmy is absent here, so the test stands in objects with
    Emmy's class names whose ``repr`` is Emmy's (the strings its JSON holds)."""
    import json
    from types import SimpleNamespace

    from conftest import shipped

    from ptxgen.compiler import to_ptx
    from ptxgen.ir import Graph

    graph, meta = shipped("a01_attention")

    class Stmt:
        def __init__(self, text: str):
            self.text = text

        def __repr__(self) -> str:
            return self.text

    def op_of(node: dict):
        cls = type(node["op"], (), {})
        op = cls()
        if node["op"] == "KernelOp":
            body = node["op_fields"]["body"]
            op.body = [Stmt(t) for t in (json.loads(body) if isinstance(body, str) else body)]
            op.name = node["op_fields"]["name"]
        return op

    emmy = SimpleNamespace(
        inputs=graph["inputs"], outputs=graph["outputs"],
        nodes={nid: SimpleNamespace(op=op_of(n), inputs=n.get("inputs", []),
                                    outputs=[SimpleNamespace(name=t["name"])
                                             for t in n.get("outputs", [])])
               for nid, n in graph["nodes"].items()})
    assert to_ptx(emmy, meta) == to_ptx(Graph.from_dict(graph), meta)

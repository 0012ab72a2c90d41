"""Emmy Kernel IR: node classes, a loader for the repr strings Emmy writes into ``<kernel>.ir.json``,
and a writer that produces the same strings.

Emmy (``emmy-ml==0.3.11``) is not a dependency. Its graph JSON stores each ``KernelOp`` body as
the Python ``repr`` of a ``Tile`` tree, for example
``Tile(axes=(Axis(name='a0', extent=Dim(1024), window=None),), body=(Load(...), ...), ...)``.
``parse_body`` reads that string with ``ast`` (never ``eval``) into the frozen dataclasses below,
and ``repr()`` of those dataclasses gives the string back character for character. The field
names and their order are Emmy's, as the shipped IR files show them (reference
``examples/*/*/*.ir.json``). Node-level facts that Emmy computes are restated here:
``Tile.extents``/``n_elements`` (the product of the axis extents), ``nested()``, ``defines()``
and ``deps()``.
"""

from __future__ import annotations

import ast
import json
import math
from collections.abc import Iterator, Sequence
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any

# --- leaf values ---------------------------------------------------------------------------


@dataclass(frozen=True)
class Dim:
    """A static axis extent (Emmy also has symbolic ones, which this backend rejects)."""

    value: int | str

    def __repr__(self) -> str:
        return f"Dim({self.value!r})"

    @property
    def is_static(self) -> bool:
        return isinstance(self.value, int)

    def as_static(self) -> int:
        if not isinstance(self.value, int):
            raise NotImplementedError(f"symbolic extent {self.value!r}")
        return self.value


@dataclass(frozen=True)
class NpDtype:
    """The ``np=dtype('float32')`` field of a DataType."""

    name: str

    def __repr__(self) -> str:
        return f"dtype({self.name!r})"


@dataclass(frozen=True)
class DataType:
    name: str
    np: NpDtype | None = None
    nbytes: int = 0


_NP_NAME = {"f32": "float32", "f64": "float64", "f16": "float16", "bf16": "bfloat16",
            "i32": "int32", "u32": "uint32", "i64": "int64", "u64": "uint64", "i16": "int16",
            "u16": "uint16", "u8": "uint8", "bool": "bool"}
_NBYTES = {"f32": 4, "f64": 8, "f16": 2, "bf16": 2, "i32": 4, "u32": 4, "i64": 8, "u64": 8,
           "i16": 2, "u16": 2, "u8": 1, "bool": 1}


def dt(name: str) -> DataType:
    """The DataType Emmy writes for dtype ``name``."""
    return DataType(name, NpDtype(_NP_NAME[name]), _NBYTES[name])


# Identities of Emmy's reduction ops, as an Accum or a seeding Loop starts them.
IDENTITY = {"add": 0.0, "sum": 0.0, "subtract": 0.0, "multiply": 1.0, "prod": 1.0,
            "maximum": -math.inf, "max": -math.inf, "amax": -math.inf,
            "minimum": math.inf, "min": math.inf, "amin": math.inf}


@dataclass(frozen=True)
class ElementwiseImpl:
    """An elementwise op, by Emmy's name (``'multiply'``, ``'exp'``, ...)."""

    name: str

    def __repr__(self) -> str:
        return f"ElementwiseImpl({self.name!r})"

    @property
    def identity(self) -> float | None:
        return IDENTITY.get(self.name)


# --- expressions ---------------------------------------------------------------------------


class Expr:
    def deps(self) -> Iterator[str]:
        return iter(())


@dataclass(frozen=True)
class Var(Expr):
    name: str

    def deps(self) -> Iterator[str]:
        yield self.name


@dataclass(frozen=True)
class Literal(Expr):
    value: Any
    dtype: str = "int"


@dataclass(frozen=True)
class BinaryExpr(Expr):
    op: str
    left: Expr
    right: Expr

    def deps(self) -> Iterator[str]:
        yield from self.left.deps()
        yield from self.right.deps()


@dataclass(frozen=True)
class TernaryExpr(Expr):
    cond: Expr
    if_true: Expr
    if_false: Expr

    def deps(self) -> Iterator[str]:
        for e in (self.cond, self.if_true, self.if_false):
            yield from e.deps()


@dataclass(frozen=True)
class FuncCallExpr(Expr):
    name: str
    args: tuple[Expr, ...] = ()

    def deps(self) -> Iterator[str]:
        for e in self.args:
            yield from e.deps()


@dataclass(frozen=True)
class CastExpr(Expr):
    dtype: str
    expr: Expr

    def deps(self) -> Iterator[str]:
        yield from self.expr.deps()


def _expr_deps(e: Any) -> Iterator[str]:
    if isinstance(e, Expr):
        yield from e.deps()
    elif isinstance(e, tuple):
        for x in e:
            yield from _expr_deps(x)


# --- statements ----------------------------------------------------------------------------


class Stmt:
    """A Kernel IR statement."""

    def nested(self) -> list[tuple[Stmt, ...]]:
        """The statement bodies inside this one."""
        return []

    def defines(self) -> tuple[str, ...]:
        """Names this statement binds (in its enclosing block)."""
        return ()

    def binds_axes(self) -> tuple[str, ...]:
        """Axis names this statement binds for its nested bodies."""
        return ()

    def deps(self) -> tuple[str, ...]:
        """Names this statement reads (not counting nested bodies)."""
        return ()


@dataclass(frozen=True)
class Window:
    parent: Axis
    base: Any = None
    bound: Any = None
    partition: bool = False


@dataclass(frozen=True)
class Axis:
    name: str
    extent: Dim
    window: Window | None = None


@dataclass(frozen=True)
class Tile(Stmt):
    axes: tuple[Axis, ...]
    body: tuple[Stmt, ...]
    block_threads: int
    aux_threads: int = 0
    raster_axes: tuple[str, ...] | None = None
    raster_group: int | None = None
    raster_orient: str = "m"

    def nested(self) -> list[tuple[Stmt, ...]]:
        return [self.body]

    def binds_axes(self) -> tuple[str, ...]:
        return tuple(a.name for a in self.axes)

    @property
    def extents(self) -> tuple[int, ...]:
        return tuple(a.extent.as_static() for a in self.axes)

    @property
    def is_static_grid(self) -> bool:
        return all(a.extent.is_static for a in self.axes)

    @property
    def n_elements(self) -> int:
        return math.prod(self.extents)


@dataclass(frozen=True)
class Loop(Stmt):
    axis: Axis
    body: tuple[Stmt, ...]
    unroll: bool = False
    seed: bool = True

    def nested(self) -> list[tuple[Stmt, ...]]:
        return [self.body]

    def binds_axes(self) -> tuple[str, ...]:
        return (self.axis.name,)


@dataclass(frozen=True)
class StridedLoop(Stmt):
    axis: Axis
    start: Expr
    step: Expr | int
    body: tuple[Stmt, ...]
    unroll: bool = False
    end: Expr | None = None
    seed: bool = True

    def nested(self) -> list[tuple[Stmt, ...]]:
        return [self.body]

    def binds_axes(self) -> tuple[str, ...]:
        return (self.axis.name,)

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps((self.start, self.step, self.end)))


@dataclass(frozen=True)
class Load(Stmt):
    names: tuple[str, ...]
    input: str
    index: tuple[Expr, ...]
    dtype: DataType | None = None

    def defines(self) -> tuple[str, ...]:
        return tuple(self.names)

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps(self.index))


@dataclass(frozen=True)
class Write(Stmt):
    output: str
    index: tuple[Expr, ...]
    values: tuple[str, ...]
    value_dtype: DataType | None = None
    atomic: bool = False
    swizzle: str = "NONE"

    def deps(self) -> tuple[str, ...]:
        return (*_expr_deps(self.index), *self.values)


@dataclass(frozen=True)
class Assign(Stmt):
    name: str
    op: ElementwiseImpl
    args: tuple[str, ...]
    dtype: DataType | None = None

    def defines(self) -> tuple[str, ...]:
        return (self.name,)

    def deps(self) -> tuple[str, ...]:
        return tuple(self.args)


@dataclass(frozen=True)
class Accum(Stmt):
    name: str
    value: str
    op: ElementwiseImpl
    dtype: DataType | None = None
    axes: tuple[str, ...] = ()
    base: str | None = None

    def defines(self) -> tuple[str, ...]:
        return (self.name,)

    def deps(self) -> tuple[str, ...]:
        return (self.name, self.value) + ((self.base,) if self.base else ())


@dataclass(frozen=True)
class Init(Stmt):
    name: str
    identity: float | None
    dtype: DataType

    def defines(self) -> tuple[str, ...]:
        return (self.name,)


@dataclass(frozen=True)
class Let(Stmt):
    name: str
    value: Expr
    dtype: DataType | None = None

    def defines(self) -> tuple[str, ...]:
        return (self.name,)

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps(self.value))


@dataclass(frozen=True)
class Select(Stmt):
    name: str
    cond: Expr
    if_true: Expr
    if_false: Expr

    def defines(self) -> tuple[str, ...]:
        return (self.name,)

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps((self.cond, self.if_true, self.if_false)))


@dataclass(frozen=True)
class Cond(Stmt):
    cond: Expr
    body: tuple[Stmt, ...]
    else_body: tuple[Stmt, ...] = ()

    def nested(self) -> list[tuple[Stmt, ...]]:
        return [self.body, self.else_body]

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps(self.cond))


@dataclass(frozen=True)
class Sync(Stmt):
    barrier_id: int = 0
    count: int | None = None
    warp: bool = False


@dataclass(frozen=True)
class Smem(Stmt):
    name: str
    extents: tuple[int, ...]
    dtype: str
    align: int = 0


@dataclass(frozen=True)
class WarpShuffle(Stmt):
    state: tuple[str, ...]
    state_b: tuple[str, ...]
    combine_states: tuple[Assign, ...]
    length: int
    dtype: DataType

    def defines(self) -> tuple[str, ...]:
        return tuple(self.state)

    def deps(self) -> tuple[str, ...]:
        return tuple(self.state)


@dataclass(frozen=True)
class TreeHalve(Stmt):
    bufs: tuple[str, ...]
    state: tuple[str, ...]
    state_b: tuple[str, ...]
    combine_states: tuple[Assign, ...]
    length: int
    tid_var: str
    dtype: DataType
    barrier_id: int = 0
    barrier_count: int | None = None
    inner: tuple[str, int] | None = None

    def defines(self) -> tuple[str, ...]:
        return tuple(self.state)

    def deps(self) -> tuple[str, ...]:
        return (*self.state, self.tid_var) + ((self.inner[0],) if self.inner else ())


@dataclass(frozen=True)
class CpAsyncCopy(Stmt):
    smem: str
    smem_index: tuple[Expr, ...]
    src: str
    src_index: tuple[Expr, ...]
    nbytes: int
    swizzle: str = "NONE"
    lane_index: tuple[Expr, ...] | None = None
    lane_rows: int | None = None

    def deps(self) -> tuple[str, ...]:
        return tuple(_expr_deps((self.smem_index, self.src_index, self.lane_index or ())))


@dataclass(frozen=True)
class CpAsyncCommit(Stmt):
    pass


@dataclass(frozen=True)
class CpAsyncWait(Stmt):
    group: int = 0


# --- parsing -------------------------------------------------------------------------------

_CLASSES: dict[str, type] = {
    c.__name__: c
    for c in (Dim, DataType, ElementwiseImpl, Var, Literal, BinaryExpr, TernaryExpr,
              FuncCallExpr, CastExpr, Window, Axis, Tile, Loop, StridedLoop, Load, Write,
              Assign, Accum, Init, Let, Select, Cond, Sync, Smem, WarpShuffle, TreeHalve,
              CpAsyncCopy, CpAsyncCommit, CpAsyncWait)
}


class IRError(ValueError):
    """A Kernel IR string this loader cannot read."""


def _node(n: ast.AST) -> Any:
    if isinstance(n, ast.Constant):
        return n.value
    if isinstance(n, ast.Tuple | ast.List):
        return tuple(_node(e) for e in n.elts)
    if isinstance(n, ast.UnaryOp) and isinstance(n.op, ast.USub):
        return -_node(n.operand)
    if isinstance(n, ast.Name):
        if n.id in ("inf", "nan"):
            return float(n.id)
        raise IRError(f"unknown name {n.id!r} in Kernel IR")
    if isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "math":
        return float(n.attr)
    if isinstance(n, ast.Call) and isinstance(n.func, ast.Name):
        name = n.func.id
        args = [_node(a) for a in n.args]
        kwargs = {k.arg: _node(k.value) for k in n.keywords}
        if name == "dtype":
            return NpDtype(*args)
        if name == "float":
            return float(args[0])
        cls = _CLASSES.get(name)
        if cls is None:
            raise NotImplementedError(f"Kernel IR node {name} is not supported")
        known = {f.name for f in fields(cls)}
        extra = set(kwargs) - known
        if extra:  # a newer Emmy field: keep the node, drop nothing silently
            raise NotImplementedError(f"Kernel IR node {name}: unknown field(s) {sorted(extra)}")
        return cls(*args, **kwargs)
    raise IRError(f"cannot read Kernel IR expression {ast.dump(n)[:80]}")


def parse_body(text: str) -> Tile:
    """The Tile a KernelOp body string describes."""
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as e:
        raise IRError(f"Kernel IR body is not a repr string: {e}") from None
    tile = _node(tree.body)
    if not isinstance(tile, Tile):
        raise IRError(f"Kernel IR body is a {type(tile).__name__}, not a Tile")
    return tile


def walk(body: Sequence[Stmt]) -> Iterator[Stmt]:
    """Every statement in ``body``, nested ones included, in program order."""
    for st in body:
        yield st
        for inner in st.nested():
            yield from walk(inner)


# --- graphs --------------------------------------------------------------------------------


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple[int, ...]
    dtype: str


@dataclass
class KernelOp:
    """A kernel node of the graph: its entry name, body and outputs."""

    name: str
    body: Tile
    outputs: tuple[str, ...]
    fields_: dict[str, Any] = field(default_factory=dict)

    @property
    def smem_buffers(self) -> dict[str, Smem]:
        """Every Smem the body declares, by name, in program order."""
        out: dict[str, Smem] = {}
        for st in walk([self.body]):
            if isinstance(st, Smem) and st.name not in out:
                out[st.name] = st
        return out


@dataclass
class Graph:
    """An Emmy graph as ``<kernel>.ir.json`` stores it."""

    inputs: list[str]
    outputs: list[str]
    nodes: dict[str, dict[str, Any]]

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> Graph:
        for key in ("inputs", "outputs", "nodes"):
            if key not in d:
                raise IRError(f"graph JSON has no {key!r}")
        return cls(list(d["inputs"]), list(d["outputs"]), dict(d["nodes"]))

    @classmethod
    def load(cls, path: str | Path) -> Graph:
        return cls.from_dict(json.loads(Path(path).read_text()))

    @classmethod
    def from_emmy(cls, g: Any) -> Graph:
        """A live Emmy graph -- the object the reference's ``to_ptx`` receives (reference
        ``compile.py:24-33``: ``graph.nodes`` maps node ids to nodes whose ``op`` is an Emmy op)
        -- in the JSON form this loader reads. A KernelOp's body becomes the ``repr`` strings of
        its statements, which is what Emmy's JSON holds; other nodes keep their op's class name.
        Uses only ``repr``, class names and the ``name``/``body``/``outputs`` attributes, so it
        needs no Emmy import."""
        def names(ts: Any) -> list[dict[str, Any]]:
            out = []
            for t in ts or ():
                shape = getattr(t, "shape", None)
                out.append({"name": getattr(t, "name", str(t)),
                            "shape": list(shape) if shape is not None else [],
                            "dtype": str(getattr(getattr(t, "dtype", None), "name",
                                                 getattr(t, "dtype", "")))})
            return out

        nodes: dict[str, dict[str, Any]] = {}
        for nid, n in dict(g.nodes).items():
            op = getattr(n, "op", n)
            kind = type(op).__name__
            fields: dict[str, Any] = {}
            if kind == "KernelOp":
                body = op.body
                stmts = list(body) if isinstance(body, list | tuple) else [body]
                fields = {"body": [repr(st) for st in stmts],
                          "name": getattr(op, "name", None) or nid}
            nodes[str(nid)] = {"op": kind, "op_fields": fields,
                               "inputs": [str(i) for i in getattr(n, "inputs", None) or ()],
                               "outputs": names(getattr(n, "outputs", None))}
        return cls([str(i) for i in getattr(g, "inputs", None) or ()],
                   [str(o) for o in getattr(g, "outputs", None) or ()], nodes)

    def kernel_ops(self) -> list[KernelOp]:
        out = []
        for node_id, n in self.nodes.items():
            if n.get("op") != "KernelOp":
                continue
            f = n["op_fields"]
            body = f["body"]
            text = body[0] if isinstance(body, list) else body
            outs = tuple(t["name"] for t in n.get("outputs", ())) or (node_id,)
            out.append(KernelOp(f.get("name") or node_id, parse_body(text), outs, dict(f)))
        return out

    def tensors(self) -> dict[str, TensorSpec]:
        out = {}
        for n in self.nodes.values():
            for t in n.get("outputs", ()):
                out[t["name"]] = TensorSpec(t["name"], tuple(t["shape"] or ()), t["dtype"])
        return out

    def to_dict(self) -> dict[str, Any]:
        return {"inputs": self.inputs, "outputs": self.outputs, "nodes": self.nodes}


def kernel_node(name: str, body: Tile, inputs: Sequence[str], outputs: Sequence[TensorSpec]
                ) -> dict[str, Any]:
    """A KernelOp graph node in Emmy's JSON layout."""
    return {
        "op": "KernelOp",
        "op_fields": {"body": [repr(body)], "name": name, "zero_delegated": [], "serial": []},
        "inputs": list(inputs),
        "outputs": [{"name": t.name, "shape": list(t.shape), "dtype": t.dtype} for t in outputs],
    }


def input_node(t: TensorSpec) -> dict[str, Any]:
    return {"op": "InputOp", "op_fields": {}, "inputs": [],
            "outputs": [{"name": t.name, "shape": list(t.shape), "dtype": t.dtype}]}


def constant_node(name: str, value: float, dtype: str = "f32") -> dict[str, Any]:
    return {
        "op": "ConstantOp",
        "op_fields": {"name": name, "value": value, "context_value": None, "load_ops": [],
                      "source_path": None, "source_parts": [], "source_shape": None,
                      "source_dtype": None, "source_graph": None},
        "inputs": [],
        "outputs": [{"name": name, "shape": [1], "dtype": dtype}],
    }

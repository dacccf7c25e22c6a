"""Usage-derived stand-in for the external ``ml_switcheroo_ir`` package (v0.0.6).

TEST INFRASTRUCTURE ONLY. The reference pins ``ml_switcheroo_ir`` as a wheel URL
(``requirements.txt:1``) that is neither vendored nor installable offline. This module
is NOT the upstream source: it is written from how the reference *uses* the package
(``ir/core.py:8-48``, ``core/dtype.py:10``, ``ir/shape_system.py:10-24``,
``interpreter/evaluator.py:11``), with just enough surface for
``import ml_switcheroo_compiler`` and for tracing, AD and ``evaluate_graph``.
It is put on ``sys.path`` only by the golden-fixture generator under ``tests/golden``.
"""

from __future__ import annotations

import typing

from pydantic import BaseModel, ConfigDict, Field

from ml_switcheroo_ir.types import DType, TensorSpec

AttributeValue = typing.Any


class NodeDict(dict):
    """Ordered id -> node mapping (a plain dict keeps insertion order)."""


class PartitionSpec(BaseModel):
    """Sharding spec: one mesh-axis name (or None) per tensor dim."""

    model_config = ConfigDict(extra="allow", arbitrary_types_allowed=True)
    axes: tuple = ()


class LogicalNode(BaseModel):
    """One graph node: an op with named inputs, attributes and inferred shape."""

    model_config = ConfigDict(extra="allow", arbitrary_types_allowed=True)
    id: str
    op_type: str
    domain: str = "ai.onnx"
    inputs: list[str] = Field(default_factory=list)
    outputs: list[str] = Field(default_factory=list)
    attributes: dict[str, typing.Any] = Field(default_factory=dict)
    shape_metadata: typing.Any = None
    output_specs: list[typing.Any] = Field(default_factory=list)
    source_ast_ref: typing.Any = None
    sharding: typing.Any = None
    device: typing.Any = None
    stream: typing.Any = None
    subgraphs: dict[str, typing.Any] = Field(default_factory=dict)


class LogicalGraph(BaseModel):
    """A dataflow graph: id -> node, named graph inputs/outputs and initializers."""

    model_config = ConfigDict(extra="allow", arbitrary_types_allowed=True)
    name: str = "graph"
    nodes: dict[str, LogicalNode] = Field(default_factory=NodeDict)
    inputs: list[str] = Field(default_factory=list)
    outputs: list[str] = Field(default_factory=list)
    initializers: dict[str, typing.Any] = Field(default_factory=dict)
    input_specs: dict[str, typing.Any] = Field(default_factory=dict)


class _Tangent:
    def __repr__(self) -> str:
        return type(self).__name__


class ZeroTangent(_Tangent):
    """Marker for a structurally-zero tangent."""


class NoTangent(_Tangent):
    """Marker for a non-differentiable value."""


class TensorShape(tuple):
    """Plain tuple of dims."""


class Polynomial:
    """Integer-coefficient multivariate polynomial holder (subclassed by the reference)."""

    def __init__(self, terms=None) -> None:
        self.terms = {k: v for k, v in (terms or {}).items() if v != 0}


class SymNode:
    """Base of symbolic expression nodes."""


class SymBinaryOp(SymNode):
    """Base of binary symbolic nodes."""


class SymUnaryOp(SymNode):
    """Base of unary symbolic nodes."""


class SymInt:
    """Base of symbolic integers."""


def topological_sort(graph: LogicalGraph) -> list[LogicalNode]:
    """Dependency order (inputs before users); insertion order breaks ties."""
    order: list[LogicalNode] = []
    seen: set[str] = set()
    nodes = graph.nodes

    def visit(nid: str) -> None:
        stack = [(nid, False)]
        while stack:
            cur, done = stack.pop()
            if done:
                if cur not in seen:
                    seen.add(cur)
                    order.append(nodes[cur])
                continue
            if cur in seen or cur not in nodes:
                continue
            stack.append((cur, True))
            for dep in reversed(nodes[cur].inputs):
                if dep in nodes and dep not in seen:
                    stack.append((dep, False))

    for nid in list(nodes):
        visit(nid)
    return order

"""Host-side mirror of the reference IR (``LogicalGraph`` / ``LogicalNode``).

The backend accepts either the reference's pydantic objects (duck-typed: ``nodes``
mapping or sequence, ``inputs``, ``outputs``, ``initializers``; per node ``id``,
``op_type``, ``inputs``, ``attributes``, ``shape_metadata``) or the JSON form written
by ``tests/golden/make_golden.py``. Only what execution needs is kept.
"""

from __future__ import annotations

import gzip
import json
import os
from dataclasses import dataclass, field
from typing import Any

from .errors import CompilationError

GRAPH_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "tests", "golden", "graphs")


@dataclass
class Node:
    id: str
    op_type: str
    inputs: list[str]
    attributes: dict[str, Any] = field(default_factory=dict)
    shape_metadata: tuple | None = None
    const_dtype: str | None = None


@dataclass
class Graph:
    name: str
    nodes: dict[str, Node]
    inputs: list[str]
    outputs: list[str]
    initializers: dict[str, Any] = field(default_factory=dict)
    roles: dict[str, str] = field(default_factory=dict)  # role -> input id (workload graphs)
    output_names: dict[str, str] = field(default_factory=dict)  # name -> output id
    meta: dict[str, Any] = field(default_factory=dict)

    def topo_order(self) -> list[Node]:
        """Dependency order over all nodes; raises CompilationError on a cycle
        (``core/utils/graph_utils.py:29-100``)."""
        order: list[Node] = []
        state: dict[str, int] = {}
        for root in self.nodes:
            if root in state:
                continue
            stack = [(root, 0)]
            while stack:
                nid, i = stack.pop()
                if i == 0:
                    if state.get(nid) == 2:
                        continue
                    state[nid] = 1
                deps = [d for d in self.nodes[nid].inputs if d in self.nodes]
                if i < len(deps):
                    stack.append((nid, i + 1))
                    d = deps[i]
                    if state.get(d) == 1:
                        raise CompilationError(f"cycle in graph {self.name!r} at node {d!r}")
                    if d not in state:
                        stack.append((d, 0))
                else:
                    state[nid] = 2
                    order.append(self.nodes[nid])
        return order


def from_json(doc: dict) -> Graph:
    nodes = {}
    for n in doc["nodes"]:
        sm = n.get("shape_metadata")
        nodes[n["id"]] = Node(n["id"], n["op_type"], list(n["inputs"]), dict(n.get("attributes") or {}),
                              tuple(sm) if sm is not None else None, n.get("const_dtype"))
    return Graph(doc.get("name", "graph"), nodes, list(doc["inputs"]), list(doc["outputs"]), {},
                 dict(doc.get("roles", {})), dict(doc.get("output_names", {})),
                 {k: doc[k] for k in ("workload", "dims") if k in doc})


def load(name_or_path: str) -> Graph:
    """Load a stored workload graph by case name (``tests/golden/graphs``) or path."""
    path = name_or_path if os.path.exists(name_or_path) else os.path.join(GRAPH_DIR, name_or_path + ".json.gz")
    with gzip.open(path, "rt", encoding="utf-8") as f:
        return from_json(json.load(f))


def coerce(graph: Any) -> Graph:
    """Accept our Graph, a JSON dict, or a reference LogicalGraph (duck-typed)."""
    if isinstance(graph, Graph):
        return graph
    if isinstance(graph, dict):
        return from_json(graph)
    raw = graph.nodes
    seq = list(raw.values()) if hasattr(raw, "values") else list(raw)
    nodes = {}
    for n in seq:
        sm = getattr(n, "shape_metadata", None)
        attrs = dict(getattr(n, "attributes", None) or {})
        cd = None
        if n.op_type == "Constant":
            import numpy as np

            cd = str(np.asarray(attrs.get("value")).dtype)
        nodes[n.id] = Node(n.id, n.op_type, list(n.inputs), attrs, tuple(sm) if sm is not None else None, cd)
    outs = graph.outputs if isinstance(graph.outputs, list) else [graph.outputs]
    return Graph(getattr(graph, "name", "graph"), nodes, list(graph.inputs), list(outs),
                 dict(getattr(graph, "initializers", None) or {}))

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
    subgraphs: dict[str, Any] = field(default_factory=dict)


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


def _canon(v: Any) -> Any:
    """A deterministic, hashable form of an attribute value (arrays by dtype, shape, bytes)."""
    if isinstance(v, dict):
        return ("d", tuple(sorted((str(k), _canon(x)) for k, x in v.items())))
    if isinstance(v, (list, tuple)):
        return ("l", tuple(_canon(x) for x in v))
    if hasattr(v, "tobytes") and hasattr(v, "dtype") and hasattr(v, "shape"):
        return ("a", str(v.dtype), tuple(v.shape), v.tobytes())
    if isinstance(v, (str, int, float, bool)) or v is None:
        return (type(v).__name__, v)
    if hasattr(v, "model_dump"):  # pydantic attribute / subgraph objects
        return ("m", type(v).__name__, _canon(v.model_dump()))
    return ("r", type(v).__name__, repr(v))


def content_key(g: Graph) -> str:
    """Digest of everything execution depends on: every node's id, op type, inputs,
    attributes and shape metadata, and the graph's inputs, outputs and initializer names.
    Two graphs with the same key run the same plan."""
    import hashlib

    h = hashlib.sha256()
    h.update(repr((tuple(g.inputs), tuple(g.outputs), tuple(sorted(g.initializers)))).encode())
    for nid in sorted(g.nodes):
        n = g.nodes[nid]
        h.update(repr((n.id, n.op_type, tuple(n.inputs), _canon(n.attributes), n.shape_metadata, n.const_dtype,
                       _canon(n.subgraphs))).encode())
    for k in sorted(g.initializers):
        h.update(repr(_canon(g.initializers[k])).encode())
    return h.hexdigest()


def from_json(doc: dict) -> Graph:
    nodes = {}
    for n in doc["nodes"]:
        sm = n.get("shape_metadata")
        nodes[n["id"]] = Node(n["id"], n["op_type"], list(n["inputs"]), dict(n.get("attributes") or {}),
                              tuple(sm) if sm is not None else None, n.get("const_dtype"), dict(n.get("subgraphs") or {}))
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
        subs = getattr(n, "subgraphs", None)
        nodes[n.id] = Node(n.id, n.op_type, list(n.inputs), attrs, tuple(sm) if sm is not None else None, cd,
                           dict(subs) if isinstance(subs, dict) else {})
    outs = graph.outputs if isinstance(graph.outputs, list) else [graph.outputs]
    return Graph(getattr(graph, "name", "graph"), nodes, list(graph.inputs), list(outs),
                 dict(getattr(graph, "initializers", None) or {}))

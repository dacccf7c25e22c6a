"""Fixtures for the drop-in boundary, recorded from the REFERENCE's own callers.

Test infrastructure: imports the reference (``ml_switcheroo_compiler``) read-only from the
source tree named by ``--reference-src`` or ``$ML_SWITCHEROO_REFERENCE_SRC``, with the
``ml_switcheroo_ir`` stand-in under ``oracle/standin``, and the ``b200`` package itself
(importing it needs no GPU). The reference cannot be installed where the GPUs are (its
build backend is not available offline), so its side of the boundary is recorded here
and replayed there against ``B200Backend``:

1. ``protocols.json``: ``b200.register()`` through the reference's
   ``register_backend`` (``backends/registry.py:426-448``), ``BackendRegistry.get("b200")``
   returning ``B200Backend``, and the reference's structural checks that route a whole
   graph to it (``grad/api.py:85-106``, ``grad/jvp_vjp.py:205-226``).
2. ``pernode_<case>``: every call the reference's ``evaluate_graph``
   (``interpreter/evaluator.py:272-305``) makes on its backend while it interprets a graph:
   ``execute_op`` (``:593``, and Clone for IndexPut ``:506``), ``array`` (Constant
   ``:761``) and ``asarray`` (Slice / GetItem ``:444,484``), with their arguments and the
   reference numpy backend's result of each. The recording backend is a subclass of
   ``B200Backend`` that forwards each call to the reference numpy backend.
3. ``graph_<case>``: the fwd+bwd ``LogicalGraph`` and input dict the reference's
   ``vjp`` pullback hands to ``backend.execute_graph`` (``grad/jvp_vjp.py:511-529``, via
   ``_execute_autodiff_graph``), pydantic-dumped, with the numpy result of that graph.

Usage: ``python tests/golden/make_boundary_golden.py --reference-src PATH``.
"""

from __future__ import annotations

import gzip
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "boundary")
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(REPO, "ml-switcheroo-compiler_b200"))
from refpath import add_reference_to_path  # noqa: E402

add_reference_to_path()

import b200  # noqa: E402
from b200.backend import B200Backend  # noqa: E402
from make_golden import D, _jsonable, register_corrected_rules  # noqa: E402
from ml_switcheroo_compiler.backends.registry import BackendRegistry  # noqa: E402
from ml_switcheroo_compiler.core.config import config  # noqa: E402
from ml_switcheroo_compiler.grad import api as grad_api  # noqa: E402
from ml_switcheroo_compiler.grad import jvp_vjp  # noqa: E402
from ml_switcheroo_compiler.interpreter.evaluator import evaluate_graph  # noqa: E402
from ml_switcheroo_ir import LogicalGraph, LogicalNode  # noqa: E402


def numpy_backend():
    return BackendRegistry.get("numpy")


class Values:
    """Numbers every array that crosses the boundary; identical objects share a key."""

    def __init__(self) -> None:
        self.arrays: dict[str, np.ndarray] = {}
        self.by_id: dict[int, str] = {}
        self.keep: list = []

    def ref(self, v):
        if isinstance(v, np.ndarray) or isinstance(v, np.generic):
            key = self.by_id.get(id(v))
            if key is None:
                key = f"v{len(self.arrays)}"
                self.arrays[key] = np.asarray(v).copy()
                self.by_id[id(v)] = key
                self.keep.append(v)
            return {"value": key}
        if isinstance(v, (list, tuple)):
            return {"seq": [self.ref(u) for u in v], "tuple": isinstance(v, tuple)}
        return {"lit": _jsonable(v)}


class Recorder(B200Backend):
    """B200Backend as the reference sees it, with every call forwarded to the reference
    numpy backend (no GPU here) and written down."""

    name = "b200"
    values: Values | None = None
    calls: list = []
    graphs: list = []

    @classmethod
    def _rec(cls, method, args, kwargs, out):
        cls.calls.append({"method": method, "args": [cls.values.ref(a) for a in args],
                          "kwargs": {k: cls.values.ref(v) for k, v in kwargs.items()}, "out": cls.values.ref(out)})
        return out

    @classmethod
    def execute_op(cls, op_type, *args, **kwargs):
        out = numpy_backend().execute_op(op_type, *args, **kwargs)
        return cls._rec("execute_op", [op_type, *args], kwargs, out)

    @classmethod
    def array(cls, data, dtype=None):
        out = numpy_backend().array(data) if dtype is None else numpy_backend().array(data, dtype)
        return cls._rec("array", [data], {} if dtype is None else {"dtype": str(dtype)}, out)

    @classmethod
    def asarray(cls, data):
        out = numpy_backend().asarray(data)
        return cls._rec("asarray", [data], {}, out)

    @classmethod
    def execute_graph(cls, graph, inputs):
        res = evaluate_graph(graph, dict(inputs), backend=numpy_backend())
        cls.graphs.append((graph.model_dump(), {k: np.asarray(v) for k, v in inputs.items()}, dict(res)))
        return res


def lg_from_json(case: str) -> tuple[LogicalGraph, dict]:
    """A stored workload graph as the reference's LogicalGraph, and its golden inputs."""
    with gzip.open(os.path.join(HERE, "graphs", case + ".json.gz"), "rt") as f:
        doc = json.load(f)
    g = LogicalGraph(name=doc.get("name", case))
    for n in doc["nodes"]:
        attrs = dict(n.get("attributes") or {})
        if n["op_type"] == "Constant" and n.get("const_dtype"):
            attrs["value"] = np.array(attrs["value"], dtype=n["const_dtype"])
        if n["op_type"] == "Checkpoint" and isinstance(attrs.get("subgraph"), dict):
            sg = attrs["subgraph"]
            sub = LogicalGraph(name=sg.get("name", "sub"))
            for m in sg["nodes"]:
                sub.nodes[m["id"]] = LogicalNode(id=m["id"], op_type=m["op_type"], inputs=list(m["inputs"]),
                                                 attributes=dict(m.get("attributes") or {}), shape_metadata=m.get("shape_metadata"))
            sub.inputs, sub.outputs = list(sg["inputs"]), list(sg["outputs"])
            attrs["subgraph"] = sub
        g.nodes[n["id"]] = LogicalNode(id=n["id"], op_type=n["op_type"], inputs=list(n["inputs"]), attributes=attrs,
                                       shape_metadata=n.get("shape_metadata"))
    g.inputs, g.outputs = list(doc["inputs"]), list(doc["outputs"])
    d = np.load(os.path.join(HERE, case + ".npz"))
    ins = {k[4:]: d[k] for k in d.files if k.startswith("in__")}
    return g, {nid: ins[r] for r, nid in doc["roles"].items()}


def save_pernode(case: str) -> None:
    g, inputs = lg_from_json(case)
    Recorder.values, Recorder.calls = Values(), []
    inputs = {k: np.ascontiguousarray(v) for k, v in inputs.items()}
    in_refs = {k: Recorder.values.ref(v) for k, v in inputs.items()}
    res = evaluate_graph(g, inputs, backend=Recorder)
    out_refs = {k: Recorder.values.ref(np.asarray(v)) if not isinstance(v, np.ndarray) else Recorder.values.ref(v)
                for k, v in res.items()}
    doc = {"case": case, "inputs": in_refs, "outputs": out_refs, "calls": Recorder.calls}
    with gzip.open(os.path.join(OUT, f"pernode_{case}.json.gz"), "wt") as f:
        json.dump(doc, f)
    np.savez_compressed(os.path.join(OUT, f"pernode_{case}.npz"), **Recorder.values.arrays)
    print("pernode", case, len(Recorder.calls), "calls", sorted({c["args"][0]["lit"] for c in Recorder.calls
                                                                 if c["method"] == "execute_op"}))


def fwd_mlp(x, W1, b1, W2, b2, labels):
    """The MLP workload's forward with canonical op names (the reference's eager dispatch
    does not apply the interpreter's aliases, so ``Neg`` would not evaluate eagerly)."""
    h = D("Relu", D("Add", D("Matmul", x, W1), b1))
    lg = D("Add", D("Matmul", h, W2), b2)
    ls = D("LogSoftmax", lg, axis=-1)
    picked = D("TakeAlongAxis", ls, labels, axis=-1)
    return D("ReduceMean", D("Negative", picked))


def save_vjp_graph() -> None:
    """The MLP workload's forward traced by the reference, pulled back through its ``vjp``:
    the pullback calls ``execute_graph`` on the active backend (the recorder)."""
    rng = np.random.default_rng(11)
    f32 = np.float32
    B, D, H, C = 16, 48, 32, 10
    x = rng.standard_normal((B, D), dtype=f32)
    W1 = (rng.uniform(-1, 1, (D, H)) * np.sqrt(6.0 / D)).astype(f32)
    b1 = (rng.standard_normal(H) * 0.1).astype(f32)
    W2 = (rng.uniform(-1, 1, (H, C)) * np.sqrt(6.0 / H)).astype(f32)
    b2 = (rng.standard_normal(C) * 0.1).astype(f32)
    labels = rng.integers(0, C, (B, 1), dtype=np.int64)
    Recorder.graphs = []
    _, pullback = jvp_vjp.vjp(fwd_mlp, x, W1, b1, W2, b2, labels)
    pullback(np.array(1.0, f32))
    assert Recorder.graphs, "the pullback did not reach execute_graph"
    for i, (dump, inputs, res) in enumerate(Recorder.graphs):
        doc = {"graph": _jsonable(dump), "inputs": sorted(inputs), "outputs": list(dump["outputs"])}
        with gzip.open(os.path.join(OUT, f"graph_vjp_mlp{i}.json.gz"), "wt") as f:
            json.dump(doc, f)
        blob = {"in__" + k: v for k, v in inputs.items()}
        blob.update({"out__" + k: np.asarray(v) for k, v in res.items()})
        np.savez_compressed(os.path.join(OUT, f"graph_vjp_mlp{i}.npz"), **blob)
        print("graph", i, len(dump["nodes"]), "nodes", "outputs", len(dump["outputs"]))


def main() -> None:
    os.makedirs(OUT, exist_ok=True)
    register_corrected_rules()
    # 1. the real class through the reference's registry and protocol checks
    cls = b200.register()
    proto = {
        "registered": BackendRegistry.get("b200") is B200Backend and cls is B200Backend,
        "api_execute_graph": bool(grad_api._is_execute_graph_backend(B200Backend)),
        "api_compile_graph": bool(grad_api._is_compile_graph_backend(B200Backend)),
        "jvp_vjp_execute_graph": bool(jvp_vjp._is_execute_graph_backend(B200Backend)),
        "jvp_vjp_compile_graph": bool(jvp_vjp._is_compile_graph_backend(B200Backend)),
        "members": sorted(m for m in ("execute_op", "array", "asarray", "zeros", "item", "get_module", "execute_graph",
                                      "compile_graph") if callable(getattr(B200Backend, m, None))),
    }
    with open(os.path.join(OUT, "protocols.json"), "w") as f:
        json.dump(proto, f, indent=1, sort_keys=True)
    print("protocols", proto)
    # 2./3. the recorder in the backend's place
    from ml_switcheroo_compiler.backends.registry import register_backend

    register_backend("b200")(Recorder)
    config.backend = "b200"
    for case in ("mlp_ragged", "rowfused_ragged", "nodes_indexing"):
        save_pernode(case)
    save_vjp_graph()
    config.backend = "numpy"


if __name__ == "__main__":
    main()

"""Golden fixtures for the node types outside the five workloads' graphs, made by the
REFERENCE itself.

Test infrastructure: imports the reference (``ml_switcheroo_compiler``) read-only from the
source tree named by ``--reference-src`` or ``$ML_SWITCHEROO_REFERENCE_SRC``, with the
``ml_switcheroo_ir`` stand-in under ``oracle/standin``. Each case is a small
``LogicalGraph`` built from the reference's IR classes with seeded inputs:

* ``nodes_fused_*``: a graph of plain ops, then rewritten by one of the reference's own
  fusion passes (``transforms/passes/operator_fusion.py``: ``fuse_elementwise_clusters``
  -> ``FusedElementwise``; ``fuse_elementwise_activation`` -> ``<Elem><Act>``;
  ``fuse_conv_bias_relu`` -> ``FusedConv2DBias<Act>``; ``fuse_horizontal_patterns`` ->
  ``HorizontalFusedOps`` + ``TupleGetItem``; ``operator_fusion_pass``, the full pass with
  the declarative and YAML rules). No reference backend evaluates the fused nodes, so the
  golden outputs are the reference numpy backend's ``evaluate_graph`` of the graph
  BEFORE fusion: a fusion must not change values. The stored graph is the fused one.
* ``nodes_indexing``: Slice (``slices`` string and dim / start / end / step), GetItem
  (negative step, integer list), IndexPut, Gather, OneHot, Recompute and a Checkpoint
  with a forward subgraph, evaluated directly by the reference's ``evaluate_graph``
  (``interpreter/evaluator.py:428-545, 720-769``) on the numpy backend.

Outputs: ``tests/golden/graphs/<case>.json.gz`` and ``tests/golden/<case>.npz`` (the same
layout as ``make_golden.py``). Usage:
``python tests/golden/make_node_golden.py --reference-src PATH``.
"""

from __future__ import annotations

import copy
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from refpath import add_reference_to_path  # noqa: E402

add_reference_to_path()

from ml_switcheroo_compiler.core.config import config  # noqa: E402
from ml_switcheroo_compiler.interpreter.evaluator import evaluate_graph  # noqa: E402
from ml_switcheroo_compiler.transforms.passes import operator_fusion as F  # noqa: E402
from ml_switcheroo_ir import LogicalGraph, LogicalNode  # noqa: E402

from make_golden import _jsonable, save_graph  # noqa: E402


def N(g, nid, op, inputs=(), shape=None, **attrs):
    g.nodes[nid] = LogicalNode(id=nid, op_type=op, inputs=list(inputs), attributes=dict(attrs),
                               shape_metadata=list(shape) if shape is not None else None)
    return nid


def new_graph(name, inputs):
    g = LogicalGraph(name=name)
    for nid, shape in inputs.items():
        N(g, nid, "Input", (), shape)
    g.inputs = list(inputs)
    return g


def node_json(n):
    d = {"id": n.id, "op_type": n.op_type, "inputs": list(n.inputs),
         "attributes": {k: (graph_json(v) if isinstance(v, LogicalGraph) else _jsonable(v))
                        for k, v in dict(n.attributes or {}).items() if k != "fun"},
         "shape_metadata": _jsonable(list(n.shape_metadata)) if n.shape_metadata is not None else None}
    if n.op_type == "Constant":
        d["const_dtype"] = str(np.asarray(n.attributes["value"]).dtype)
    return d


def graph_json(g):
    return {"name": g.name, "inputs": list(g.inputs), "outputs": list(g.outputs), "nodes": [node_json(n) for n in g.nodes.values()]}


def export(g, case, arrays, golden):
    doc = graph_json(g)
    doc.update({"format": "logical-graph-json/1", "workload": "nodes", "dims": {},
                "roles": {nid: nid for nid in g.inputs}, "output_names": {o: o for o in g.outputs}})
    save_graph(doc, os.path.join(HERE, "graphs", case + ".json.gz"))
    blob = {"in__" + k: np.asarray(v) for k, v in arrays.items()}
    for o in g.outputs:
        blob["out__" + o] = np.asarray(golden[o])
    np.savez_compressed(os.path.join(HERE, case + ".npz"), **blob)
    ops = sorted({n.op_type for n in g.nodes.values()})
    print(case, ops, {k: (v.shape, str(v.dtype)) for k, v in blob.items() if k.startswith("out__")})


def fused_case(case, g, arrays, fuse):
    ref = evaluate_graph(g, dict(arrays))  # the unfused graph on the reference numpy backend
    fg = copy.deepcopy(g)
    changed = fuse(fg)
    assert changed, f"{case}: the fusion pass changed nothing"
    # a rewrite may rename an output node (declarative rules append "_fused"): outputs
    # correspond by position
    assert len(fg.outputs) == len(g.outputs)
    export(fg, case, arrays, {fo: ref[o] for fo, o in zip(fg.outputs, g.outputs)})


def main() -> None:
    config.backend = "numpy"
    rng = np.random.default_rng(7)
    f32 = np.float32
    R, C = 64, 96

    # --- elementwise clusters -> FusedElementwise (scalar_expr) --------------------
    # Every intermediate has one consumer: on a DAG with shared intermediates the
    # reference's cluster pass writes a scalar_expr that names inputs the node does not
    # have (its in_k renumbering is a plain string replace), so only chains give a node
    # whose expression equals the graph it replaced.
    g = new_graph("fused_ew", {"x": [R, C], "a": [C], "b": [C], "y": [R, C], "c": [R, 1], "z": [C], "w": [R, C]})
    N(g, "m", "Mul", ["x", "a"], [R, C])
    N(g, "s", "Add", ["m", "b"], [R, C])
    N(g, "ge", "Gelu", ["s"], [R, C])
    N(g, "t", "Tanh", ["ge"], [R, C])
    N(g, "e", "Exp", ["t"], [R, C])
    N(g, "d", "Div", ["e", "y"], [R, C])
    N(g, "q", "Sub", ["d", "c"], [R, C])
    N(g, "n", "Neg", ["q"], [R, C])
    N(g, "r", "Relu", ["n"], [R, C])
    N(g, "mx", "Maximum", ["r", "z"], [R, C])
    N(g, "ab", "Abs", ["mx"], [R, C])
    N(g, "sq", "Sqrt", ["ab"], [R, C])
    N(g, "mn", "Minimum", ["sq", "w"], [R, C])
    g.outputs = ["mn"]
    arrays = {"x": rng.standard_normal((R, C)).astype(f32), "a": rng.uniform(0.5, 1.5, C).astype(f32),
              "b": (rng.standard_normal(C) * 0.1).astype(f32), "y": rng.uniform(0.5, 2.0, (R, C)).astype(f32),
              "c": rng.uniform(0.5, 3.0, (R, 1)).astype(f32), "z": (rng.standard_normal(C) * 0.2).astype(f32),
              "w": rng.uniform(0.0, 1.5, (R, C)).astype(f32)}
    fused_case("nodes_fused_ew", g, arrays, F.fuse_elementwise_clusters)

    # --- elementwise + activation -> <Elem><Act> -----------------------------------
    g = new_graph("fused_act", {"x": [R, C], "y": [R, C], "b": [C]})
    N(g, "s", "Add", ["x", "b"], [R, C])
    N(g, "r", "Relu", ["s"], [R, C])
    N(g, "m", "Mul", ["x", "y"], [R, C])
    N(g, "g2", "Gelu", ["m"], [R, C])
    N(g, "d", "Sub", ["y", "x"], [R, C])
    N(g, "t", "Tanh", ["d"], [R, C])
    N(g, "o", "Add", ["r", "g2"], [R, C])
    N(g, "o2", "Add", ["o", "t"], [R, C])
    g.outputs = ["o2"]
    arrays = {"x": rng.standard_normal((R, C)).astype(f32), "y": rng.standard_normal((R, C)).astype(f32),
              "b": (rng.standard_normal(C) * 0.5).astype(f32)}
    fused_case("nodes_fused_act", g, arrays, F.fuse_elementwise_activation)

    # --- conv + bias + activation -> FusedConv2DBiasRelu ----------------------------
    g = new_graph("fused_conv", {"X": [4, 3, 12, 12], "W": [8, 3, 3, 3], "bias": [8, 1, 1]})
    N(g, "c", "Conv2D", ["X", "W"], [4, 8, 12, 12], stride=[1, 1], padding="SAME")
    N(g, "cb", "Add", ["c", "bias"], [4, 8, 12, 12])
    N(g, "cr", "Relu", ["cb"], [4, 8, 12, 12])
    g.outputs = ["cr"]
    arrays = {"X": rng.standard_normal((4, 3, 12, 12)).astype(f32), "W": (rng.standard_normal((8, 3, 3, 3)) * 0.3).astype(f32),
              "bias": (rng.standard_normal((8, 1, 1)) * 0.1).astype(f32)}
    fused_case("nodes_fused_conv", g, arrays, F.fuse_conv_bias_relu)

    # --- siblings on the same inputs -> HorizontalFusedOps + TupleGetItem -------------
    g = new_graph("fused_horizontal", {"x": [R, C]})
    N(g, "e", "Exp", ["x"], [R, C])
    N(g, "t", "Tanh", ["x"], [R, C])
    N(g, "s", "Sqrt", ["x"], [R, C])
    N(g, "o", "Add", ["e", "t"], [R, C])
    N(g, "o2", "Mul", ["o", "s"], [R, C])
    g.outputs = ["o2"]
    arrays = {"x": rng.uniform(0.1, 2.0, (R, C)).astype(f32)}
    fused_case("nodes_fused_horizontal", g, arrays, F.fuse_horizontal_patterns)

    # --- the whole pass (declarative + YAML rules, vertical, horizontal, clusters) ----
    g = new_graph("fused_full", {"x": [R, 128], "W": [128, C], "bias": [C], "y": [R, C]})
    N(g, "mm", "Matmul", ["x", "W"], [R, C])
    N(g, "ab", "Add", ["mm", "bias"], [R, C])
    N(g, "ge", "Gelu", ["ab"], [R, C])
    N(g, "m2", "Mul", ["ge", "y"], [R, C])
    N(g, "lg", "Log", ["y"], [R, C])
    N(g, "ex", "Exp", ["lg"], [R, C])
    N(g, "o", "Add", ["m2", "ex"], [R, C])
    g.outputs = ["o"]
    arrays = {"x": rng.standard_normal((R, 128)).astype(f32), "W": (rng.standard_normal((128, C)) * 0.1).astype(f32),
              "bias": (rng.standard_normal(C) * 0.1).astype(f32), "y": rng.uniform(0.5, 2.0, (R, C)).astype(f32)}
    fused_case("nodes_fused_full", g, arrays, F.operator_fusion_pass)

    # --- interpreter indexing nodes, Gather, OneHot, Recompute, Checkpoint -------------
    g = new_graph("indexing", {"x": [6, 8, 10], "v": [3, 10], "idx": [6, 4], "lab": [5], "u": [6, 8]})
    N(g, "s1", "Slice", ["x"], None, slices="(slice(1, 5, None), slice(None, None, 2))")
    N(g, "s2", "Slice", ["x"], None, dim=2, start=2, end=9, step=3)
    N(g, "g1", "GetItem", ["x"], None, key="(Ellipsis, slice(None, None, -1))")
    N(g, "g2", "GetItem", ["x"], None, key="(slice(None), [0, 3, 3, -1])")
    N(g, "g3", "GetItem", ["x"], None, key="(2, None, slice(-3, None))")
    N(g, "p1", "IndexPut", ["x", "v"], None, key="(1, slice(2, 5))")
    N(g, "ga", "Gather", ["u", "one", "idx"], None)
    N(g, "one", "Constant", [], None, value=1)
    N(g, "oh", "OneHot", ["lab", "depth"], None, dtype="float32", on_value=2.0, off_value=-0.5)
    N(g, "depth", "Constant", [], None, value=7)
    N(g, "rc", "Recompute", ["u", "u"], None, original_op="Mul", original_attrs={})
    sub = new_graph("ckpt_body", {"cin": [6, 8]})
    N(sub, "ct", "Tanh", ["cin"], [6, 8])
    N(sub, "cm", "Mul", ["ct", "cin"], [6, 8])
    sub.outputs = ["cm"]
    N(g, "ck", "Checkpoint", ["u"], [6, 8], subgraph=sub, evicted=True)
    g.outputs = ["s1", "s2", "g1", "g2", "g3", "p1", "ga", "oh", "rc", "ck"]
    arrays = {"x": rng.standard_normal((6, 8, 10)).astype(f32), "v": rng.standard_normal((3, 10)).astype(f32),
              "idx": rng.integers(-8, 8, (6, 4)).astype(np.int64), "lab": np.array([0, 6, 3, -1, 2], dtype=np.int64),
              "u": rng.standard_normal((6, 8)).astype(f32)}
    ref = evaluate_graph(g, dict(arrays))
    export(g, "nodes_indexing", arrays, ref)


if __name__ == "__main__":
    main()

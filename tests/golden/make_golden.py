"""Generate the workload graphs and golden vectors from the REFERENCE itself.

Test infrastructure: this script is the only committed code that imports the
reference (``ml_switcheroo_compiler``), read-only, from the source tree named by ``--reference-src`` or
``$ML_SWITCHEROO_REFERENCE_SRC``,
with the usage-derived ``ml_switcheroo_ir`` stand-in under ``oracle/standin``.
It is run here (CPU container) and its outputs are committed:

* ``tests/golden/graphs/<workload>.json``  the fwd+bwd ``LogicalGraph`` exactly as the
  reference's tracer (``grad/jvp_vjp.py:483``) and graph AD (``transforms/autodiff.py:382``)
  emit it, serialized node by node (ids, op types, inputs, attributes, shape metadata);
* ``tests/golden/<case>.npz``  seeded inputs and the reference numpy backend's
  ``evaluate_graph`` outputs (``interpreter/evaluator.py:272``) for small cases.

Several reference VJP rules are defective for these graphs (un-broadcast missing for
Add/Multiply, Softmax/LogSoftmax rules mis-parsed, batched Matmul transposes all axes,
Gelu fwd/bwd mismatch, ReduceMean divides by the full element count, Reshape rule keeps
the forward shape, Gather/TakeAlongAxis have zero gradients). Corrected rules are
registered through the reference's own public plugin API ``register_vjp``
(``transforms/autodiff_rules/vjp_registry.py:95``; the Python registry is consulted
before the YAML rules, ``vjp_registry.py:126``). The reference source is not edited.
Every corrected rule emits only ops that the reference numpy backend evaluates.

Usage:  python tests/golden/make_golden.py --reference-src PATH [--graphs] [--goldens] [--only NAME]
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from refpath import add_reference_to_path  # noqa: E402

REF_SRC = add_reference_to_path()
sys.path.insert(0, os.path.join(REPO, "ml-switcheroo-compiler_b200"))

from b200.workloads import GOLDEN_CASES, GRAPH_CASES, WORKLOADS, make_inputs  # noqa: E402

# ---------------------------------------------------------------------------------
# reference imports
# ---------------------------------------------------------------------------------
from ml_switcheroo_compiler.core.config import config  # noqa: E402
from ml_switcheroo_compiler.grad.jvp_vjp import (  # noqa: E402
    _attach_cotangent_inputs,
    _build_traced_logical_graph,
    _convert_to_tensors,
)
from ml_switcheroo_compiler.backends.registry import get_active_backend  # noqa: E402
from ml_switcheroo_compiler.core.utils.graph_utils import topological_sort  # noqa: E402
from ml_switcheroo_compiler.interpreter.environment import Environment  # noqa: E402
from ml_switcheroo_compiler.interpreter.evaluator import _evaluate_node, evaluate_graph  # noqa: E402
from ml_switcheroo_compiler.ops.base import emit_ir_node  # noqa: E402
from ml_switcheroo_compiler.ops.dispatcher import dispatch_op as D  # noqa: E402
from ml_switcheroo_compiler.transforms.autodiff import grad as graph_grad  # noqa: E402
from ml_switcheroo_compiler.transforms.autodiff_rules.common import UnconnectedGradients  # noqa: E402
from ml_switcheroo_compiler.transforms.autodiff_rules.vjp_registry import _VJP_REGISTRY, register_vjp  # noqa: E402

config.backend = "numpy"

# ---------------------------------------------------------------------------------
# corrected VJP rules (registered through register_vjp)
# ---------------------------------------------------------------------------------


def _shape(graph, nid):
    n = graph.nodes.get(nid)
    return tuple(n.shape_metadata) if n is not None and n.shape_metadata is not None else None


def _const(graph, value):
    # float32-valued constant: the evaluator hands node.attributes["value"] to
    # backend.array (evaluator.py:760-761); an np.float32 keeps numpy in fp32.
    return emit_ir_node(graph, "Constant", [], shape_metadata=(), attributes={"value": np.float32(value)})


def _unbroadcast(graph, cot, out_shape, target_id):
    """Sum ``cot`` down to the shape of ``target_id`` (numpy broadcasting rules)."""
    tshape = _shape(graph, target_id)
    if tshape is None or tuple(tshape) == tuple(out_shape or ()):
        return cot
    return emit_ir_node(graph, "BroadcastReduce", [cot, target_id], shape_metadata=tshape)


def _binary_rule(kind):
    def rule(graph, node, cot):
        a, b = node.inputs[0], node.inputs[1]
        out_shape = _shape(graph, node.id)
        sa, sb = _shape(graph, a), _shape(graph, b)
        if kind == "add":
            ga, gb = cot, cot
        elif kind == "sub":
            ga = cot
            gb = emit_ir_node(graph, "Negative", [cot], shape_metadata=out_shape)
        else:  # mul
            ga = emit_ir_node(graph, "Multiply", [cot, b], shape_metadata=out_shape)
            gb = emit_ir_node(graph, "Multiply", [cot, a], shape_metadata=out_shape)
        del sa, sb
        return (_unbroadcast(graph, ga, out_shape, a), _unbroadcast(graph, gb, out_shape, b))

    return rule


def _softmax_rule(graph, node, cot):
    # dx = y * (g - sum(g * y, axis, keepdims))
    y = node.id
    shp = _shape(graph, y)
    axis = node.attributes.get("axis", -1)
    gy = emit_ir_node(graph, "Multiply", [cot, y], shape_metadata=shp)
    red = list(shp)
    red[axis] = 1
    s = emit_ir_node(graph, "ReduceSum", [gy], shape_metadata=tuple(red), attributes={"axis": axis, "keepdims": True})
    d = emit_ir_node(graph, "Subtract", [cot, s], shape_metadata=shp)
    return (emit_ir_node(graph, "Multiply", [y, d], shape_metadata=shp),)


def _log_softmax_rule(graph, node, cot):
    # dx = g - exp(y) * sum(g, axis, keepdims)
    y = node.id
    shp = _shape(graph, y)
    axis = node.attributes.get("axis", -1)
    red = list(shp)
    red[axis] = 1
    s = emit_ir_node(graph, "ReduceSum", [cot], shape_metadata=tuple(red), attributes={"axis": axis, "keepdims": True})
    e = emit_ir_node(graph, "Exp", [y], shape_metadata=shp)
    es = emit_ir_node(graph, "Multiply", [e, s], shape_metadata=shp)
    return (emit_ir_node(graph, "Subtract", [cot, es], shape_metadata=shp),)


def _gelu_tanh_rule(graph, node, cot):
    # Forward is 0.5 x (1 + tanh(k (x + c x^3))) (core_math_ops/math_nn.py:184-199), so
    # d/dx = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3 c x^2),  t = tanh(k (x + c x^3)).
    x = node.inputs[0]
    shp = _shape(graph, x)
    k = float(np.sqrt(2.0 / np.pi))
    c = 0.044715

    def E(op, *ins):
        return emit_ir_node(graph, op, list(ins), shape_metadata=shp)

    x2 = E("Multiply", x, x)
    x3 = E("Multiply", x2, x)
    inner = E("Multiply", E("Add", x, E("Multiply", x3, _const(graph, c))), _const(graph, k))
    t = E("Tanh", inner)
    left = E("Multiply", E("Add", t, _const(graph, 1.0)), _const(graph, 0.5))
    sech2 = E("Subtract", _const(graph, 1.0), E("Multiply", t, t))
    dinner = E("Multiply", E("Add", E("Multiply", x2, _const(graph, 3.0 * c)), _const(graph, 1.0)), _const(graph, k))
    right = E("Multiply", E("Multiply", E("Multiply", x, sech2), dinner), _const(graph, 0.5))
    return (E("Multiply", cot, E("Add", left, right)),)


def _matmul_rule(graph, node, cot):
    # C = A @ B with A [..., M, K], B [..., K, N] (or B [K, N] shared over the batch).
    a, b = node.inputs[0], node.inputs[1]
    sa, sb = _shape(graph, a), _shape(graph, b)
    sc = _shape(graph, node.id)

    def swap_last2(nid, shp):
        perm = list(range(len(shp)))
        perm[-1], perm[-2] = perm[-2], perm[-1]
        tshape = tuple(shp[p] for p in perm)
        return emit_ir_node(graph, "Transpose", [nid], shape_metadata=tshape, attributes={"axes": perm})

    ga = emit_ir_node(graph, "Matmul", [cot, swap_last2(b, sb)], shape_metadata=sa)
    if len(sa) == len(sb):
        gb = emit_ir_node(graph, "Matmul", [swap_last2(a, sa), cot], shape_metadata=sb)
    else:
        # shared 2-D weight: flatten the batch dims into rows first
        rows = int(np.prod(sa[:-1]))
        a2 = emit_ir_node(graph, "Reshape", [a], shape_metadata=(rows, sa[-1]), attributes={"shape": [rows, sa[-1]]})
        c2 = emit_ir_node(graph, "Reshape", [cot], shape_metadata=(rows, sc[-1]), attributes={"shape": [rows, sc[-1]]})
        gb = emit_ir_node(graph, "Matmul", [swap_last2(a2, (rows, sa[-1])), c2], shape_metadata=sb)
    return (ga, gb)


def _transpose_rule(graph, node, cot):
    x = node.inputs[0]
    sx = _shape(graph, x)
    axes = node.attributes.get("axes")
    if axes is None:
        inv = None
        attrs = {}
    else:
        axes = [int(v) % len(sx) for v in axes]
        inv = [0] * len(axes)
        for i, p in enumerate(axes):
            inv[p] = i
        attrs = {"axes": inv}
    return (emit_ir_node(graph, "Transpose", [cot], shape_metadata=sx, attributes=attrs),)


def _reshape_rule(graph, node, cot):
    x = node.inputs[0]
    sx = _shape(graph, x)
    return (emit_ir_node(graph, "Reshape", [cot], shape_metadata=sx, attributes={"shape": list(sx)}),)


def _reduce_mean_rule(graph, node, cot):
    # dx = broadcast(g) / (number of elements reduced), not / numel(x)
    x = node.inputs[0]
    sx = _shape(graph, x)
    axis = node.attributes.get("axis", None)
    if axis is None:
        count = int(np.prod(sx))
    else:
        axes = axis if isinstance(axis, (list, tuple)) else [axis]
        count = int(np.prod([sx[int(ax)] for ax in axes]))
    bl = emit_ir_node(graph, "BroadcastLike", [cot, x], shape_metadata=sx)
    return (emit_ir_node(graph, "Multiply", [bl, _const(graph, 1.0 / count)], shape_metadata=sx),)


def _take_along_axis_rule(graph, node, cot):
    # scatter the cotangent back into a zero tensor shaped like the source
    x, idx = node.inputs[0], node.inputs[1]
    sx = _shape(graph, x)
    axis = node.attributes.get("axis", -1)
    z = emit_ir_node(graph, "ZerosLike", [x], shape_metadata=sx)
    gx = emit_ir_node(graph, "ScatterAdd", [z, idx, cot], shape_metadata=sx, attributes={"dim": axis})
    return (gx, UnconnectedGradients.NONE)


def _take_rule(graph, node, cot):
    # Take(table, ids, axis=0) == table[ids]; d table = scatter-add of the cotangent rows
    # (numpy ``add.at`` inside TensorScatterAdd accumulates repeated ids).
    table, ids = node.inputs[0], node.inputs[1]
    st, si = _shape(graph, table), _shape(graph, ids)
    nrow = int(np.prod(si))
    z = emit_ir_node(graph, "ZerosLike", [table], shape_metadata=st)
    idx = emit_ir_node(graph, "Reshape", [ids], shape_metadata=(nrow, 1), attributes={"shape": [nrow, 1]})
    c2 = emit_ir_node(graph, "Reshape", [cot], shape_metadata=(nrow,) + tuple(st[1:]), attributes={"shape": [nrow] + list(st[1:])})
    gt = emit_ir_node(graph, "TensorScatterAdd", [z, idx, c2], shape_metadata=st)
    return (gt, UnconnectedGradients.NONE)


CORRECTED_RULES = {
    "Take": _take_rule,
    "Add": _binary_rule("add"),
    "Subtract": _binary_rule("sub"),
    "Multiply": _binary_rule("mul"),
    "Softmax": _softmax_rule,
    "LogSoftmax": _log_softmax_rule,
    "Gelu": _gelu_tanh_rule,
    "Matmul": _matmul_rule,
    "MatMul": _matmul_rule,
    "Transpose": _transpose_rule,
    "Reshape": _reshape_rule,
    "ReduceMean": _reduce_mean_rule,
    "TakeAlongAxis": _take_along_axis_rule,
}


def _as_shape(v):
    return tuple(v.shape) if hasattr(v, "shape") else tuple(v)


def _take_shape(table, ids, *rest, **kw):
    # Take(table, ids, axis=0) -> ids.shape + table.shape[1:]
    return tuple(_as_shape(ids)) + tuple(_as_shape(table)[1:])


def register_corrected_rules() -> None:
    from ml_switcheroo_compiler.ops.shape_inference import _SHAPE_INFERENCE_REGISTRY, register_shape_inference

    if "Take" not in _SHAPE_INFERENCE_REGISTRY:
        register_shape_inference("Take")(_take_shape)
    for name, fn in CORRECTED_RULES.items():
        if name not in _VJP_REGISTRY:
            register_vjp(name)(fn)


# ---------------------------------------------------------------------------------
# forward functions of the five workloads (reference op vocabulary)
# ---------------------------------------------------------------------------------


def fwd_mlp(x, W1, b1, W2, b2, labels):
    h = D("Relu", D("Add", D("Matmul", x, W1), b1))
    lg = D("Add", D("Matmul", h, W2), b2)
    ls = D("LogSoftmax", lg, axis=-1)
    picked = D("TakeAlongAxis", ls, labels, axis=-1)
    return D("ReduceMean", D("Neg", picked))


def fwd_rowfused(x, a, b, gamma, beta):
    p = D("Add", D("Multiply", x, a), b)
    return D("Softmax", D("LayerNorm", D("Gelu", p), gamma, beta, eps=1e-5), axis=-1)


def fwd_bmm(A, B, bias):
    return D("Relu", D("Add", D("Matmul", A, B), bias))


def fwd_cnn(X, w1, w2, w3, Wl, bl, labels):
    n = X.shape[0]
    h = D("Relu", D("Conv2D", X, w1, stride=[1, 1], padding="VALID"))
    h = D("Relu", D("Conv2D", h, w2, stride=[2, 2], padding="VALID"))
    h = D("Relu", D("Conv2D", h, w3, stride=[2, 2], padding="VALID"))
    c, hh, ww = h.shape[1], h.shape[2], h.shape[3]
    pooled = D("ReduceMean", D("Reshape", h, shape=(n, c, hh * ww)), axis=-1, keepdims=True)
    p = D("Reshape", pooled, shape=(n, c))
    lg = D("Add", D("Matmul", p, Wl), bl)
    picked = D("TakeAlongAxis", D("LogSoftmax", lg, axis=-1), labels, axis=-1)
    return D("ReduceMean", D("Neg", picked))


def fwd_transformer(*args):
    """Pre-LN encoder stack on 2-D activations [B*S, d]; next-token CE via a weight mask."""
    from b200.workloads import transformer_roles

    a = dict(zip(transformer_roles(_TFM_DIMS["L"]), args))
    B, S, d, H = _TFM_DIMS["B"], _TFM_DIMS["S"], _TFM_DIMS["d"], _TFM_DIMS["H"]
    hd = d // H
    T = B * S
    tok = D("Take", a["tok_emb"], a["ids"], axis=0)
    x = D("Reshape", D("Add", D("Reshape", tok, shape=(B, S, d)), a["pos_emb"]), shape=(T, d))
    for i in range(_TFM_DIMS["L"]):
        p = lambda k: a[f"l{i}_{k}"]  # noqa: E731
        hn = D("LayerNorm", x, p("ln1_g"), p("ln1_b"), eps=1e-5)

        def heads(w, bvec, perm):
            y = D("Add", D("Matmul", hn, w), bvec)
            return D("Transpose", D("Reshape", y, shape=(B, S, H, hd)), axes=perm)

        q = heads(p("Wq"), p("bq"), [0, 2, 1, 3])
        kT = heads(p("Wk"), p("bk"), [0, 2, 3, 1])
        v = heads(p("Wv"), p("bv"), [0, 2, 1, 3])
        att = D("Softmax", D("Multiply", D("Matmul", q, kT), a["attn_scale"]), axis=-1)
        ctx = D("Reshape", D("Transpose", D("Matmul", att, v), axes=[0, 2, 1, 3]), shape=(T, d))
        x = D("Add", x, D("Add", D("Matmul", ctx, p("Wo")), p("bo")))
        hn2 = D("LayerNorm", x, p("ln2_g"), p("ln2_b"), eps=1e-5)
        f = D("Gelu", D("Add", D("Matmul", hn2, p("W1")), p("b1")))
        x = D("Add", x, D("Add", D("Matmul", f, p("W2")), p("b2")))
    hf = D("LayerNorm", x, a["lnf_g"], a["lnf_b"], eps=1e-5)
    logits = D("Matmul", hf, a["Whead"])
    picked = D("TakeAlongAxis", D("LogSoftmax", logits, axis=-1), a["labels"], axis=-1)
    return D("ReduceSum", D("Multiply", picked, a["wmask"]))


_TFM_DIMS: dict = {}

FORWARDS = {"mlp": fwd_mlp, "rowfused": fwd_rowfused, "bmm": fwd_bmm, "cnn": fwd_cnn, "transformer": fwd_transformer}


# ---------------------------------------------------------------------------------
# graph build + export
# ---------------------------------------------------------------------------------


def _jsonable(v):
    if isinstance(v, np.generic):
        return v.item()
    if isinstance(v, np.ndarray):
        return v.tolist()
    if isinstance(v, (list, tuple)):
        return [_jsonable(u) for u in v]
    if isinstance(v, dict):
        return {str(k): _jsonable(u) for k, u in v.items()}
    if isinstance(v, (int, float, str, bool)) or v is None:
        return v
    if hasattr(v, "value") and isinstance(getattr(v, "value"), str):  # enums
        return v.value
    return str(v)


def _bshape(*shapes):
    return tuple(int(d) for d in np.broadcast_shapes(*[tuple(sh) for sh in shapes]))


def static_shapes(g, input_shapes) -> dict:
    """Shape of every forward node from the input shapes alone (no values computed)."""
    shp = dict(input_shapes)
    for n in topological_sort(g):
        if n.id in shp or n.op_type in ("Input", "Output"):
            continue
        ins = [shp[i] for i in n.inputs]
        a = n.attributes or {}
        op = n.op_type
        if op in ("Add", "Subtract", "Multiply", "TrueDivide"):
            out = _bshape(*ins)
        elif op in ("Relu", "Gelu", "Neg", "Negative", "Exp", "Tanh", "Softmax", "LogSoftmax", "LayerNorm"):
            out = ins[0]
        elif op in ("Matmul", "MatMul"):
            sa, sb = ins
            out = _bshape(sa[:-2], sb[:-2]) + (sa[-2], sb[-1])
        elif op == "Reshape":
            out = tuple(int(d) for d in (a.get("shape") or a.get("newshape")))
        elif op == "Transpose":
            axes = a.get("axes") or list(reversed(range(len(ins[0]))))
            out = tuple(ins[0][int(p)] for p in axes)
        elif op in ("ReduceSum", "ReduceMean", "ReduceMax"):
            axis, keep = a.get("axis"), bool(a.get("keepdims", False))
            if axis is None:
                out = tuple(1 for _ in ins[0]) if keep else ()
            else:
                axes = [int(x) % len(ins[0]) for x in (axis if isinstance(axis, (list, tuple)) else [axis])]
                out = tuple((1 if i in axes else d) for i, d in enumerate(ins[0]) if keep or i not in axes)
        elif op == "TakeAlongAxis":
            out = _bshape(ins[0][:-1], ins[1][:-1]) + (ins[1][-1],)
        elif op == "Take":
            out = tuple(ins[1]) + tuple(ins[0][1:])
        elif op == "Conv2D":
            (n_, _, h, w), (co, _, kh, kw) = ins
            st = a.get("stride", [1, 1])
            out = (n_, co, (h - kh) // st[0] + 1, (w - kw) // st[1] + 1)
        else:
            raise NotImplementedError(op)
        shp[n.id] = tuple(int(d) for d in out)
    return shp


def annotate_shapes(g, inputs) -> None:
    """Overwrite each forward node's ``shape_metadata`` with the shape numpy computes.

    The tracer's static shape inference leaves wrong or placeholder metadata on some
    nodes (e.g. ``('None',)`` after ``TakeAlongAxis``, ``()`` after ``Neg``), and the
    VJP rules read it. Evaluating the forward graph once with the reference numpy
    backend (same node loop as ``evaluate_graph``, evaluator.py:293-297) gives the
    true shapes.
    """
    env = Environment(dict(inputs))
    backend = get_active_backend()
    for n in topological_sort(g):
        _evaluate_node(n, env, backend)
        if n.id in env and n.op_type not in ("Output",):
            v = env.get(n.id)
            if hasattr(v, "shape"):
                n.shape_metadata = tuple(int(d) for d in v.shape)


def build_graph(workload: str, dims: dict):
    """Trace the forward, attach cotangents, run graph AD; return (graph, roles, outputs)."""
    spec = WORKLOADS[workload]
    arrays = make_inputs(workload, dims, seed=0)
    prim_roles = spec["inputs"](dims) if callable(spec["inputs"]) else spec["inputs"]
    _TFM_DIMS.clear()
    _TFM_DIMS.update(dims)
    prims = [arrays[r] for r in prim_roles]
    g = _build_traced_logical_graph(FORWARDS[spec["forward"]], _convert_to_tensors(prims), workload)
    roles = dict(zip(prim_roles, g.inputs[: len(prim_roles)]))
    fwd_out = g.nodes[g.outputs[0]].inputs[0]
    shapes = static_shapes(g, {roles[r]: tuple(arrays[r].shape) for r in prim_roles})
    for nid, sh in shapes.items():
        if g.nodes[nid].op_type != "Input":
            g.nodes[nid].shape_metadata = sh
    out_node_id, cot_map, cot_ids = _attach_cotangent_inputs(g)
    roles["cotangent"] = cot_ids[0]
    wrt_roles = spec["wrt"](dims) if callable(spec["wrt"]) else spec["wrt"]
    wrt = [roles[r] for r in wrt_roles]
    gg = graph_grad(g, wrt, out_node_id, cotangent_id=cot_map)
    outputs = {spec["fwd_output"]: fwd_out}
    for r, gid in zip(wrt_roles, list(gg.outputs)):
        outputs["d_" + r] = gid
    if spec.get("argmax_of_output"):
        shp = tuple(gg.nodes[fwd_out].shape_metadata)
        am = emit_ir_node(gg, "Argmax", [fwd_out], shape_metadata=shp[:-1], attributes={"axis": -1})
        outputs["argmax"] = am
    gg.outputs = list(outputs.values())
    return gg, roles, outputs, arrays


def export_graph(gg, roles, outputs, workload, dims) -> dict:
    nodes = []
    for n in gg.nodes.values():
        extra = {}
        if n.op_type == "Constant":
            # numpy dtype the reference evaluates this constant in (np.array(value))
            extra["const_dtype"] = str(np.asarray(n.attributes["value"]).dtype)
        nodes.append(
            {
                **extra,
                "id": n.id,
                "op_type": n.op_type,
                "inputs": list(n.inputs),
                "attributes": _jsonable(dict(n.attributes or {})),
                "shape_metadata": _jsonable(list(n.shape_metadata)) if n.shape_metadata is not None else None,
            }
        )
    return {
        "format": "logical-graph-json/1",
        "name": gg.name,
        "workload": workload,
        "dims": dims,
        "inputs": list(gg.inputs),
        "outputs": list(gg.outputs),
        "roles": roles,
        "output_names": outputs,
        "nodes": nodes,
    }


def save_graph(doc: dict, path: str) -> None:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with gzip.open(path, "wt", encoding="utf-8") as f:
        json.dump(doc, f, separators=(",", ":"), sort_keys=False)


def evaluate_reference(gg, roles, arrays):
    inputs = {nid: arrays[r] for r, nid in roles.items()}
    return evaluate_graph(gg, inputs)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    register_corrected_rules()

    for case, (workload, dims) in GRAPH_CASES.items():
        if args.only and args.only not in case:
            continue
        gg, roles, outputs, _ = build_graph(workload, dims)
        doc = export_graph(gg, roles, outputs, workload, dims)
        save_graph(doc, os.path.join(HERE, "graphs", case + ".json.gz"))
        print("graph", case, len(doc["nodes"]), "nodes")
    for case, (workload, dims) in GOLDEN_CASES.items():
        if args.only and args.only not in case:
            continue
        gg, roles, outputs, arrays = build_graph(workload, dims)
        doc = export_graph(gg, roles, outputs, workload, dims)
        save_graph(doc, os.path.join(HERE, "graphs", case + ".json.gz"))
        res = evaluate_reference(gg, roles, arrays)
        blob = {"in__" + r: np.asarray(arrays[r]) for r in roles}
        for name, nid in outputs.items():
            blob["out__" + name] = np.asarray(res[nid])
        np.savez_compressed(os.path.join(HERE, case + ".npz"), **blob)
        print("golden", case, {k: (v.shape, str(v.dtype)) for k, v in blob.items() if k.startswith("out__")})


if __name__ == "__main__":
    main()

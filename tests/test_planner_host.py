"""Host-side planner logic (no GPU): pattern matching on the reference-traced graphs,
elementwise clustering limits, scheduling, graph loading and pruning."""

import numpy as np
import pytest
import torch

from conftest import load_golden


def _meta_from_oracle(case):
    """Shapes/dtypes of every value from the CPU oracle (stand-in for the recorded run)."""
    from b200 import graph as G
    from b200.fusion import Meta
    from oracle import evaluator as O

    g = G.load(case)
    og = O.load_graph(case)
    ins, _ = load_golden(case)
    env = {nid: ins[r] for r, nid in g.roles.items()}
    for node in O.topo_order(og):
        if node["op_type"] == "Input":
            continue
        vals = [env[i] for i in node["inputs"]]
        if node["op_type"] == "Output":
            env[node["id"]] = vals[0]
            continue
        if node["op_type"] == "Constant":
            env[node["id"]] = float(node["attributes"]["value"])
            continue
        env[node["id"]] = O.execute_op(node["op_type"], *vals, **O._kwargs(node, node["op_type"]))
    conv = {np.dtype("float32"): torch.float32, np.dtype("float64"): torch.float32, np.dtype("int64"): torch.int64,
            np.dtype("bool"): torch.bool}
    meta = {}
    for k, v in env.items():
        if isinstance(v, (int, float)):
            meta[k] = Meta(v)
        else:
            a = np.asarray(v)
            meta[k] = Meta(torch.empty(a.shape, dtype=conv[a.dtype]))
    return g, meta


@pytest.mark.parametrize("case", ["rowfused_small", "rowfused_ragged"])
def test_rowfused_pattern_matches_reference_graph(case):
    from b200.executor import Plan
    from b200.fusion import find_rowfused

    g, meta = _meta_from_oracle(case)
    plan_nodes = Plan.__new__(Plan)
    order = g.topo_order()
    live = {n.id: n for n in order if n.op_type != "Input"}
    users = {}
    for n in live.values():
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    found = find_rowfused(g, live, meta, users)
    assert len(found) == 1
    m = found[0]
    assert set(m.outputs) >= {"y", "dx", "da", "db", "am"}
    assert m.outputs["dx"] == g.output_names["d_x"]
    assert m.outputs["da"] == g.output_names["d_a"]
    assert m.outputs["db"] == g.output_names["d_b"]
    assert m.outputs["am"] == g.output_names["argmax"]
    assert m.bind["x"] == g.roles["x"] and m.bind["cot"] == g.roles["cotangent"]
    del plan_nodes


def test_pattern_rejects_other_graphs():
    from b200.fusion import find_rowfused

    g, meta = _meta_from_oracle("mlp_small")
    live = {n.id: n for n in g.topo_order() if n.op_type != "Input"}
    users = {}
    for n in live.values():
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    assert find_rowfused(g, live, meta, users) == []


def test_elementwise_clusters_respect_program_limits():
    from b200 import _lib as L
    from b200.fusion import _alloc_registers, _cluster_io, cluster_elementwise

    g, meta = _meta_from_oracle("transformer_small")
    need, stack = set(), list(g.outputs)
    while stack:
        v = stack.pop()
        if v not in need and v in g.nodes:
            need.add(v)
            stack.extend(g.nodes[v].inputs)
    order = [n for n in g.topo_order() if n.op_type != "Input" and n.id in need]
    users = {}
    for n in order:
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    clusters = cluster_elementwise(g, order, meta, set(), users, set(g.outputs))
    assert any(len(c) >= 5 for c in clusters)  # the GELU-derivative chains fuse
    for c in clusters:
        ext_in, outs = _cluster_io(g, c, users, set(g.outputs))
        assert len(ext_in) <= L.EW_MAX_IN and 1 <= len(outs) <= L.EW_MAX_OUT
        prog, regs = _alloc_registers(g, c, ext_in, outs)
        assert all(max(r[1], r[2], r[3], r[4]) < L.EW_MAX_REG for r in prog)
        shapes = {meta[n.id].shape for n in c}
        assert len(shapes) == 1


def test_graph_prune_and_cycle():
    from b200 import graph as G
    from b200.errors import CompilationError

    g = G.load("cnn_small")
    order = g.topo_order()
    assert len(order) == len(g.nodes)
    pos = {n.id: i for i, n in enumerate(order)}
    for n in order:
        for i in n.inputs:
            assert pos[i] < pos[n.id]
    bad = G.from_json({"name": "c", "inputs": [], "outputs": ["b"],
                       "nodes": [{"id": "a", "op_type": "Relu", "inputs": ["b"]}, {"id": "b", "op_type": "Relu", "inputs": ["a"]}]})
    with pytest.raises(CompilationError):
        bad.topo_order()


def test_schedule_orders_fused_groups():
    from b200.executor import Step
    from b200.fusion import _schedule

    s1 = Step(["b"], ["a"], lambda e: None, "s1")
    s2 = Step(["c"], ["b"], lambda e: None, "s2")
    s3 = Step(["d"], ["c", "a"], lambda e: None, "s3")
    order = _schedule([(["d"], s3), (["c"], s2), (["b"], s1)])
    assert [s.label for s in order] == ["s1", "s2", "s3"]


@pytest.mark.parametrize("case", ["mlp_small", "cnn_small", "transformer_small"])
def test_xent_pattern_matches_reference_graphs(case):
    from b200.fusion import find_xent

    g, meta = _meta_from_oracle(case)
    need, stack = set(), list(g.outputs)
    while stack:
        v = stack.pop()
        if v not in need and v in g.nodes:
            need.add(v)
            stack.extend(g.nodes[v].inputs)
    live = {n.id: n for n in g.topo_order() if n.op_type != "Input" and n.id in need}
    users = {}
    for n in live.values():
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    found = find_xent(g, live, meta, users, set(g.outputs))
    assert len(found) == 1 and set(found[0].outputs) == {"dx", "picked"}


def test_attention_softmax_patterns_match_transformer_graph():
    """Every attention softmax (scaled by the attn_scale input) and its VJP fuse; the
    VJP output feeds only GEMMs, so it is produced in bf16 alone."""
    from b200 import ops
    from b200.fusion import find_softmax, find_softmax_bwd

    g, meta = _meta_from_oracle("transformer_small")
    need, stack = set(), list(g.outputs)
    while stack:
        v = stack.pop()
        if v not in need and v in g.nodes:
            need.add(v)
            stack.extend(g.nodes[v].inputs)
    live = {n.id: n for n in g.topo_order() if n.op_type != "Input" and n.id in need}
    users = {}
    for n in live.values():
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    old = ops.Config.matmul_dtype
    ops.Config.matmul_dtype = "bf16"
    try:
        fwd = find_softmax(g, live, meta, users, set(g.outputs))
        bwd = find_softmax_bwd(g, live, meta, users, set(g.outputs))
    finally:
        ops.Config.matmul_dtype = old
    n_layers = 2
    fwd = [m for m in fwd if m.bind["log"] == "False"]  # the LogSoftmax of the logits goes to the xent kernel
    assert len(fwd) == n_layers and len(bwd) == n_layers
    scale = g.roles["attn_scale"]
    for m in fwd:
        assert m.bind["scale"] == scale and m.bind["log"] == "False"
        assert m.bind["bf16"] == "True" and m.bind["f32"] == "True"  # att@v GEMM + the VJP
    for m in bwd:
        assert m.bind["scale"] == scale
        assert m.bind["bf16"] == "True" and m.bind["f32"] == "False"
    assert {m.bind["y"] for m in bwd} == {m.bind["y"] for m in fwd}


def test_gelu_bwd_pattern_matches_transformer_ffn():
    """The GELU VJP chain of every FFN fuses with its bias gradient, and its output
    (only read by the two weight/input-gradient GEMMs) is produced in bf16 alone."""
    from b200 import ops
    from b200.fusion import find_gelu_bwd

    g, meta = _meta_from_oracle("transformer_small")
    need, stack = set(), list(g.outputs)
    while stack:
        v = stack.pop()
        if v not in need and v in g.nodes:
            need.add(v)
            stack.extend(g.nodes[v].inputs)
    live = {n.id: n for n in g.topo_order() if n.op_type != "Input" and n.id in need}
    users = {}
    for n in live.values():
        for i in n.inputs:
            users.setdefault(i, []).append(n.id)
    old = ops.Config.matmul_dtype
    ops.Config.matmul_dtype = "bf16"
    try:
        found = find_gelu_bwd(g, live, meta, users, set(g.outputs))
    finally:
        ops.Config.matmul_dtype = old
    assert len(found) == 2
    for m in found:
        assert "db" in m.outputs and m.outputs["db"] in set(g.outputs)
        assert m.bind["bf16"] == "True" and m.bind["f32"] == "False"

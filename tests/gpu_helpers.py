"""Helpers shared by the -m gpu tests."""

import numpy as np
import torch

from conftest import load_golden

BF16_WORKLOADS = {"bmm", "cnn", "transformer"}


def set_policy(workload: str) -> None:
    from b200 import ops

    bf = workload in BF16_WORKLOADS
    ops.Config.matmul_dtype = "bf16" if bf else "f32"
    ops.Config.conv_dtype = "bf16" if bf else "f32"


def to_np(v):
    if isinstance(v, torch.Tensor):
        v = v.detach()
        if v.dtype == torch.bfloat16:
            v = v.float()
        return v.cpu().numpy()
    return np.asarray(v)


def assert_close(name, got, ref, rtol, atol_scale=None):
    got = to_np(got)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    if ref.dtype.kind in "iub":
        np.testing.assert_array_equal(got, ref, err_msg=name)
        return
    scale = float(np.abs(ref).max()) if ref.size else 1.0
    atol = rtol * max(scale, 1e-30) if atol_scale is None else atol_scale
    np.testing.assert_allclose(got.astype(np.float64), ref.astype(np.float64), rtol=rtol, atol=atol, err_msg=name)


def run_case(case: str, mode: str = "graph"):
    """Evaluate a golden case on the b200 backend; returns ({name: value}, golden outs, graph)."""
    from b200 import graph as G
    from b200.backend import B200Backend
    from b200.executor import GraphRunner

    ins, outs = load_golden(case)
    g = G.load(case)
    set_policy(g.meta["workload"])
    inputs = {nid: torch.from_numpy(np.ascontiguousarray(ins[r])).cuda() for r, nid in g.roles.items()}
    if mode == "graph":
        res = B200Backend.execute_graph(g, inputs)
    elif mode == "pernode":
        res = GraphRunner(g, fuse=False)(inputs)
    elif mode == "compiled":
        fn = B200Backend.compile_graph(g)
        fn(inputs)
        res = fn(inputs)
    elif mode == "compiled_host":  # replays fed from pinned host tensors (copied into the static buffers)
        fn = B200Backend.compile_graph(g)
        fn(inputs)
        host = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        fn(host)
        res = {k: v.clone() for k, v in fn(host).items()}
    else:
        raise ValueError(mode)
    return {name: res[nid] for name, nid in g.output_names.items()}, outs, g

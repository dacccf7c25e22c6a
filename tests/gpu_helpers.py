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


def rms(a) -> float:
    a = np.asarray(a, dtype=np.float64)
    return float(np.sqrt(np.mean(a * a))) if a.size else 0.0


def assert_close(name, got, ref, rtol, floor=0.0):
    """Elementwise: |got - ref| <= rtol * |ref| + atol for every element, with the
    absolute floor atol = rtol * max(rms(ref), floor).

    Why a floor at all: an entry much smaller than its output's typical magnitude is a sum
    whose terms cancelled, so its absolute rounding error is set by the size of those
    terms, which is the output's RMS, not by the entry itself. The floor bounds that error
    at rtol of the RMS. ``floor`` (default 0) covers outputs that are zero in exact
    arithmetic (pure rounding noise, RMS included): the caller derives it from a related
    output. Integer / bool outputs (argmax, labels, gathers) must be bit-exact."""
    got = to_np(got)
    ref = np.asarray(ref)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    if ref.dtype.kind in "iub":
        np.testing.assert_array_equal(got, ref, err_msg=name)
        return
    g64, r64 = got.astype(np.float64), ref.astype(np.float64)
    atol = rtol * max(rms(r64), float(floor), 1e-30)
    err = np.abs(g64 - r64)
    lim = atol + rtol * np.abs(r64)
    bad = ~(err <= lim)
    if bad.any():
        k = int(np.argmax(np.where(bad, err / lim, 0)))
        raise AssertionError(f"{name}: {int(bad.sum())} of {ref.size} elements outside rtol {rtol} (atol {atol:.3g}); "
                             f"worst at flat index {k}: got {g64.flat[k]:.6g}, ref {r64.flat[k]:.6g}, "
                             f"|diff| / limit = {float(err.flat[k] / lim.flat[k]):.3g}")


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

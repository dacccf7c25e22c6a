"""The drop-in boundary, driven by what the reference's own callers do.

The calls were recorded from the reference (``tests/golden/make_boundary_golden.py``),
with a recording subclass of ``B200Backend`` in the backend's place:

* ``protocols.json``: the real ``B200Backend`` registered through the reference's
  ``register_backend`` is what ``BackendRegistry.get("b200")`` returns, and the
  reference's structural checks route whole graphs to its ``execute_graph`` /
  ``compile_graph`` (``grad/api.py:85-106``, ``grad/jvp_vjp.py:205-226``);
* per-node: every ``execute_op`` / ``array`` / ``asarray`` call the reference's
  ``evaluate_graph`` makes while interpreting a graph (``interpreter/evaluator.py:428-593``,
  ``:761``), replayed in order against ``B200Backend`` with the reference's own argument
  values (numpy arrays for graph inputs, the backend's previous results otherwise), each
  result compared with the reference numpy backend's;
* whole graph: the ``LogicalGraph`` (a pydantic object, rebuilt from its dump with the
  IR classes) and inputs that the reference's ``vjp`` pullback passes to
  ``backend.execute_graph`` (``grad/jvp_vjp.py:511-529``), run through
  ``execute_graph`` and ``compile_graph``.

fp32 results at rtol 1e-4 elementwise (absolute floor 1e-4 x RMS), integer results
bit-exact.
"""

import glob
import gzip
import json
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT
from gpu_helpers import assert_close, to_np

BOUNDARY = os.path.join(GOLDEN, "boundary")


def test_reference_registry_and_protocols_accept_the_backend():
    """Recorded from the reference: registration and the whole-graph protocol checks."""
    with open(os.path.join(BOUNDARY, "protocols.json")) as f:
        proto = json.load(f)
    assert proto["registered"]
    assert proto["api_execute_graph"] and proto["api_compile_graph"]
    assert proto["jvp_vjp_execute_graph"] and proto["jvp_vjp_compile_graph"]
    from b200.backend import B200Backend

    for m in ("execute_op", "array", "asarray", "zeros", "item", "get_module", "execute_graph", "compile_graph"):
        assert m in proto["members"] and callable(getattr(B200Backend, m))


def _decode(ref, arrays, results):
    if "value" in ref:
        k = ref["value"]
        return results.get(k, arrays[k])
    if "seq" in ref:
        seq = [_decode(r, arrays, results) for r in ref["seq"]]
        return tuple(seq) if ref["tuple"] else seq
    return ref["lit"]


def _check(name, got, ref):
    if isinstance(got, (tuple, list)):
        for i, (g, r) in enumerate(zip(got, ref)):
            _check(f"{name}[{i}]", g, r)
        return
    r = np.asarray(ref)
    if r.dtype == np.float64:  # the reference's Python-float constants; the backend computes fp32
        r = r.astype(np.float32)
    g = np.asarray(got) if not isinstance(got, torch.Tensor) else to_np(got)
    if r.dtype.kind in "iub":
        np.testing.assert_array_equal(g, r, err_msg=name)
    else:
        assert_close(name, g.reshape(r.shape) if g.size == r.size else g, r, 1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(os.path.basename(p)[8:-8] for p in glob.glob(os.path.join(BOUNDARY, "pernode_*.json.gz"))))
def test_reference_interpreter_calls_replayed(cuda, case):
    from b200.backend import B200Backend

    with gzip.open(os.path.join(BOUNDARY, f"pernode_{case}.json.gz"), "rt") as f:
        doc = json.load(f)
    d = np.load(os.path.join(BOUNDARY, f"pernode_{case}.npz"))
    arrays = {k: d[k] for k in d.files}
    results: dict = {}
    for i, call in enumerate(doc["calls"]):
        args = [_decode(a, arrays, results) for a in call["args"]]
        kwargs = {k: _decode(v, arrays, results) for k, v in call["kwargs"].items()}
        got = getattr(B200Backend, call["method"])(*args, **kwargs)
        if call["method"] != "asarray" or isinstance(got, torch.Tensor):
            assert got is None or isinstance(got, (torch.Tensor, float, int, tuple, list)), (i, call["method"], type(got))
        torch.cuda.synchronize()
        out = call["out"]
        label = f"{case} call {i} {call['method']}({args[0] if call['method'] == 'execute_op' else ''})"
        if "value" in out:
            _check(label, got, arrays[out["value"]])
            results[out["value"]] = got
        elif "seq" in out:
            _check(label, got, [arrays[r["value"]] for r in out["seq"]])
        else:
            assert got == out["lit"] or float(got) == pytest.approx(float(out["lit"]), rel=1e-6), label
    assert doc["calls"]


def _standin_graph(dump):
    sys.path.insert(0, os.path.join(ROOT, "oracle", "standin"))
    from ml_switcheroo_ir import LogicalGraph

    return LogicalGraph.model_validate(dump)


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(os.path.basename(p)[6:-8] for p in glob.glob(os.path.join(BOUNDARY, "graph_*.json.gz"))))
def test_reference_pullback_graph_through_execute_and_compile(cuda, case):
    from b200.backend import B200Backend

    with gzip.open(os.path.join(BOUNDARY, f"graph_{case}.json.gz"), "rt") as f:
        doc = json.load(f)
    d = np.load(os.path.join(BOUNDARY, f"graph_{case}.npz"))
    ins = {k[4:]: d[k] for k in d.files if k.startswith("in__")}
    outs = {k[5:]: d[k] for k in d.files if k.startswith("out__")}
    lg = _standin_graph(doc["graph"])
    with pytest.raises(TypeError):
        hash(lg)  # the reference's graphs are unhashable: the backend keys its plans by content
    inputs = {k: B200Backend.asarray(v) for k, v in ins.items()}  # as the pullback does (jvp_vjp.py:748-752)
    res = B200Backend.execute_graph(lg, inputs)
    for k, r in outs.items():
        _check(f"{case}:execute_graph:{k}", res[k], r)
    # a second, equal graph object (the reference builds a new one per pullback call)
    # reuses the cached plan and gives the same values
    n_runners = len(B200Backend._runners)
    res2 = B200Backend.execute_graph(_standin_graph(doc["graph"]), inputs)
    assert len(B200Backend._runners) == n_runners
    for k in outs:
        if isinstance(res[k], torch.Tensor):
            assert torch.equal(res2[k], res[k]), k
        else:
            assert res2[k] == res[k], k
    # compile_graph: fresh outputs per call (a result held from call 1 is not overwritten)
    fn = B200Backend.compile_graph(lg)
    first = fn(inputs)
    kept = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in first.items()}
    scaled = {k: (v * 2 if v.is_floating_point() and k == sorted(inputs)[0] else v) for k, v in inputs.items()}
    fn(scaled)
    second = fn(inputs)
    for k, r in outs.items():
        _check(f"{case}:compile_graph:{k}", second[k], r)
        if isinstance(first[k], torch.Tensor):
            assert torch.equal(first[k], kept[k]), f"{k}: a later call overwrote an earlier call's output"

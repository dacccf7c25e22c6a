"""Time the reference's own numpy ``evaluate_graph`` beside the oracle port, on one host.

CPU baseline infrastructure. The reference cannot be installed where the GPUs are (its
build backend is not available offline), so ``bench.py --impl reference`` times the
port (``oracle/evaluator.py``). This script measures how the two compare on the same
graph and inputs, here, where the reference's source tree is available: it imports the
reference read-only from ``--reference-src PATH`` (or ``$ML_SWITCHEROO_REFERENCE_SRC``)
with the usage-derived ``ml_switcheroo_ir`` stand-in, rebuilds each stored workload graph
as the reference's ``LogicalGraph``, and times one warm-up plus ``--samples`` evaluations
of each implementation (numpy backend, fp32, the operands' own layouts).

Usage: ``python oracle/time_reference.py --reference-src PATH [--cases mlp_full transformer_b1]``
"""

from __future__ import annotations

import argparse
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
sys.path.insert(0, os.path.join(REPO, "ml-switcheroo-compiler_b200"))
sys.path.insert(0, REPO)
from refpath import add_reference_to_path  # noqa: E402

add_reference_to_path()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", nargs="+", default=["mlp_full", "rowfused_small", "transformer_b1"])
    ap.add_argument("--samples", type=int, default=3)
    args = ap.parse_args()

    from make_boundary_golden import lg_from_json  # noqa: F401  (the LogicalGraph rebuild)

    import gzip
    import json

    import numpy as np
    from ml_switcheroo_compiler.backends.registry import BackendRegistry
    from ml_switcheroo_compiler.interpreter.evaluator import evaluate_graph
    from ml_switcheroo_ir import LogicalGraph, LogicalNode

    from b200.workloads import make_inputs
    from oracle import evaluator as O

    numpy_backend = BackendRegistry.get("numpy")
    print(f"host: {os.cpu_count()} cores")
    for case in args.cases:
        path = os.path.join(REPO, "tests", "golden", "graphs", case + ".json.gz")
        with gzip.open(path, "rt") as f:
            doc = json.load(f)
        g = LogicalGraph(name=case)
        for n in doc["nodes"]:
            attrs = dict(n.get("attributes") or {})
            if n["op_type"] == "Constant" and n.get("const_dtype"):
                attrs["value"] = np.array(attrs["value"], dtype=n["const_dtype"])
            g.nodes[n["id"]] = LogicalNode(id=n["id"], op_type=n["op_type"], inputs=list(n["inputs"]), attributes=attrs,
                                           shape_metadata=n.get("shape_metadata"))
        g.inputs, g.outputs = list(doc["inputs"]), list(doc["outputs"])
        arrays = make_inputs(doc["workload"], doc["dims"], seed=0)
        inputs = {nid: arrays[r] for r, nid in doc["roles"].items()}
        og = O.load_graph(case)

        def ref():
            evaluate_graph(g, dict(inputs), backend=numpy_backend)

        def port():
            O.evaluate(og, dict(inputs))

        res = {}
        for name, fn in (("reference", ref), ("port", port)):
            fn()
            ts = []
            for _ in range(args.samples):
                t0 = time.perf_counter()
                fn()
                ts.append(time.perf_counter() - t0)
            res[name] = statistics.median(ts)
        print(f"{case}: reference evaluate_graph {res['reference']:.3f} s, port {res['port']:.3f} s, "
              f"port / reference time {res['port'] / res['reference']:.3f} (median of {args.samples})", flush=True)


if __name__ == "__main__":
    main()

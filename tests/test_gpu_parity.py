"""Whole-graph parity: every golden case (fwd+bwd graph traced and differentiated by the
reference, evaluated by the reference numpy backend) run on the b200 backend.

Tolerances (written per workload): fp32 workloads rtol 1e-4 of each output's max
magnitude; bf16-math workloads rtol 2e-2; integer outputs (argmax) bit-exact.
"""

import numpy as np
import pytest

from gpu_helpers import assert_close, run_case

CASES = ["mlp_small", "mlp_ragged", "rowfused_small", "rowfused_ragged", "bmm_small", "cnn_small", "transformer_small"]
RTOL = {"mlp": 1e-4, "rowfused": 1e-4, "bmm": 2e-2, "cnn": 2e-2, "transformer": 2e-2}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["pernode", "graph", "compiled"])
@pytest.mark.parametrize("case", CASES)
def test_graph_parity(cuda, case, mode):
    got, ref, g = run_case(case, mode)
    rtol = RTOL[g.meta["workload"]]
    for name, r in ref.items():
        if name == "argmax":
            # bit-exact index output: compare on the same y the kernel produced
            y = got["y"].float().cpu().numpy()
            am = got["argmax"].cpu().numpy()
            np.testing.assert_array_equal(am, np.argmax(y, axis=-1))
            np.testing.assert_array_equal(am, r)
            continue
        assert_close(f"{case}:{name}", got[name], r, rtol)

"""Whole-graph parity: every golden case (fwd+bwd graph traced and differentiated by the
reference, evaluated by the reference numpy backend) run on the b200 backend.

ReLU decisions: a pre-activation within rounding of zero may be classified either way by
two correct evaluations, and each flip moves a whole weight-gradient row by a discrete
term. For the bf16 comparison the backend's own masks are replayed into the oracle, which
checks that they differ from its own only where |pre-activation| <= 1e-2 x its RMS.

Tolerances (written per workload; elementwise, ``gpu_helpers.assert_close``):
* fp32 workloads (mlp, rowfused, the node-type cases): rtol 1e-4 per element, absolute
  floor 1e-4 x the output's RMS, against the reference golden vectors; integer outputs
  (argmax) bit-exact.
* bf16-math workloads (bmm, cnn, transformer): rtol 2e-2 per element, absolute floor
  2e-2 x the output's RMS or twice the largest difference bf16 operand rounding itself
  makes to that output, whichever is larger, plus an RMS bound of twice the rounding's
  RMS effect (``gpu_helpers.bf16_report`` says why), against the oracle evaluated under
  the same bf16 operand-rounding policy (contraction operands rounded to bf16, fp32
  accumulation).
  Outputs that are zero in exact arithmetic (the attention key-bias gradients: softmax
  is invariant to a per-row shift) are rounding noise, so their floor is 1e-3 of the
  largest output instead. Against the pure-fp32 reference golden the norm-wise relative
  error must stay within 0.1 (bf16 rounding alone gives up to 0.057 on the
  cancellation-heavy first-conv weight gradient at batch 4).
"""

import numpy as np
import pytest
import torch

from gpu_helpers import assert_close, bf16_report, check_decisions, gpu_decisions, run_case, to_np

CASES = ["mlp_small", "mlp_ragged", "rowfused_small", "rowfused_ragged", "bmm_small", "cnn_small", "transformer_small",
         # node types outside the workloads: the reference's fusion-pass outputs (golden = the
         # reference's evaluation of the graph before fusion) and the interpreter's indexing /
         # Recompute / Checkpoint nodes plus Gather and OneHot (tests/golden/make_node_golden.py)
         "nodes_fused_ew", "nodes_fused_act", "nodes_fused_conv", "nodes_fused_horizontal", "nodes_fused_full",
         "nodes_indexing"]
RTOL = {"mlp": 1e-4, "rowfused": 1e-4, "bmm": 2e-2, "cnn": 2e-2, "transformer": 2e-2, "nodes": 1e-4}
BF16 = {"bmm", "cnn", "transformer"}


def _exact_zero(name: str) -> bool:
    """Gradients that vanish in exact arithmetic: the attention key bias (softmax over the
    key axis is invariant to adding the same q.bk to every score of a row)."""
    return name.startswith("d_") and name.endswith("_bk")


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["pernode", "graph", "compiled", "compiled_host"])
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
        if g.meta["workload"] in BF16:
            continue
        assert_close(f"{case}:{name}", got[name], r, rtol)
    if g.meta["workload"] in BF16:
        from conftest import load_golden
        from oracle import evaluator as O

        ins, _ = load_golden(case)
        # the backend's ReLU decisions replayed into the oracle (checked to differ from the
        # oracle's own only at |pre-activation| ~ 0); every other value is the oracle's own
        dev_in = {nid: torch.from_numpy(np.ascontiguousarray(ins[r])).cuda() for r, nid in g.roles.items()}
        rep: list = []
        dec = gpu_decisions(g, dev_in)
        emu = O.evaluate_roles(O.load_graph(case), ins, contraction_rounding="bf16", decisions=dec, decision_report=rep)
        check_decisions(rep)
        emu32 = O.evaluate_roles(O.load_graph(case), ins, decisions=dec)  # without the bf16 rounding
        # outputs that are zero in exact arithmetic (e.g. the key-bias gradient of softmax
        # attention) are compared against an absolute floor: 1e-3 of the largest output
        floor = 1e-3 * max(float(np.abs(np.asarray(v)).max()) for v in emu.values() if np.asarray(v).size)
        for name, r in ref.items():
            e = np.asarray(emu[name], dtype=np.float32)
            msg = bf16_report(f"{case}:{name}(bf16 policy)", got[name], e, np.asarray(emu32[name], dtype=np.float32), rtol,
                              floor=floor if _exact_zero(name) else 0.0)
            assert msg is None, msg
            v = to_np(got[name]).astype(np.float64)
            nrel = np.linalg.norm(v - r) / max(np.linalg.norm(r), floor * np.sqrt(r.size), 1e-30)
            assert nrel <= 0.1, (name, nrel)

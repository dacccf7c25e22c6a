"""Oracle parity at the benchmark sizes.

Each case keeps every full-size dimension of its workload and at most shrinks the batch
to one data-parallel rank's shard, so the kernel variants the benchmark selects are the
ones checked:

* ``rowfused_full``: x[8192, 4096], the whole fwd+bwd graph, including the column
  gradients d_a / d_b (sums over all 8192 rows) and the 8192 argmax indices;
* ``bmm_z2``: two of the sixteen [2048, 2048] batch matrices (the two-rank shard);
* ``cnn_n64``: 64 images of [3, 32, 32] (the eight-rank shard);
* ``transformer_b8``: 8 sequences of 512 tokens, d 1024, 16 heads, FFN 4096, vocab 32000
  (the eight-rank shard): the 32000-wide cross-entropy rows, the 512-wide attention
  softmax and the large-N GEMM tiles of the full model.

Every output is compared element by element with the CPU oracle on the same seeded
inputs (``gpu_helpers.close_report``): fp32 graphs at rtol 1e-4, bf16-math graphs at rtol
2e-2 against the oracle run with the same bf16 operand rounding, each with an absolute
floor of rtol x the RMS of the output's non-zero entries, raised for the bf16 graphs to
twice the largest difference bf16 operand rounding itself makes to that output (the
oracle run with and without the rounding), together with an RMS bound of twice the
rounding's RMS effect (``gpu_helpers.bf16_report`` says why); argmax bit-exact. The
backend's ReLU VJP masks are replayed into the oracle, which checks that they differ
from its own only at |pre-activation| <= 1e-2 x RMS (a pre-activation within rounding of
zero may be classified either way, and each flip moves a whole weight-gradient row). The attention key-bias gradients are
zero in exact arithmetic (softmax is invariant to a per-row shift of its scores), so both
sides hold rounding noise there; they are held to an absolute floor of 1e-3 x the largest
output instead. The oracle runs its contractions through a batched CPU BLAS
(``blas_layout=True``), which changes only fp32 summation order.
"""

import gc

import numpy as np
import pytest
import torch

from gpu_helpers import bf16_report, check_decisions, close_report, gpu_decisions, set_policy, to_np

pytestmark = pytest.mark.gpu

CASES = [("rowfused_full", 1e-4, None), ("bmm_z2", 2e-2, "bf16"), ("cnn_n64", 2e-2, "bf16"),
         ("transformer_b8", 2e-2, "bf16")]


def _exact_zero(name: str) -> bool:
    return name.startswith("d_") and name.endswith("_bk")


@pytest.mark.parametrize("case,rtol,rounding", CASES)
def test_fullsize_outputs_match_oracle(cuda, case, rtol, rounding):
    from b200 import graph as G
    from b200.backend import B200Backend
    from b200.workloads import make_inputs
    from oracle import evaluator as O

    g = G.load(case)
    set_policy(g.meta["workload"])
    arrays = make_inputs(g.meta["workload"], g.meta["dims"], seed=0)
    inputs = {nid: torch.from_numpy(np.ascontiguousarray(arrays[r])).cuda() for r, nid in g.roles.items()}
    res = B200Backend.execute_graph(g, inputs)
    torch.cuda.synchronize()
    got = {name: to_np(res[nid]) for name, nid in g.output_names.items()}
    del res
    decisions = gpu_decisions(g, inputs)  # the ReLU VJP masks, replayed into the oracle
    del inputs
    gc.collect()
    torch.cuda.empty_cache()

    rep: list = []
    ref = O.evaluate_roles(O.load_graph(case), arrays, contraction_rounding=rounding, blas_layout=True, decisions=decisions,
                           decision_report=rep)
    check_decisions(rep)
    assert set(ref) == set(got)
    ref32 = None
    if rounding:  # the same graph without bf16 operand rounding: the size of the rounding's own effect
        ref32 = O.evaluate_roles(O.load_graph(case), arrays, blas_layout=True, decisions=decisions)
    floor = 1e-3 * max(float(np.abs(np.asarray(v)).max()) for v in ref.values() if np.asarray(v).size)
    problems = []
    for name, r in ref.items():
        r = np.asarray(r)
        if r.dtype == np.float64:  # Python-float constants promote a scalar loss to float64
            r = r.astype(np.float32)
        fl = floor if _exact_zero(name) else 0.0
        if ref32 is not None and r.dtype.kind == "f":
            msg = bf16_report(f"{case}:{name}", got[name], r, np.asarray(ref32[name], dtype=np.float32), rtol, floor=fl)
        else:
            msg = close_report(f"{case}:{name}", got[name], r, rtol, floor=fl)
        if msg:
            problems.append(msg)
    assert not problems, f"{len(problems)} of {len(ref)} outputs outside tolerance:\n" + "\n".join(problems)

"""The CPU oracle restates the reference's evaluate_graph + numpy kernels.

Pinned two ways: (1) against golden vectors produced by running the reference's own
``evaluate_graph`` on the numpy backend (``tests/golden/make_golden.py``), on every
stored case; (2) against the reference's known-answer tests for ops on this path
(``tests/backends/test_hardware_parity.py:164-205``,
``tests/interpreter/test_evaluator.py:66-100``,
``tests/distributed/test_multi_process_collectives.py:83-103``).
"""

import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from oracle import evaluator as O

CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_golden(case):
    ins, outs = load_golden(case)
    g = O.load_graph(case)
    res = O.evaluate_roles(g, ins)
    assert set(res) == set(outs)
    for k, ref in outs.items():
        v = np.asarray(res[k])
        assert v.shape == ref.shape and v.dtype == ref.dtype, (k, v.shape, ref.shape, v.dtype, ref.dtype)
        if ref.dtype.kind in "iub":
            np.testing.assert_array_equal(v, ref)
        else:
            # bit-identical except conv (summation order of the per-tap einsum differs) and
            # FusedElementwise (float32 C-expression arithmetic against the unfused numpy ops)
            tol = 1e-6 * max(1.0, float(np.abs(ref).max()))
            assert float(np.abs(v.astype(np.float64) - ref).max()) <= tol, k


def test_known_answers_from_reference_tests():
    a = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    b = np.array([[0.5, -0.5], [1.5, 0.0]], np.float32)
    np.testing.assert_allclose(O.execute_op("MatMul", a, b), a @ b, rtol=1e-5, atol=1e-5)
    x = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    np.testing.assert_allclose(O.execute_op("ReduceSum", x, axis=-1, keepdims=True), [[3.0], [7.0]])
    np.testing.assert_allclose(O.execute_op("ReduceMean", x, axis=-1, keepdims=True), [[1.5], [3.5]])
    xa = np.array([-2.0, -1.0, 0.0, 1.0, 2.0], np.float32)
    np.testing.assert_allclose(O.execute_op("Tanh", xa), np.tanh(xa), rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(O.execute_op("Relu", np.array([-1.0, 2.0])), [0.0, 2.0])
    np.testing.assert_array_equal(
        O.execute_op("Where", np.array([True, False]), np.array([1.0, 2.0]), np.array([3.0, 4.0])), [1.0, 4.0]
    )


def test_allreduce_semantics_sum_over_ranks():
    # 4 ranks holding [r+1, 2(r+1)] sum to [10, 20]
    parts = [np.array([r + 1.0, 2.0 * (r + 1)], np.float32) for r in range(4)]
    np.testing.assert_allclose(np.sum(parts, axis=0), [10.0, 20.0])


def test_oracle_unknown_op_raises():
    g = {"name": "t", "inputs": ["a"], "outputs": ["b"],
         "nodes": [{"id": "a", "op_type": "Input", "inputs": []}, {"id": "b", "op_type": "UnknownOp", "inputs": ["a"]}]}
    with pytest.raises(O.UnimplementedOp):
        O.evaluate(g, {"a": np.zeros(2, np.float32)})


def test_oracle_cycle_detected():
    g = {"name": "t", "inputs": [], "outputs": ["b"],
         "nodes": [{"id": "a", "op_type": "Relu", "inputs": ["b"]}, {"id": "b", "op_type": "Relu", "inputs": ["a"]}]}
    with pytest.raises(ValueError):
        O.topo_order(g)


def test_argmax_first_max_wins():
    x = np.array([[1.0, 3.0, 3.0, 0.0], [2.0, 2.0, 2.0, 2.0]], np.float32)
    np.testing.assert_array_equal(O.execute_op("Argmax", x, axis=-1), [1, 0])


def _optim_cases():
    import os

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ops", "optim.npz"))
    ops = sorted({k.split("/")[0] for k in z.files})
    for op in ops:
        k = 0
        while f"{op}/{k}/in0" in z.files:
            ins = [z[f"{op}/{k}/in{j}"] for j in range(4) if f"{op}/{k}/in{j}" in z.files]
            outs = [z[f"{op}/{k}/out{j}"] for j in range(3) if f"{op}/{k}/out{j}" in z.files]
            kw = {"lr": float(z[f"{op}/{k}/lr"])} if f"{op}/{k}/lr" in z.files else {}
            yield op, k, ins, outs, kw
            k += 1


def test_oracle_optimizer_steps_match_reference_bit_exact():
    """ApplyAdam / Adagrad / Ftrl / RMSProp restatements against the reference numpy
    backend's own outputs (tests/golden/make_optim_golden.py): bit-identical."""
    from oracle import evaluator as O

    seen = set()
    for op, k, ins, outs, kw in _optim_cases():
        res = O.execute_op(op, *ins, **kw)
        assert len(res) == len(outs)
        for r, ref in zip(res, outs):
            assert r.dtype == np.float32
            np.testing.assert_array_equal(r, ref, err_msg=f"{op} case {k}")
        seen.add(op)
    assert seen == {"ApplyAdam", "ApplyAdagrad", "ApplyFtrl", "ApplyRMSProp"}

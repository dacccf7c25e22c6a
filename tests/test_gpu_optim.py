"""Optimizer update steps on the GPU (``b200_apply_optimizer_f32``), bit-exact against the
reference numpy backend's outputs (``tests/golden/ops/optim.npz``) and against the oracle on
larger, ragged and misaligned tensors; several tensors per launch and in-place updates."""

import os

import numpy as np
import pytest
import torch

from gpu_helpers import to_np

pytestmark = pytest.mark.gpu

OPS = ("ApplyAdam", "ApplyAdagrad", "ApplyFtrl", "ApplyRMSProp")


def _golden():
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ops", "optim.npz"))
    for op in OPS:
        k = 0
        while f"{op}/{k}/in0" in z.files:
            ins = [z[f"{op}/{k}/in{j}"] for j in range(4) if f"{op}/{k}/in{j}" in z.files]
            outs = [z[f"{op}/{k}/out{j}"] for j in range(3) if f"{op}/{k}/out{j}" in z.files]
            kw = {"lr": float(z[f"{op}/{k}/lr"])} if f"{op}/{k}/lr" in z.files else {}
            yield op, k, ins, outs, kw
            k += 1


def test_optimizer_steps_bit_exact_against_reference_goldens(cuda):
    from b200.backend import B200Backend

    n = 0
    for op, k, ins, outs, kw in _golden():
        res = B200Backend.execute_op(op, *ins, **kw)  # numpy operands: copied to the device
        assert len(res) == len(outs)
        for r, ref in zip(res, outs):
            np.testing.assert_array_equal(to_np(r), ref, err_msg=f"{op} case {k}")
        n += 1
    assert n == 16


@pytest.mark.parametrize("op", OPS)
def test_optimizer_multi_tensor_in_place_matches_oracle(cuda, op):
    from b200 import ops
    from oracle import evaluator as O

    rng = np.random.default_rng(5)
    nst = 1 if op == "ApplyAdagrad" else 2
    sizes = [1, 7, 4096, 1 << 20, 12345]
    host = []
    for s in sizes:
        p, g = rng.standard_normal(s).astype(np.float32), rng.standard_normal(s).astype(np.float32)
        st = [np.abs(rng.standard_normal(s)).astype(np.float32) * np.float32(0.1) for _ in range(nst)]
        host.append((p, st, g))
    # device copies, the third one at a 4-byte offset (scalar path)
    def dev(a, off):
        buf = torch.zeros(a.size + off, device="cuda")
        buf[off:] = torch.from_numpy(a).cuda()
        return buf[off:]
    params = [dev(p, 1 if i == 2 else 0) for i, (p, _, _) in enumerate(host)]
    states = [tuple(dev(x, 0) for x in st) for _, st, _ in host]
    grads = [dev(g, 0) for _, _, g in host]
    out = [(p,) + s for p, s in zip(params, states)]  # in place
    ops.apply_optimizer(op, params, states, grads, lr=0.02, out=out)
    torch.cuda.synchronize()
    for (p, st, g), o in zip(host, out):
        ref = O.execute_op(op, p, *st, g, lr=0.02)
        for r, x in zip(ref, o):
            np.testing.assert_array_equal(to_np(x), r)

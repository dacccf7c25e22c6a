"""Kernel-level checks through the C ABI against numpy / fp32 references, including the
edge cases: empty and ragged sizes, broadcasting, strided views, ties, bf16 tensor-core
GEMM in every operand layout."""

import numpy as np
import pytest
import torch

from gpu_helpers import to_np

pytestmark = pytest.mark.gpu


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(autouse=True)
def _policy(cuda):
    from b200 import ops

    ops.Config.matmul_dtype = "f32"
    ops.Config.conv_dtype = "f32"
    yield


def rng(seed=0):
    return np.random.default_rng(seed)


def test_elementwise_broadcast_and_chain():
    from b200 import ops

    r = rng()
    x = r.standard_normal((33, 17), dtype=np.float32)
    col = r.standard_normal(17, dtype=np.float32)
    row = r.standard_normal((33, 1), dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_add(T(x), T(col))), x + col, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_multiply(T(x), T(row))), x * row, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_subtract(T(x), 0.5)), x - 0.5, rtol=1e-6)
    np.testing.assert_array_equal(to_np(ops.op_greater(T(x), 0.0)), x > 0)
    np.testing.assert_allclose(to_np(ops.op_gelu(T(x))), 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x**3))), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_exp(T(x))), np.exp(x), rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_tanh(T(x))), np.tanh(x), rtol=1e-5, atol=1e-7)
    # transposed (strided) view input
    xt = T(x).t()
    np.testing.assert_allclose(to_np(ops.op_add(xt, 1.0)), x.T + 1.0, rtol=1e-6)
    # bool * float
    m = x > 0
    np.testing.assert_allclose(to_np(ops.op_multiply(T(x), T(m))), x * m, rtol=1e-6)
    # empty
    assert to_np(ops.op_add(T(np.zeros((0, 5), np.float32)), 1.0)).shape == (0, 5)
    # scalar (0-d) tensors
    np.testing.assert_allclose(to_np(ops.op_multiply(T(np.array(2.0, np.float32)), T(x))), 2 * x)


def test_reductions_axes_and_split():
    from b200 import ops

    r = rng(1)
    x = r.standard_normal((7, 300, 5), dtype=np.float32)
    for axis in (None, 0, 1, 2, -1, (0, 1), (1, 2), (0, 2)):
        for kd in (False, True):
            got = to_np(ops.op_reduce_sum(T(x), axis=axis, keepdims=kd))
            np.testing.assert_allclose(got, np.sum(x, axis=axis, keepdims=kd), rtol=1e-5, atol=1e-4)
            got = to_np(ops.op_reduce_mean(T(x), axis=axis, keepdims=kd))
            np.testing.assert_allclose(got, np.mean(x, axis=axis, keepdims=kd), rtol=1e-5, atol=1e-5)
            got = to_np(ops.op_reduce_max(T(x), axis=axis, keepdims=kd))
            np.testing.assert_array_equal(got, np.max(x, axis=axis, keepdims=kd))
    # short rows (8 lanes per row), a partial last warp, a bf16 source
    z = r.standard_normal((1001, 36), dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_reduce_mean(T(z), axis=-1)), z.mean(-1), rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(to_np(ops.op_reduce_max(T(z), axis=-1)), z.max(-1))
    zb = T(z).to(torch.bfloat16)
    np.testing.assert_allclose(to_np(ops.op_reduce_sum(zb, axis=-1)), to_np(zb.float()).sum(-1), rtol=1e-5, atol=1e-5)
    # column reduction with many rows (split + atomics path)
    y = r.standard_normal((8192, 64), dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_reduce_sum(T(y), axis=0)), y.sum(0), rtol=1e-4, atol=1e-3)
    np.testing.assert_array_equal(to_np(ops.op_reduce_max(T(y), axis=0)), y.max(0))
    b = r.standard_normal(64, dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_broadcast_reduce(T(y), T(b))), y.sum(0), rtol=1e-4, atol=1e-3)


def test_argmax_ties_first_and_exact():
    from b200 import ops

    x = np.array([[1.0, 3.0, 3.0, 0.0], [2.0, 2.0, 2.0, 2.0], [-1.0, -5.0, -1.0, -0.5]], np.float32)
    np.testing.assert_array_equal(to_np(ops.op_argmax(T(x), axis=-1)), np.argmax(x, -1))
    r = rng(2)
    big = r.standard_normal((300, 4097), dtype=np.float32)
    big[:, 4096] = big.max(1)  # tie with an earlier max -> earlier index wins
    np.testing.assert_array_equal(to_np(ops.op_argmax(T(big), axis=-1)), np.argmax(big, -1))
    np.testing.assert_array_equal(to_np(ops.op_argmax(T(big), axis=0)), np.argmax(big, 0))
    assert int(to_np(ops.op_argmax(T(big)))) == int(np.argmax(big))


@pytest.mark.parametrize("cols", [1, 10, 1000, 4096, 32000])
def test_softmax_logsoftmax(cols):
    from b200 import ops

    r = rng(3)
    x = (r.standard_normal((5, cols)) * 3).astype(np.float32)
    e = np.exp(x - x.max(-1, keepdims=True))
    np.testing.assert_allclose(to_np(ops.op_softmax(T(x))), e / e.sum(-1, keepdims=True), rtol=1e-5, atol=1e-7)
    ls = x - x.max(-1, keepdims=True) - np.log(e.sum(-1, keepdims=True))
    np.testing.assert_allclose(to_np(ops.op_log_softmax(T(x))), ls, rtol=1e-5, atol=1e-5)
    if cols > 1:
        np.testing.assert_allclose(to_np(ops.op_softmax(T(x), axis=0)), np.exp(x) / np.exp(x).sum(0), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("cols", [7, 1024, 4096])
def test_layernorm_fwd_and_grads(cols):
    from b200 import ops
    from oracle import evaluator as O

    r = rng(4)
    x = r.standard_normal((37, cols), dtype=np.float32)
    g = r.uniform(0.5, 1.5, cols).astype(np.float32)
    b = r.standard_normal(cols, dtype=np.float32)
    dy = r.standard_normal((37, cols), dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_layer_norm(T(x), T(g), T(b), eps=1e-5)), O.execute_op("LayerNorm", x, g, b, eps=1e-5), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(to_np(ops.op_layer_norm_input_grad(T(dy), T(x), T(g), eps=1e-5)),
                               O.execute_op("LayerNormInputGrad", dy, x, g, eps=1e-5), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(to_np(ops.op_layer_norm_gamma_grad(T(dy), T(x), eps=1e-5)),
                               O.execute_op("LayerNormGammaGrad", dy, x, eps=1e-5), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(to_np(ops.op_layer_norm_beta_grad(T(dy))), O.execute_op("LayerNormBetaGrad", dy), rtol=1e-4, atol=1e-4)


def test_indexing_ops():
    from b200 import ops
    from oracle import evaluator as O

    r = rng(5)
    x = r.standard_normal((9, 10), dtype=np.float32)
    idx = r.integers(0, 10, (9, 1))
    np.testing.assert_array_equal(to_np(ops.op_take_along_axis(T(x), T(idx), axis=-1)), np.take_along_axis(x, idx, -1))
    src = r.standard_normal((9, 1), dtype=np.float32)
    z = np.zeros_like(x)
    np.testing.assert_allclose(to_np(ops.op_scatter_add(T(z), T(idx), T(src), dim=-1)), O.execute_op("ScatterAdd", z, idx, src, dim=-1))
    # repeated index within a row keeps the last write, like put_along_axis
    idx2 = np.array([[3, 3]] * 9)
    src2 = r.standard_normal((9, 2), dtype=np.float32)
    np.testing.assert_allclose(to_np(ops.op_scatter_add(T(x), T(idx2), T(src2), dim=-1)), O.execute_op("ScatterAdd", x, idx2, src2, dim=-1))
    table = r.standard_normal((50, 8), dtype=np.float32)
    ids = r.integers(0, 50, 200)
    np.testing.assert_array_equal(to_np(ops.op_take(T(table), T(ids), axis=0)), np.take(table, ids, axis=0))
    table6 = r.standard_normal((50, 6), dtype=np.float32)  # rows not a whole number of 16-byte groups
    np.testing.assert_array_equal(to_np(ops.op_take(T(table6), T(ids), axis=0)), np.take(table6, ids, axis=0))
    upd = r.standard_normal((200, 8), dtype=np.float32)
    ref = O.execute_op("TensorScatterAdd", np.zeros_like(table), ids.reshape(200, 1), upd)
    np.testing.assert_allclose(to_np(ops.op_tensor_scatter_add(T(np.zeros_like(table)), T(ids.reshape(200, 1)), T(upd))), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_fp32_layouts_and_epilogue(ta, tb):
    from b200 import _lib as L
    from b200 import ops

    r = rng(6)
    M, N, K = 70, 45, 33
    a = r.standard_normal((K, M) if ta else (M, K), dtype=np.float32)
    b = r.standard_normal((N, K) if tb else (K, N), dtype=np.float32)
    A = T(a).t() if ta else T(a)
    B = T(b).t() if tb else T(b)
    an, bn = (a.T if ta else a), (b.T if tb else b)
    np.testing.assert_allclose(to_np(ops.gemm(A, B)), an @ bn, rtol=1e-4, atol=1e-4)
    bias = r.standard_normal(N, dtype=np.float32)
    out, mask = ops.gemm(A, B, bias=T(bias), epilogue=L.EPI_RELU, want_mask=True)
    pre = an @ bn + bias
    np.testing.assert_allclose(to_np(out), np.maximum(pre, 0), rtol=1e-4, atol=1e-4)
    agree = to_np(mask) == (pre > 0)
    assert agree.mean() > 0.999


def _bf16(a):
    from b200.workloads import _bf16_round

    return _bf16_round(a)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("shape", [(128, 128, 64), (256, 512, 192), (200, 136, 72), (129, 257, 8)])
def test_gemm_bf16_tcgen05_layouts(ta, tb, shape):
    from b200 import ops

    M, N, K = shape
    r = rng(7)
    a = _bf16(r.standard_normal((K, M) if ta else (M, K), dtype=np.float32))
    b = _bf16(r.standard_normal((N, K) if tb else (K, N), dtype=np.float32))
    A = T(a).to(torch.bfloat16)
    B = T(b).to(torch.bfloat16)
    A = A.t() if ta else A
    B = B.t() if tb else B
    an, bn = (a.T if ta else a), (b.T if tb else b)
    ref = an.astype(np.float64) @ bn.astype(np.float64)
    got = to_np(ops.gemm(A, B, ab_dtype=torch.bfloat16))
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3 * np.sqrt(K))


@pytest.mark.parametrize("Z,M,N,K,ta,tb", [(2, 2048, 2048, 2048, False, False), (1, 1000, 1000, 320, True, False),
                                            (3, 512, 768, 64, False, True), (1, 4088, 1024, 1024, False, False)])
def test_gemm_bf16_cta_pairs_many_tiles(Z, M, N, K, ta, tb):
    """The CTA-pair kernel (256 x 256 tiles, M >= 256, N > 128) over many tiles per pair, a
    long K (the stage ring and both accumulators wrap many times), a single K block (direct
    stores), ragged M and N, and transposed operands; sampled rows against float64."""
    from b200 import ops

    r = rng(M + N + K + Z)
    a = _bf16(r.standard_normal((Z, K, M) if ta else (Z, M, K), dtype=np.float32) * 0.05)
    b = _bf16(r.standard_normal((Z, N, K) if tb else (Z, K, N), dtype=np.float32) * 0.05)
    A, B = T(a).to(torch.bfloat16), T(b).to(torch.bfloat16)
    A = A.transpose(-1, -2) if ta else A
    B = B.transpose(-1, -2) if tb else B
    an = np.swapaxes(a, -1, -2) if ta else a
    bn = np.swapaxes(b, -1, -2) if tb else b
    got = to_np(ops.gemm(A, B, ab_dtype=torch.bfloat16))
    rows = np.unique(np.concatenate([r.choice(M, 24, replace=False), [0, 127, 128, 255, 256, M - 1]]))
    for z in range(Z):
        ref = an[z, rows].astype(np.float64) @ bn[z].astype(np.float64)
        np.testing.assert_allclose(got[z, rows], ref, rtol=1e-4, atol=1e-4 * np.sqrt(K))


def test_gemm_bf16_batched_bias_relu_mask_bf16_out():
    from b200 import _lib as L
    from b200 import ops

    r = rng(8)
    Z, M, N, K = 3, 256, 384, 256
    a = _bf16(r.standard_normal((Z, M, K), dtype=np.float32) * 0.05)
    b = _bf16(r.standard_normal((Z, K, N), dtype=np.float32) * 0.05)
    bias = r.standard_normal(N, dtype=np.float32) * 0.02
    A, B = T(a).to(torch.bfloat16), T(b).to(torch.bfloat16)
    pre = np.matmul(a.astype(np.float64), b.astype(np.float64)) + bias
    out, mask = ops.gemm(A, B, bias=T(bias), epilogue=L.EPI_RELU, want_mask=True, ab_dtype=torch.bfloat16)
    np.testing.assert_allclose(to_np(out), np.maximum(pre, 0), rtol=1e-4, atol=1e-4)
    assert (to_np(mask) == (pre > 0)).mean() > 0.999
    o16 = ops.gemm(A, B, ab_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    np.testing.assert_allclose(to_np(o16), pre - bias, rtol=1e-2, atol=1e-2)
    # batched with transposed operands (the backward-pass layouts)
    g = _bf16(r.standard_normal((Z, M, N), dtype=np.float32))
    G = T(g).to(torch.bfloat16)
    dA = ops.gemm(G, B.transpose(-1, -2), ab_dtype=torch.bfloat16)
    np.testing.assert_allclose(to_np(dA), np.matmul(g, np.swapaxes(b, -1, -2)), rtol=1e-4, atol=1e-3)
    dB = ops.gemm(A.transpose(-1, -2), G, ab_dtype=torch.bfloat16)
    np.testing.assert_allclose(to_np(dB), np.matmul(np.swapaxes(a, -1, -2), g), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("padding,stride", [("VALID", 1), ("VALID", 2), ("SAME", 1), ("SAME", 2)])
def test_conv2d_fwd_dgrad_wgrad(padding, stride):
    from b200 import ops
    from oracle import evaluator as O

    r = rng(9)
    x = r.standard_normal((2, 5, 11, 10), dtype=np.float32)
    w = r.standard_normal((7, 5, 3, 3), dtype=np.float32)
    kw = dict(stride=[stride, stride], padding=padding)
    y_ref = O.execute_op("Conv2D", x, w, **kw)
    np.testing.assert_allclose(to_np(ops.op_conv2d(T(x), T(w), **kw)), y_ref, rtol=1e-4, atol=1e-4)
    dy = r.standard_normal(y_ref.shape, dtype=np.float32)
    dx_ref = O.execute_op("Conv2DInputGrad", dy, w, target_shape=list(x.shape), **kw)
    np.testing.assert_allclose(to_np(ops.op_conv2d_input_grad(T(dy), T(w), target_shape=list(x.shape), **kw)), dx_ref, rtol=1e-4, atol=1e-4)
    dw_ref = O.execute_op("Conv2DWeightGrad", x, dy, target_shape=list(w.shape), **kw)
    np.testing.assert_allclose(to_np(ops.op_conv2d_weight_grad(T(x), T(dy), target_shape=list(w.shape), **kw)), dw_ref, rtol=1e-4, atol=1e-3)


def test_unknown_op_raises_no_fallback():
    from b200 import B200Backend, UnimplementedMathError

    with pytest.raises(UnimplementedMathError):
        B200Backend.execute_op("NotARealOp", T(np.zeros(3, np.float32)))


def test_device_error_flag_for_bad_index():
    from b200 import _lib as L
    from b200 import ops

    x = T(np.zeros((2, 4), np.float32))
    bad = T(np.array([[1], [9]], np.int64))
    y = ops.op_take_along_axis(x, bad, axis=-1)  # out-of-range index: recorded, skipped
    rc = L.lib().b200_check_device_error(ops.stream_ptr())
    assert rc == L.ERR_ARG
    assert L.lib().b200_check_device_error(ops.stream_ptr()) == L.OK  # flag cleared
    del y


def test_mask_mul_colsum_bf16_and_f32():
    from b200 import _lib as L
    from b200 import ops

    r = rng(11)
    for R, C in ((37, 2048), (5, 13), (1000, 24)):
        g = r.standard_normal((R, C), dtype=np.float32)
        m = r.random((R, C)) > 0.5
        ref = g * m
        ws_b = int(L.lib().b200_mask_mul_colsum_workspace_bytes(R, C))
        ws = torch.empty(max(1, ws_b), dtype=torch.uint8, device="cuda")
        yb = torch.empty(R, C, dtype=torch.bfloat16, device="cuda")
        yf = torch.empty(R, C, dtype=torch.float32, device="cuda")
        cs = torch.empty(C, dtype=torch.float32, device="cuda")
        G, M = T(g), T(m)
        L.call("b200_mask_mul_colsum", G.data_ptr(), M.data_ptr(), yb.data_ptr(), yf.data_ptr(), cs.data_ptr(), R, C,
               ws.data_ptr(), ws_b, ops.stream_ptr())
        np.testing.assert_array_equal(to_np(yf), ref)
        np.testing.assert_allclose(to_np(yb), ref, rtol=8e-3, atol=1e-6)
        np.testing.assert_allclose(to_np(cs), ref.sum(0), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("R,V", [(7, 10), (64, 32000), (3, 1)])
def test_logsoftmax_pick_fwd_bwd(R, V):
    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O

    r = rng(12)
    x = (r.standard_normal((R, V)) * 3).astype(np.float32)
    lab = r.integers(0, V, (R, 1))
    d = r.standard_normal((R, 1)).astype(np.float32)
    ls = O.execute_op("LogSoftmax", x, axis=-1)
    picked_ref = O.execute_op("TakeAlongAxis", ls, lab, axis=-1)
    dls = O.execute_op("ScatterAdd", np.zeros_like(ls), lab, d, dim=-1)
    dx_ref = dls - np.exp(ls) * dls.sum(-1, keepdims=True)
    X, LB, D = T(x), T(lab), T(d)
    picked = torch.empty(R, 1, device="cuda")
    dx = torch.empty(R, V, device="cuda")
    lsd = torch.empty(R, V, device="cuda")
    L.call("b200_logsoftmax_pick", L.F32, X.data_ptr(), LB.data_ptr(), D.data_ptr(), picked.data_ptr(), lsd.data_ptr(),
           dx.data_ptr(), None, R, V, ops.stream_ptr())
    np.testing.assert_allclose(to_np(picked), picked_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(lsd), ls, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(dx), dx_ref, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("C,path,gb", [(4096, "shift", True), (4096, "general", True), (1000, "general", True),
                                       (77, "shift", True), (6000, "general", True), (4096, "shift", False),
                                       (4096, "general", False), (3000, "shift", False), (3000, "general", False),
                                       (2056, "general", False), (1000, "shift", False)])
def test_rowfused_kernel_both_softmax_paths(C, path, gb):
    """The fused row kernel against the oracle: gamma = 1 / beta = 0 takes the fixed-shift
    softmax path, signed gamma / wide beta the per-row max path; with and without the
    dgamma/dbeta accumulators, 4 / 8 columns per thread, whole and ragged rows."""
    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O

    r = rng(13)
    R = 37
    x = r.standard_normal((R, C), dtype=np.float32)
    a = r.uniform(0.5, 1.5, C).astype(np.float32)
    b = (r.standard_normal(C) * 0.1).astype(np.float32)
    if path == "shift":
        gamma, beta = np.ones(C, np.float32), np.zeros(C, np.float32)
    else:
        gamma = r.uniform(-1.5, 1.5, C).astype(np.float32)
        beta = r.standard_normal(C).astype(np.float32)  # signed gamma -> per-row max path
    cot = r.standard_normal((R, C), dtype=np.float32)
    g = O.execute_op("Gelu", x * a + b)
    n = O.execute_op("LayerNorm", g, gamma, beta, eps=1e-5)
    y = O.execute_op("Softmax", n, axis=-1)
    dn = y * (cot - (cot * y).sum(-1, keepdims=True))
    dg = O.execute_op("LayerNormInputGrad", dn, g, gamma, eps=1e-5)
    p = x * a + b
    k, c_ = np.sqrt(2 / np.pi), 0.044715
    t = np.tanh(k * (p + c_ * p**3))
    dp = dg * (0.5 * (1 + t) + 0.5 * p * (1 - t * t) * k * (1 + 3 * c_ * p * p))
    refs = {"y": y, "dx": dp * a, "da": (dp * x).sum(0), "db": dp.sum(0)}
    if gb:
        refs.update({"dgamma": O.execute_op("LayerNormGammaGrad", dn, g, eps=1e-5), "dbeta": dn.sum(0)})
    dev = "cuda"
    out = {k_: torch.empty(R, C, device=dev) for k_ in ("y", "dx")}
    out.update({k_: torch.empty(C, device=dev) for k_ in ("da", "db", "dgamma", "dbeta")})
    am = torch.empty(R, dtype=torch.int64, device=dev)
    wsb = int(L.lib().b200_rowfused_workspace_bytes(R, C))
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    ins = [T(v) for v in (x, a, b, gamma, beta, cot)]
    L.call("b200_rowfused_fwd_bwd", *[v.data_ptr() for v in ins], out["y"].data_ptr(), am.data_ptr(), out["dx"].data_ptr(),
           out["da"].data_ptr(), out["db"].data_ptr(), out["dgamma"].data_ptr() if gb else None,
           out["dbeta"].data_ptr() if gb else None, R, C, 1e-5, ws.data_ptr(), wsb, ops.stream_ptr())
    for k_, ref in refs.items():
        got = to_np(out[k_])
        scale = float(np.abs(ref).max())
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * scale, err_msg=k_)
    ygot = to_np(out["y"])
    np.testing.assert_array_equal(to_np(am), np.argmax(ygot, axis=-1))


@pytest.mark.parametrize("C", [4096, 3000])
def test_rowfused_argmax_ties_and_misaligned_rows(C):
    """argmax(y) takes the first of equal maxima: constant rows (every y equal -> 0), rows
    with the same peak value planted at two columns, and the same inputs through pointers
    offset by 4 bytes (scalar-load kernel) give identical results."""
    from b200 import _lib as L
    from b200 import ops

    r = rng(21)
    R = 64
    x = r.standard_normal((R, C), dtype=np.float32)
    x[0:4] = 0.25                            # constant rows
    for i in range(4, 16):                   # equal peak at two columns
        j1, j2 = sorted(r.choice(C, 2, replace=False))
        x[i, j1] = x[i, j2] = 9.0
    a, b = np.ones(C, np.float32), np.zeros(C, np.float32)
    gamma, beta = np.ones(C, np.float32), np.zeros(C, np.float32)
    cot = r.standard_normal((R, C), dtype=np.float32)

    def run(offset):
        def dev(v):
            flat = torch.zeros(v.size + offset, dtype=torch.float32, device="cuda")
            flat[offset:] = torch.from_numpy(np.ascontiguousarray(v).reshape(-1)).cuda()
            return flat[offset:].view(v.shape)
        ins = [dev(v) for v in (x, a, b, gamma, beta, cot)]
        y, dx = dev(np.zeros((R, C), np.float32)), dev(np.zeros((R, C), np.float32))
        da, db = torch.empty(C, device="cuda"), torch.empty(C, device="cuda")
        am = torch.empty(R, dtype=torch.int64, device="cuda")
        wsb = int(L.lib().b200_rowfused_workspace_bytes(R, C))
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        L.call("b200_rowfused_fwd_bwd", *[v.data_ptr() for v in ins], y.data_ptr(), am.data_ptr(), dx.data_ptr(),
               da.data_ptr(), db.data_ptr(), None, None, R, C, 1e-5, ws.data_ptr(), wsb, ops.stream_ptr())
        torch.cuda.synchronize()
        return to_np(y), to_np(am), to_np(dx), to_np(da), to_np(db)

    y0, am0, dx0, da0, db0 = run(0)
    np.testing.assert_array_equal(am0, np.argmax(y0, axis=-1))
    assert (am0[0:4] == 0).all()
    y1, am1, dx1, da1, db1 = run(1)
    np.testing.assert_array_equal(am1, np.argmax(y1, axis=-1))
    for got, ref in ((y1, y0), (dx1, dx0), (da1, da0), (db1, db0)):
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * float(np.abs(ref).max()))


@pytest.mark.parametrize("N,C,H,O,k,stride,padding", [(2, 3, 32, 64, 3, 1, "VALID"), (3, 64, 30, 64, 3, 2, "VALID"),
                                                      (2, 64, 14, 128, 3, 2, "VALID"), (2, 5, 11, 7, 3, 2, "SAME"),
                                                      (3, 9, 13, 300, 5, 3, "SAME"), (2, 16, 9, 24, 4, 1, "SAME"),
                                                      (2, 8, 12, 16, 3, 3, "SAME"), (1, 240, 6, 8, 3, 1, "VALID"),
                                                      (1, 2, 10, 3, 1, 2, "VALID"), (1, 2, 9, 3, 2, 4, "SAME"),
                                                      (2, 64, 13, 64, 3, 1, "SAME"), (5, 128, 6, 64, 3, 1, "VALID")])
def test_conv2d_tensor_core_path(N, C, H, O, k, stride, padding):
    """bf16 tcgen05 convolutions against the oracle with the same operand rounding: the
    implicit GEMM (several column tiles at O = 300, strides 1-4, SAME padding with
    even and odd kernels, strides above the kernel size so that some input pixels get no
    gradient; with 64-channel blocks the tiles come in as TMA boxes, several images per
    tile when the images are small) and, above 2048 taps x channels (C = 240, 3 x 3), the
    GEMM over staged operands."""
    from b200 import ops
    from oracle import evaluator as O_

    r = rng(14)
    x = r.standard_normal((N, C, H, H), dtype=np.float32)
    w = (r.standard_normal((O, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    kw = dict(stride=[stride, stride], padding=padding)
    ops.Config.conv_dtype = "bf16"
    try:
        y = ops.op_conv2d(T(x), T(w), **kw)
        y_ref = O_.execute_op("Conv2D", x, w, contraction_rounding="bf16", **kw)
        np.testing.assert_allclose(to_np(y), y_ref, rtol=1e-3, atol=1e-3 * np.abs(y_ref).max())
        dy = r.standard_normal(y_ref.shape, dtype=np.float32)
        dx = ops.op_conv2d_input_grad(T(dy), T(w), target_shape=list(x.shape), **kw)
        dx_ref = O_.execute_op("Conv2DInputGrad", dy, w, target_shape=list(x.shape), contraction_rounding="bf16", **kw)
        np.testing.assert_allclose(to_np(dx), dx_ref, rtol=1e-3, atol=1e-3 * np.abs(dx_ref).max())
        dw = ops.op_conv2d_weight_grad(T(x), T(dy), target_shape=list(w.shape), **kw)
        dw_ref = O_.execute_op("Conv2DWeightGrad", x, dy, target_shape=list(w.shape), contraction_rounding="bf16", **kw)
        np.testing.assert_allclose(to_np(dw), dw_ref, rtol=1e-3, atol=2e-3 * np.abs(dw_ref).max())
    finally:
        ops.Config.conv_dtype = "f32"


@pytest.mark.parametrize("N,C,H,O,stride,padding", [(4, 3, 32, 64, 1, "VALID"), (3, 64, 30, 64, 2, "VALID"),
                                                    (2, 64, 14, 128, 2, "VALID"), (2, 6, 10, 20, 2, "SAME")])
def test_conv2d_fused_epilogues(N, C, H, O, stride, padding):
    """Implicit-GEMM convolution epilogues: relu(Conv2D) from the forward kernel, and
    Conv2DInputGrad * (pre > 0) from the input-gradient kernel, against the oracle's
    bf16-operand convolutions followed by the same elementwise ops. The forward with the
    epilogue also equals the unfused forward then Relu, bit for bit."""
    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O_

    r = rng(15)
    x = r.standard_normal((N, C, H, H), dtype=np.float32)
    w = (r.standard_normal((O, C, 3, 3)) * np.sqrt(2.0 / (C * 9))).astype(np.float32)
    kw = dict(stride=[stride, stride], padding=padding)
    ops.Config.conv_dtype = "bf16"
    try:
        n0 = L.launch_count()
        y = ops.op_conv2d(T(x), T(w), relu=True, **kw)
        # the bf16 channels-last copy of x, the packed bf16 weights, the implicit GEMM
        assert L.launch_count() - n0 == 3
        # the epilogue's channels-last bf16 copy of relu(y) (kept for the next convolution)
        # equals a fresh copy of y, padding channels included
        cp = (O + 7) // 8 * 8
        twin = ops.channels_last(y, cp)
        fresh = torch.empty_like(twin)
        L.call("b200_conv2d_channels_last", y.data_ptr(), fresh.data_ptr(), y.shape[0], O, y.shape[2] * y.shape[3], cp,
               ops.stream_ptr())
        assert torch.equal(twin, fresh)
        y_plain = ops.op_conv2d(T(x), T(w), **kw)
        assert torch.equal(y, torch.where(y_plain > 0, y_plain, torch.zeros_like(y_plain)))
        pre = O_.execute_op("Conv2D", x, w, contraction_rounding="bf16", **kw)
        ref = np.maximum(pre, 0)
        np.testing.assert_allclose(to_np(y), ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())
        # the input gradient masked by a pre-activation of the input's shape
        dy = r.standard_normal(pre.shape, dtype=np.float32)
        m = r.standard_normal(x.shape, dtype=np.float32)
        dx = ops.op_conv2d_input_grad(T(dy), T(w), target_shape=list(x.shape), mask=T(m), **kw)
        dx_ref = O_.execute_op("Conv2DInputGrad", dy, w, target_shape=list(x.shape), contraction_rounding="bf16", **kw)
        dx_ref = dx_ref * (m > 0)
        np.testing.assert_allclose(to_np(dx), dx_ref, rtol=1e-3, atol=1e-3 * np.abs(dx_ref).max())
        assert (to_np(dx)[m <= 0] == 0).all()
        cpx = (C + 7) // 8 * 8
        twin = ops.channels_last(dx, cpx)
        fresh = torch.empty_like(twin)
        L.call("b200_conv2d_channels_last", dx.data_ptr(), fresh.data_ptr(), N, C, H * H, cpx, ops.stream_ptr())
        assert torch.equal(twin, fresh)
    finally:
        ops.Config.conv_dtype = "f32"


def test_conv2d_implicit_gemm_bounds():
    """Shapes the implicit GEMM does not take are reported (2048 reduction indices at most,
    channels padded to a multiple of 8),
    and a fused epilogue for them raises instead of running anything else."""
    from b200 import _lib as L
    from b200 import ops
    from b200.errors import UnimplementedMathError

    lib = L.lib()
    assert lib.b200_conv2d_igemm_supported(0, 2, 224, 8, 8, 16, 3, 3, 6, 6, 1, 1, 0, 0) == 1  # 2016 reduction indices
    assert lib.b200_conv2d_igemm_supported(0, 2, 228, 8, 8, 16, 3, 3, 6, 6, 1, 1, 0, 0) == 0  # 232 padded x 9 = 2088
    assert lib.b200_conv2d_igemm_supported(1, 2, 16, 8, 8, 228, 3, 3, 6, 6, 1, 1, 0, 0) == 0  # dgrad: O x taps
    assert lib.b200_conv2d_igemm_supported(2, 2, 228, 8, 8, 16, 3, 3, 6, 6, 1, 1, 0, 0) == 0  # wgrad: C x taps
    ops.Config.conv_dtype = "bf16"
    try:
        x = torch.zeros(1, 228, 8, 8, device="cuda")
        w = torch.zeros(4, 228, 3, 3, device="cuda")
        with pytest.raises(UnimplementedMathError):
            ops.op_conv2d(x, w, stride=[1, 1], padding="VALID", relu=True)
        assert ops.op_conv2d(x, w, stride=[1, 1], padding="VALID").shape == (1, 4, 6, 6)  # staged GEMM path
    finally:
        ops.Config.conv_dtype = "f32"


@pytest.mark.parametrize("shape", [((300, 256), (256, 384), True), ((4, 64, 128), (128, 200), True),
                                   ((512, 1024), (1024, 1024), False)])
def test_gemm_residual_epilogue_matches_separate_add(shape):
    """(a.b + bias) + r from the GEMM epilogue is bit-identical to the GEMM with its bias
    followed by a separate Add (the same two fp32 roundings), for single-CTA and CTA-pair
    tiles, a ragged N, a folded batch and no bias; the planner's pattern picks it up."""
    from b200 import ops

    (sa, sb, with_bias) = shape
    r = rng(sum(sa) + sum(sb))
    a = T(r.standard_normal(sa).astype(np.float32))
    b = T((r.standard_normal(sb) / np.sqrt(sb[0])).astype(np.float32))
    bias = T(r.standard_normal(sb[1]).astype(np.float32)) if with_bias else None
    res = T(r.standard_normal(sa[:-1] + (sb[1],)).astype(np.float32))
    ops.Config.matmul_dtype = "bf16"
    try:
        fused = ops.gemm(a, b, bias=bias, resid=res)
        # a zero bias keeps the reference GEMM off the split-K path (same summation order)
        zb = bias if bias is not None else torch.zeros(sb[1], device="cuda")
        ref = ops.op_add(ops.gemm(a, b, bias=zb), res)
    finally:
        ops.Config.matmul_dtype = "f32"
    np.testing.assert_array_equal(to_np(fused), to_np(ref))


def test_gemm_bf16_two_level_batch_views():
    """Attention-style head-split views go to the tensor cores without copies."""
    from b200 import ops

    r = rng(15)
    B_, S, H, hd = 2, 128, 4, 64
    y = _bf16(r.standard_normal((B_ * S, H * hd), dtype=np.float32))
    Y = T(y).to(torch.bfloat16)
    q = Y.view(B_, S, H, hd).permute(0, 2, 1, 3)          # [B, H, S, hd], strides (S*d, hd, d, 1)
    kT = Y.view(B_, S, H, hd).permute(0, 2, 3, 1)         # [B, H, hd, S]
    qn = y.reshape(B_, S, H, hd).transpose(0, 2, 1, 3)
    kn = y.reshape(B_, S, H, hd).transpose(0, 2, 3, 1)
    ref = np.matmul(qn.astype(np.float64), kn.astype(np.float64))
    got = to_np(ops.gemm(q, kT, ab_dtype=torch.bfloat16))
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-3)
    att = _bf16(r.standard_normal((B_, H, S, S), dtype=np.float32))
    ctx = to_np(ops.gemm(T(att).to(torch.bfloat16), q, ab_dtype=torch.bfloat16))
    np.testing.assert_allclose(ctx, np.matmul(att.astype(np.float64), qn.astype(np.float64)), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("rows,cols", [(37, 512), (16, 96), (9, 2048), (5, 1000), (3, 3000), (40, 4)])
@pytest.mark.parametrize("log", [0, 1])
def test_softmax_rows_scaled_dual_output(rows, cols, log):
    from b200 import _lib as L

    r = rng(rows * 7 + cols + log)
    x = (r.standard_normal((rows, cols)) * 4).astype(np.float32)
    s = np.float32(0.125)
    t = (x * s).astype(np.float64)
    e = np.exp(t - t.max(-1, keepdims=True))
    ref = (t - t.max(-1, keepdims=True) - np.log(e.sum(-1, keepdims=True))) if log else e / e.sum(-1, keepdims=True)
    X, S = T(x), T(np.array(s, np.float32))
    Y = torch.empty_like(X)
    YB = torch.empty(X.shape, dtype=torch.bfloat16, device=X.device)
    L.call("b200_softmax_rows", X.data_ptr(), S.data_ptr(), Y.data_ptr(), YB.data_ptr(), rows, cols, log, 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(Y), ref, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(to_np(YB.float()), ref, rtol=1e-2, atol=1e-2 if log else 1e-4)


@pytest.mark.parametrize("rows,cols", [(37, 512), (16, 96), (9, 2048), (5, 1000), (3, 3000)])
def test_softmax_bwd_rows(rows, cols):
    from b200 import _lib as L

    r = rng(rows + cols)
    x = r.standard_normal((rows, cols)).astype(np.float32)
    y = np.exp(x - x.max(-1, keepdims=True))
    y = (y / y.sum(-1, keepdims=True)).astype(np.float32)
    g = r.standard_normal((rows, cols)).astype(np.float32)
    s = np.float32(0.3)
    y64, g64 = y.astype(np.float64), g.astype(np.float64)
    ref = s * (y64 * (g64 - (g64 * y64).sum(-1, keepdims=True)))
    Y, G, S = T(y), T(g), T(np.array(s, np.float32))
    D = torch.empty_like(Y)
    DB = torch.empty(Y.shape, dtype=torch.bfloat16, device=Y.device)
    L.call("b200_softmax_bwd_rows", Y.data_ptr(), G.data_ptr(), S.data_ptr(), D.data_ptr(), DB.data_ptr(), rows, cols, 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(D), ref, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(to_np(DB.float()), ref, rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("cols", [96, 1024, 2048, 1000])
def test_layernorm_rows_bf16_output(cols):
    from b200 import ops
    from oracle import evaluator as O

    r = rng(cols)
    x = (r.standard_normal((45, cols)) * 3 + 1).astype(np.float32)
    g = r.uniform(0.5, 1.5, cols).astype(np.float32)
    b = r.standard_normal(cols).astype(np.float32)
    ref = O.execute_op("LayerNorm", x, g, b, eps=1e-5)
    y, yb = ops.layer_norm(T(x), T(g), T(b), 1e-5, -1, f32=True, bf16=True)
    np.testing.assert_allclose(to_np(y), ref, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(to_np(yb.float()), ref, rtol=1e-2, atol=1e-2)
    y2, yb2 = ops.layer_norm(T(x), T(g), T(b), 1e-5, -1, f32=False, bf16=True)
    assert y2 is None and torch.equal(yb2, yb)


@pytest.mark.parametrize("M,N,K", [(300, 384, 256), (200, 136, 72), (64, 40, 128)])
@pytest.mark.parametrize("epi", ["gelu", "relu"])
def test_gemm_dual_output_pre_and_bf16_activation(M, N, K, epi):
    """pre = A.B + bias in fp32 and act(pre) in bf16 from one epilogue (ragged tiles are
    clipped by the bulk stores)."""
    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O

    r = rng(M + N + K)
    a = _bf16(r.standard_normal((M, K), dtype=np.float32) * 0.1)
    b = _bf16(r.standard_normal((K, N), dtype=np.float32) * 0.1)
    bias = (r.standard_normal(N) * 0.1).astype(np.float32)
    pre = (a.astype(np.float64) @ b.astype(np.float64) + bias).astype(np.float32)
    act = O.execute_op("Gelu", pre) if epi == "gelu" else np.maximum(pre, 0)
    e = L.EPI_GELU if epi == "gelu" else L.EPI_RELU
    res = ops.gemm(T(a).to(torch.bfloat16), T(b).to(torch.bfloat16), bias=T(bias), epilogue=e, act_bf16=True,
                   want_mask=(epi == "relu"), ab_dtype=torch.bfloat16)
    np.testing.assert_allclose(to_np(res[0]), pre, rtol=1e-4, atol=1e-4)
    assert res[1].dtype == torch.bfloat16
    np.testing.assert_allclose(to_np(res[1].float()), act, rtol=1e-2, atol=1e-2)
    if epi == "relu":
        assert (to_np(res[2]) == (pre > 0)).mean() > 0.999


@pytest.mark.parametrize("R,C", [(300, 4096), (37, 1000), (5, 7)])
def test_gelu_bwd_colsum_matches_vjp_chain(R, C):
    from b200 import _lib as L
    from oracle import evaluator as O

    r = rng(R + C)
    g = r.standard_normal((R, C)).astype(np.float32)
    p = (r.standard_normal((R, C)) * 2).astype(np.float32)
    k, c = np.float32(np.sqrt(2.0 / np.pi)), np.float32(0.044715)
    mul, add = (lambda a, b: O.execute_op("Multiply", a, b)), (lambda a, b: O.execute_op("Add", a, b))
    p2 = mul(p, p)
    t = O.execute_op("Tanh", mul(add(p, mul(mul(p2, p), c)), k))
    left = mul(add(t, np.float32(1)), np.float32(0.5))
    sech2 = O.execute_op("Subtract", np.float32(1), mul(t, t))
    dinner = mul(add(mul(p2, np.float32(3 * 0.044715)), np.float32(1)), k)
    ref = mul(g, add(left, mul(mul(mul(p, sech2), dinner), np.float32(0.5))))
    G, P = T(g), T(p)
    Y = torch.empty_like(G)
    YB = torch.empty(G.shape, dtype=torch.bfloat16, device=G.device)
    DB = torch.empty(C, dtype=torch.float32, device=G.device)
    ws_n = int(L.lib().b200_gelu_bwd_colsum_workspace_bytes(R, C))
    WS = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=G.device)
    L.call("b200_gelu_bwd_colsum", G.data_ptr(), P.data_ptr(), YB.data_ptr(), Y.data_ptr(), DB.data_ptr(), R, C,
           WS.data_ptr(), ws_n, 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(Y), ref, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(to_np(YB.float()), ref, rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(to_np(DB), ref.astype(np.float64).sum(0), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("ta", [False, True])
def test_gemm_split_k_weight_gradient_shape(ta):
    """Few output tiles and a long K (a weight gradient): split over K, summed in order."""
    from b200 import ops

    r = rng(21)
    M, N, K = 256, 384, 16384
    a = _bf16(r.standard_normal((K, M) if ta else (M, K), dtype=np.float32) * 0.05)
    b = _bf16(r.standard_normal((K, N), dtype=np.float32) * 0.05)
    A = T(a).to(torch.bfloat16)
    A = A.t() if ta else A
    an = a.T if ta else a
    assert ops._split_k(M, N, K) > 1
    got = to_np(ops.gemm(A, T(b).to(torch.bfloat16), ab_dtype=torch.bfloat16))
    np.testing.assert_allclose(got, an.astype(np.float64) @ b.astype(np.float64), rtol=1e-4, atol=1e-3)


def test_gemm_out_transposed_layout_and_twin():
    """GEMM written through a permuted view (head merge) with a bf16 twin of the same strides."""
    from b200 import ops

    r = rng(22)
    Bn, H, S, hd = 2, 4, 128, 64
    att = _bf16(r.standard_normal((Bn, H, S, S), dtype=np.float32) * 0.1)
    v = _bf16(r.standard_normal((Bn, H, S, hd), dtype=np.float32))
    ref = np.matmul(att.astype(np.float64), v.astype(np.float64)).transpose(0, 2, 1, 3)
    y = torch.empty(Bn, S, H, hd, dtype=torch.float32, device="cuda")
    yb = torch.empty(Bn, S, H, hd, dtype=torch.bfloat16, device="cuda")
    ok = ops.gemm_out(T(att).to(torch.bfloat16), T(v).to(torch.bfloat16), y.permute(0, 2, 1, 3), yb.permute(0, 2, 1, 3),
                      ab_dtype=torch.bfloat16)
    assert ok
    np.testing.assert_allclose(to_np(y), ref, rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(to_np(yb.float()), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("shape", [(64, 1024), (37, 100), (5, 12), (3, 7, 8), (1001,), (2, 3)])
def test_elementwise_flat_modes_dtypes(shape):
    """Flat-path kernels: dense / scalar / last-dim vector / per-row operands, bf16 and
    bool inputs and outputs, single-op kernels and multi-op register programs, ragged
    group tails (n % 8 != 0) and rows that split 8-element groups."""
    from b200 import ops

    r = rng(sum(shape))
    x = r.standard_normal(shape).astype(np.float32)
    y = r.standard_normal(shape).astype(np.float32)
    vec = r.standard_normal(shape[-1]).astype(np.float32)
    rowv = r.standard_normal(shape[:-1] + (1,)).astype(np.float32)
    X, Y = T(x), T(y)
    np.testing.assert_allclose(to_np(ops.op_add(X, Y)), x + y, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_subtract(X, T(vec))), x - vec, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_multiply(X, T(rowv))), x * rowv, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_true_divide(X, 3.0)), x / np.float32(3.0), rtol=1e-6)
    np.testing.assert_array_equal(to_np(ops.op_greater(X, T(rowv))), x > rowv)
    np.testing.assert_allclose(to_np(ops.op_relu(X)), np.maximum(x, 0))
    # casts both ways
    xb = ops.cast(X, torch.bfloat16)
    np.testing.assert_array_equal(to_np(xb.float()), to_np(X.to(torch.bfloat16).float()))
    np.testing.assert_array_equal(to_np(ops.cast(xb, torch.float32)), to_np(xb.float()))
    # bf16 operand in a binary op, fp32 result
    np.testing.assert_allclose(to_np(ops.op_add(xb, Y)), to_np(xb.float()) + y, rtol=1e-6)
    # a multi-op register program with a row operand and two outputs
    p = ops.Prog()
    a, b, c = p.load(X), p.load(Y), p.load(T(rowv))
    t1 = p.op("MUL", a, b)
    t2 = p.op("ADD", t1, c)
    t3 = p.op("TANH", t2)
    out = p.run([(t3, torch.float32), (t3, torch.bfloat16)], shape)
    ref = np.tanh(x * y + rowv)
    np.testing.assert_allclose(to_np(out[0]), ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_np(out[1].float()), ref, rtol=1e-2, atol=1e-2)
    # sums of several inputs (the straight-line sum kernel) keep the program's left-to-right
    # order: bit-identical to numpy's fp32 ((a + b) + c) + d, with a vector operand and a
    # repeated input
    z = r.standard_normal(shape).astype(np.float32)
    p = ops.Prog()
    la, lb, lc, lv = p.load(X), p.load(Y), p.load(T(z)), p.load(T(vec))
    s1 = p.op("ADD", la, lb)
    s2 = p.op("ADD", lc, s1)
    s3 = p.op("ADD", s2, lv)
    s4 = p.op("ADD", s3, la)
    out = p.run([(s4, torch.float32), (s4, torch.bfloat16)], shape)
    ref = (((x + y) + z) + vec) + x
    np.testing.assert_array_equal(to_np(out[0]), ref)
    np.testing.assert_array_equal(to_np(out[1].float()), to_np(T(ref).to(torch.bfloat16).float()))


def test_elementwise_merged_dims():
    """Adjacent dims whose strides line up are merged before the path is chosen: a
    [N, C, 1, 1] operand broadcast over [N, C, H, W] becomes one value per row of H * W
    (row length 36, not a multiple of 8), a [1, C, 1, 1] operand stays a broadcast that no
    merge can flatten, and a permuted view keeps its own strides."""
    from b200 import ops

    r = rng(5)
    x = r.standard_normal((64, 128, 6, 6)).astype(np.float32)
    g = r.standard_normal((64, 128, 1, 1)).astype(np.float32)
    ch = r.standard_normal((1, 128, 1, 1)).astype(np.float32)
    X = T(x)
    np.testing.assert_allclose(to_np(ops.op_multiply(X, T(g))), x * g, rtol=1e-6)
    np.testing.assert_allclose(to_np(ops.op_add(X, T(ch))), x + ch, rtol=1e-6)
    p = ops.Prog()
    a, b, c = p.load(X), p.load(T(g)), p.load(T(ch))
    t1 = p.op("GT", a, c)
    t2 = p.op("MUL", t1, b)
    out = p.run([(t2, torch.float32)], x.shape)
    np.testing.assert_array_equal(to_np(out[0]), (x > ch) * g)
    xp = X.permute(0, 2, 3, 1)  # [64, 6, 6, 128] view over NCHW storage
    gp = T(g).permute(0, 2, 3, 1)
    np.testing.assert_allclose(to_np(ops.op_multiply(xp, gp)), x.transpose(0, 2, 3, 1) * g.transpose(0, 2, 3, 1), rtol=1e-6)


def test_elementwise_chains_and_programs():
    """Straight-line op chains (immediates on either side, the previous result on the right,
    unary links, ragged length) and a program that reuses an earlier value (the general
    register-program kernel) agree with numpy's fp32 results."""
    from b200 import ops

    r = rng(9)
    n = 1000003
    x = r.standard_normal(n).astype(np.float32)
    y = r.standard_normal(n).astype(np.float32)
    X, Y = T(x), T(y)
    p = ops.Prog()
    a, b = p.load(X), p.load(Y)
    c = p.imm(0.5)
    t1 = p.op("SUB", c, a)       # 0.5 - x
    t2 = p.op("MUL", b, t1)      # y * (0.5 - x): the result on the right
    t3 = p.op("TANH", t2)
    t4 = p.op("MAX", t3, p.imm(-0.25))
    out = p.run([(t4, torch.float32), (t4, torch.bfloat16)], (n,))
    ref = np.maximum(np.tanh(y * (np.float32(0.5) - x)), np.float32(-0.25))
    np.testing.assert_allclose(to_np(out[0]), ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_np(out[1].float()), ref, rtol=1e-2, atol=1e-2)
    p = ops.Prog()
    a, b = p.load(X), p.load(Y)
    t1 = p.op("MUL", a, b)
    t2 = p.op("ADD", t1, a)
    t3 = p.op("MUL", t1, t2)     # t1 read again after t2: not a chain
    out = p.run([(t3, torch.float32)], (n,))
    np.testing.assert_array_equal(to_np(out[0]), (x * y) * ((x * y) + x))


@pytest.mark.parametrize("R,V", [(33, 32000), (17, 1000), (9, 4096), (5, 12)])
def test_logsoftmax_pick_register_rows_bf16_dx(R, V):
    from b200 import _lib as L
    from b200 import ops

    r = rng(R * V)
    x = (r.standard_normal((R, V)) * 3).astype(np.float32)
    lab = r.integers(0, V, (R, 1)).astype(np.int64)
    d = r.standard_normal((R, 1)).astype(np.float32)
    x64 = x.astype(np.float64)
    lse = np.log(np.exp(x64 - x64.max(-1, keepdims=True)).sum(-1, keepdims=True)) + x64.max(-1, keepdims=True)
    sm = np.exp(x64 - lse)
    onehot = np.zeros_like(sm)
    onehot[np.arange(R), lab[:, 0]] = 1
    dx_ref = d * (onehot - sm)
    picked_ref = np.take_along_axis(x64 - lse, lab, -1)
    X, LB, D = T(x), T(lab), T(d)
    picked = torch.empty(R, 1, device=X.device)
    dx = torch.empty(R, V, device=X.device)
    dxb = torch.empty(R, V, dtype=torch.bfloat16, device=X.device)
    L.call("b200_logsoftmax_pick", L.F32, X.data_ptr(), LB.data_ptr(), D.data_ptr(), picked.data_ptr(), None,
           dx.data_ptr(), dxb.data_ptr(), R, V, ops.stream_ptr())
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(picked), picked_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(dx), dx_ref, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(to_np(dxb.float()), dx_ref, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("R,C", [(300, 1024), (77, 512), (9, 96), (5, 1000), (3, 4096)])
def test_layernorm_bwd_rows_fused_matches_oracle(R, C):
    from b200 import _lib as L
    from oracle import evaluator as O

    r = rng(R + C)
    x = (r.standard_normal((R, C)) * 2 + 0.5).astype(np.float32)
    dy = r.standard_normal((R, C)).astype(np.float32)
    g = r.uniform(0.5, 1.5, C).astype(np.float32)
    X, DY, G = T(x), T(dy), T(g)
    dx = torch.empty_like(X)
    dg = torch.empty(C, device=X.device)
    db = torch.empty(C, device=X.device)
    n = int(L.lib().b200_layernorm_bwd_workspace_bytes(R, C))
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=X.device)
    L.call("b200_layernorm_bwd_rows", DY.data_ptr(), X.data_ptr(), G.data_ptr(), dx.data_ptr(), None, dg.data_ptr(),
           db.data_ptr(), R, C, 1e-5, ws.data_ptr(), n, 0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(dx), O.execute_op("LayerNormInputGrad", dy, x, g, eps=1e-5), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(to_np(dg), O.execute_op("LayerNormGammaGrad", dy, x, eps=1e-5), rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(to_np(db), O.execute_op("LayerNormBetaGrad", dy), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("n,V,D", [(3000, 50, 96), (4096, 32000, 64), (2500, 1, 33)])
def test_scatter_add_rows_deterministic_in_position_order(n, V, D):
    """Row scatter-add sums each row's sources in position order: equal to a sequential
    fp32 accumulation, and bit-identical from run to run (one giant bucket included)."""
    from b200 import ops

    r = rng(n + V)
    base = r.standard_normal((V, D)).astype(np.float32)
    ids = r.integers(0, V, (n, 1)).astype(np.int64)
    if V > 1:
        ids[: n // 2, 0] = 0  # half the positions share one row
    upd = r.standard_normal((n, D)).astype(np.float32)
    ref = base.copy()
    for i in range(n):  # np.add.at order, fp32
        ref[ids[i, 0]] += upd[i]
    got1 = ops.op_tensor_scatter_add(T(base), T(ids), T(upd))
    got2 = ops.op_tensor_scatter_add(T(base), T(ids), T(upd))
    torch.cuda.synchronize()
    assert torch.equal(got1, got2)
    np.testing.assert_allclose(to_np(got1), ref, rtol=1e-5, atol=1e-4)


def test_column_reduce_split_deterministic():
    from b200 import ops

    r = rng(31)
    x = r.standard_normal((32768, 1024)).astype(np.float32)
    X = T(x)
    a = ops.op_reduce_sum(X, axis=0)
    b = ops.op_reduce_sum(X, axis=0)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    np.testing.assert_allclose(to_np(a), x.astype(np.float64).sum(0), rtol=1e-4, atol=1e-3)
    m = ops.op_reduce_mean(X, axis=0)
    np.testing.assert_allclose(to_np(m), x.astype(np.float64).mean(0), rtol=1e-4, atol=1e-5)
    mx = ops.op_reduce_max(X, axis=0)
    np.testing.assert_array_equal(to_np(mx), x.max(0))


@pytest.mark.parametrize("B_,H,S,hd", [(2, 4, 512, 64), (1, 3, 200, 64), (2, 2, 32, 16), (1, 2, 384, 128)])
def test_attention_rows_fused_softmax_and_vjp(B_, H, S, hd):
    """Scores GEMM with the softmax in its epilogue (and dO.V^T with the softmax VJP), on
    the head-split views attention uses ([B*S, H*hd] read as [B, H, S, hd] without copies):
    against float64 on the same bf16 operands. Ragged rows / columns (S = 200), a head dim
    of 16 and of 128, and both dtypes of the saved softmax output in the backward."""
    from b200 import ops

    r = rng(B_ * 1000 + S + hd)
    q = _bf16(r.standard_normal((B_ * S, H * hd), dtype=np.float32))
    k = _bf16(r.standard_normal((B_ * S, H * hd), dtype=np.float32))
    Q = T(q).to(torch.bfloat16).view(B_, S, H, hd).permute(0, 2, 1, 3)   # [B, H, S, hd]
    KT = T(k).to(torch.bfloat16).view(B_, S, H, hd).permute(0, 2, 3, 1)  # [B, H, hd, S]
    scale = np.float32(1.0 / np.sqrt(hd))
    qn = q.reshape(B_, S, H, hd).transpose(0, 2, 1, 3).astype(np.float64)
    kn = k.reshape(B_, S, H, hd).transpose(0, 2, 3, 1).astype(np.float64)
    z = np.matmul(qn, kn) * np.float64(scale)
    e = np.exp(z - z.max(-1, keepdims=True))
    yref = e / e.sum(-1, keepdims=True)
    from b200 import _lib

    sc = T(np.array(scale))
    n0 = _lib.launch_count()
    y, yb = ops.gemm_softmax_rows(Q, KT, sc, True, True)
    assert _lib.launch_count() - n0 == 1  # the fused kernel, not the GEMM + softmax fallback
    np.testing.assert_allclose(to_np(y), yref, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(to_np(yb.float()), yref, rtol=1e-2, atol=1e-4)
    none, yb1 = ops.gemm_softmax_rows(Q, KT, sc, False, True)
    assert none is None
    np.testing.assert_array_equal(to_np(yb1.float()), to_np(yb.float()))
    # backward: G = dO.V^T, dx = scale * y * (G - rowsum(G y))
    do = _bf16(r.standard_normal((B_ * S, H * hd), dtype=np.float32))
    v = _bf16(r.standard_normal((B_ * S, H * hd), dtype=np.float32))
    DO = T(do).to(torch.bfloat16).view(B_, S, H, hd).permute(0, 2, 1, 3)
    VT = T(v).to(torch.bfloat16).view(B_, S, H, hd).permute(0, 2, 3, 1)
    G = np.matmul(do.reshape(B_, S, H, hd).transpose(0, 2, 1, 3).astype(np.float64),
                  v.reshape(B_, S, H, hd).transpose(0, 2, 3, 1).astype(np.float64))
    for ysaved in (y, yb):
        yv = to_np(ysaved.float()).astype(np.float64)
        dref = np.float64(scale) * yv * (G - (G * yv).sum(-1, keepdims=True))
        n0 = _lib.launch_count()
        dx, dxb = ops.gemm_softmax_bwd_rows(DO, VT, ysaved, sc, True, True)
        assert _lib.launch_count() - n0 == 1
        if ysaved is y:  # one output at a time (a lighter staging layout, a deeper y ring)
            none, dx1 = ops.gemm_softmax_bwd_rows(DO, VT, ysaved, sc, False, True)
            assert none is None
            np.testing.assert_array_equal(to_np(dx1.float()), to_np(dxb.float()))
        np.testing.assert_allclose(to_np(dx), dref, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(to_np(dxb.float()), dref, rtol=1e-2, atol=1e-3)

"""CPU ORACLE (test infrastructure only): numpy restatement of the reference's
graph interpreter and of the numpy-backend op kernels on the fwd+bwd hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only to check results or as the timed CPU reference. The
``b200`` backend never calls it.

Interpreter: ``evaluate`` follows ``interpreter/evaluator.py:272-305`` (env = inputs,
nodes in dependency order, every node evaluated, outputs read back) and
``_evaluate_node`` (``evaluator.py:738-769``: Input / Output / Identity / Constant /
dispatch) with the op aliases of ``_get_op_alias`` (``evaluator.py:771-791``) and the
kwargs rules of ``_prepare_node_kwargs`` (``evaluator.py:793-832``).

Op kernels: each ``_op_*`` cites the reference kernel it restates. numpy dtype
behaviour is kept (fp32 stays fp32; a Python-float constant is a float64 0-d array,
``evaluator.py:760-761``).

Parity of this restatement is pinned by ``tests/test_oracle.py`` against the golden
vectors that ``tests/golden/make_golden.py`` produced by running the reference's own
``evaluate_graph`` on the same graphs, and against the reference's known-answer tests
(``tests/backends/test_hardware_parity.py:164-205``,
``tests/distributed/test_multi_process_collectives.py:83-103``).
"""

from __future__ import annotations

import gzip
import json
import math
import os
from typing import Any

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests", "golden")

_ALIASES = {  # evaluator.py:771-791
    "Sub": "Subtract",
    "Mul": "Multiply",
    "Div": "TrueDivide",
    "Neg": "Negative",
    "Pow": "Power",
    "MatMul": "Matmul",
    "Expand": "BroadcastTo",
    "Permute": "Transpose",
}


def load_graph(name_or_path: str) -> dict:
    """Load a serialized LogicalGraph (``tests/golden/graphs/<name>.json.gz``)."""
    path = name_or_path
    if not os.path.exists(path):
        path = os.path.join(GOLDEN_DIR, "graphs", name_or_path + ".json.gz")
    with gzip.open(path, "rt", encoding="utf-8") as f:
        return json.load(f)


def topo_order(graph: dict) -> list[dict]:
    """Dependency order over all nodes (``core/utils/graph_utils.py:29-100`` is a DFS;
    any dependency order gives identical values for this side-effect-free graph)."""
    nodes = {n["id"]: n for n in graph["nodes"]}
    order, state = [], {}
    for root in nodes:
        if root in state:
            continue
        stack = [(root, 0)]
        while stack:
            nid, i = stack.pop()
            if i == 0:
                if state.get(nid) == 2:
                    continue
                state[nid] = 1
            deps = [d for d in nodes[nid]["inputs"] if d in nodes]
            if i < len(deps):
                stack.append((nid, i + 1))
                d = deps[i]
                if state.get(d) == 1:
                    raise ValueError("cycle in graph")  # CompilationError in the reference
                if d not in state:
                    stack.append((d, 0))
            else:
                state[nid] = 2
                order.append(nodes[nid])
    return order


def _kwargs(node: dict, target: str) -> dict:
    """``_prepare_node_kwargs`` (evaluator.py:793-832)."""
    kw = {k: v for k, v in (node.get("attributes") or {}).items() if k not in ("var_name", "is_parameter", "param_name")}
    conv_like = {"Conv", "Conv1D", "Conv2D", "Conv3D", "ConvTranspose", "ConvTranspose2D", "MaxPool2D", "AvgPool2D", "StridedSlice"}
    if "strides" in kw and target not in conv_like:
        kw.pop("strides")
    meta = node.get("shape_metadata")
    if meta:
        mt = tuple(int(d) if isinstance(d, int) else str(d) for d in meta)
        if target in ("Expand", "BroadcastTo", "ConstantOfShape", "Zeros", "Ones", "Full") and "shape" not in kw:
            kw["shape"] = mt
        if target == "Reshape" and "newshape" not in kw:
            kw["newshape"] = mt
    return kw


# ----------------------------------------------------------------------------------
# op kernels
# ----------------------------------------------------------------------------------


# When set (``evaluate(..., blas_layout=True)``), fp32 contractions run on dense operands
# through a batched CPU BLAS (torch.matmul on host tensors). numpy hands strided batch
# views (attention's head split and its transposes) to a plain C loop instead of BLAS,
# which is two orders of magnitude slower at the benchmark sizes. The arithmetic is the
# same fp32 matmul with fp32 accumulation; only the summation order inside BLAS differs,
# so this mode is for the size-scaled parity tests, which compare with a tolerance, not
# for the bit-exact pins against the reference's fixtures.
_BLAS_LAYOUT = False


def _op_matmul(a, b, transpose_a=False, transpose_b=False, **_):
    # backends/eager/core_math_ops/math_matrix.py:21-44
    if transpose_a:
        a = np.swapaxes(a, -1, -2)
    if transpose_b:
        b = np.swapaxes(b, -1, -2)
    if _BLAS_LAYOUT and a.dtype == np.float32 and b.dtype == np.float32 and a.ndim >= 2 and b.ndim >= 2:
        import torch

        return torch.matmul(torch.from_numpy(np.ascontiguousarray(a)), torch.from_numpy(np.ascontiguousarray(b))).numpy()
    return np.matmul(a, b)


def _op_gelu(x, **_):
    # backends/eager/core_math_ops/math_nn.py:184-199 (tanh approximation)
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * (x**3))))


def _op_softmax(a, axis=-1, **_):
    # backends/numpy/eager/math_advanced/math_signal.py:450-467
    e = np.exp(a - np.max(a, axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


def _op_log_softmax(a, axis=-1, **_):
    # backends/numpy/eager/math_advanced/math_log_exp.py:87-104
    c = np.max(a, axis=axis, keepdims=True)
    return a - c - np.log(np.sum(np.exp(a - c), axis=axis, keepdims=True))


def _ln_stats(x, eps, axis):
    mean = np.mean(x, axis=axis, keepdims=True)
    var = np.var(x, axis=axis, keepdims=True)
    return mean, var


def _op_layer_norm(x, gamma=None, beta=None, eps=1e-5, axis=-1, **kw):
    # backends/numpy/eager/nn_ops.py:219-241
    eps = float(kw.get("epsilon", eps))
    gamma = np.ones(x.shape[-1], x.dtype) if gamma is None else gamma
    beta = np.zeros(x.shape[-1], x.dtype) if beta is None else beta
    mean, var = _ln_stats(x, eps, axis)
    return gamma * ((x - mean) / np.sqrt(var + eps)) + beta


def _op_layer_norm_input_grad(d_out, x, gamma=None, eps=1e-5, axis=-1, **_):
    # backends/numpy/eager/nn_ops.py:244-273
    gamma = np.ones(x.shape[-1], x.dtype) if gamma is None else gamma
    d = float(x.shape[int(axis)])
    mean, var = _ln_stats(x, eps, axis)
    inv_std = 1.0 / np.sqrt(var + eps)
    x_hat = (x - mean) * inv_std
    d_y = d_out * gamma
    term2 = np.sum(d_y, axis=axis, keepdims=True)
    term3 = x_hat * np.sum(d_y * x_hat, axis=axis, keepdims=True)
    return (inv_std / d) * (d * d_y - term2 - term3)


def _op_layer_norm_gamma_grad(d_out, x, eps=1e-5, axis=-1, **_):
    # backends/numpy/eager/nn_ops.py:276-297
    mean, var = _ln_stats(x, eps, axis)
    x_hat = (x - mean) / np.sqrt(var + eps)
    ax = x.ndim + int(axis) if int(axis) < 0 else int(axis)
    return np.sum(d_out * x_hat, axis=tuple(i for i in range(x.ndim) if i != ax))


def _op_layer_norm_beta_grad(d_out, axis=-1, **_):
    # backends/numpy/eager/nn_ops.py:300-318
    ax = d_out.ndim + int(axis) if int(axis) < 0 else int(axis)
    return np.sum(d_out, axis=tuple(i for i in range(d_out.ndim) if i != ax))


def _axis(axis):
    return tuple(axis) if isinstance(axis, list) else axis


def _op_reduce_sum(x, axis=None, keepdims=False, **_):
    # backends/eager/core_math_ops/math_reduction.py:37-54
    return np.sum(x, axis=_axis(axis), keepdims=keepdims)


def _op_reduce_mean(x, axis=None, keepdims=False, **_):
    # backends/eager/core_math_ops/math_reduction.py:57-74
    return np.mean(x, axis=_axis(axis), keepdims=keepdims)


def _op_reduce_max(x, axis=None, keepdims=False, **_):
    # backends/eager/core_math_ops/math_reduction.py:97-114
    return np.max(x, axis=_axis(axis), keepdims=keepdims)


def _op_numel(x, **_):
    # backends/eager/core_math_ops/math_reduction.py:156-173 (a Python float)
    return float(np.asarray(x).size)


def _op_broadcast_like(src, tgt, **_):
    # backends/eager/core_math_ops/math_reduction.py:227-249
    if np.shape(src) == np.shape(tgt):
        return src
    return np.broadcast_to(src, np.shape(tgt))


def _op_broadcast_reduce(cot, tgt, **_):
    # backends/eager/core_math_ops/math_reduction.py:192-224
    cs, ts = np.shape(cot), np.shape(tgt)
    if cs == ts:
        return cot
    res = cot
    if len(cs) > len(ts):
        res = np.sum(res, axis=tuple(range(len(cs) - len(ts))))
    for i, (cd, td) in enumerate(zip(np.shape(res), ts)):
        if td == 1 and cd > 1:
            res = np.sum(res, axis=i, keepdims=True)
    return res


def _op_argmax(x, axis=None, **_):
    # backends/numpy/eager/math_reductions.py:129-140 (np.argmax: first maximum wins)
    return np.argmax(x, axis=axis)


def _op_relu(x, **_):
    # backends/numpy/eager/activation_ops.py:12 (np.maximum(x, 0))
    return np.maximum(x, 0)


def _op_transpose(x, axes=None, **_):
    # backends/numpy/eager/array_manipulation.py:121
    return np.transpose(x, axes)


def _op_reshape(x, shape=None, newshape=None, **_):
    # backends/numpy/eager/array_manipulation.py:87
    return np.reshape(x, tuple(shape if shape is not None else newshape))


def _op_take_along_axis(x, indices, axis=-1, **_):
    # backends/numpy/eager/advanced_indexing.py:163-177
    return np.take_along_axis(x, indices, axis=axis)


def _op_scatter_add(inp, index, src, dim=0, **_):
    # backends/numpy/eager/advanced_indexing.py:309-326 (put_along_axis of take+src;
    # a repeated index along ``dim`` keeps the last write, as in the reference)
    out = np.copy(inp)
    np.put_along_axis(out, index, np.add(np.take_along_axis(out, index, axis=dim), src), axis=dim)
    return out


def _op_tensor_scatter_add(tensor, indices, updates, **_):
    # backends/numpy/eager/math_scatter.py:39-60 (np.add.at accumulates repeats)
    res = np.array(tensor)
    idx = tuple(np.moveaxis(np.array(indices), -1, 0))
    np.add.at(res, idx, np.array(updates))
    return res


def _op_take(a, indices, axis=None, **_):
    # numpy-backend fallback to np.take (backends/numpy/eager/__init__.py:114-125)
    return np.take(a, indices, axis=axis)


def _conv_pads(in_hw, k_hw, s_hw, padding, out_hw):
    # backends/numpy/eager/conv.py:590-633 (_compute_conv2d_padding_values, dilation 1)
    if isinstance(padding, str) and padding.upper() == "SAME":
        ph = max(0, (out_hw[0] - 1) * s_hw[0] + k_hw[0] - in_hw[0])
        pw = max(0, (out_hw[1] - 1) * s_hw[1] + k_hw[1] - in_hw[1])
        return ph // 2, ph - ph // 2, pw // 2, pw - pw // 2
    return 0, 0, 0, 0


def _conv_out_hw(in_hw, k_hw, s_hw, padding):
    if isinstance(padding, str) and padding.upper() == "SAME":
        return (-(-in_hw[0] // s_hw[0]), -(-in_hw[1] // s_hw[1]))
    return ((in_hw[0] - k_hw[0]) // s_hw[0] + 1, (in_hw[1] - k_hw[1]) // s_hw[1] + 1)


def _stride2(stride):
    return (stride, stride) if isinstance(stride, int) else (int(stride[0]), int(stride[1]))


def _op_conv2d(x, w, stride=(1, 1), padding="SAME", groups=1, **kw):
    # backends/numpy/eager/conv.py:462-489 (NCHW x OIHW, no bias, no dilation)
    s = _stride2(kw.get("strides", stride))
    n, c, h, wd = x.shape
    o, ci, kh, kw_ = w.shape
    oh, ow = _conv_out_hw((h, wd), (kh, kw_), s, padding)
    pt, pb, pl, pr = _conv_pads((h, wd), (kh, kw_), s, padding, (oh, ow))
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr))) if (pt or pb or pl or pr) else x
    out = np.zeros((n, o, oh, ow), dtype=np.result_type(x, w))
    for i in range(kh):
        for j in range(kw_):
            patch = xp[:, :, i : i + oh * s[0] : s[0], j : j + ow * s[1] : s[1]]
            out += np.einsum("nihw,oi->nohw", patch, w[:, :, i, j])
    return out


def _op_conv2d_input_grad(d_out, w, stride=(1, 1), padding="SAME", target_shape=None, **kw):
    # backends/numpy/eager/conv.py:634-697 (groups 1, dilation 1)
    s = _stride2(kw.get("strides", stride))
    n, c, h, wd = (int(v) for v in target_shape)
    o, ci, kh, kw_ = w.shape
    oh, ow = d_out.shape[2], d_out.shape[3]
    pt, pb, pl, pr = _conv_pads((h, wd), (kh, kw_), s, padding, (oh, ow))
    dx = np.zeros((n, c, h + pt + pb, wd + pl + pr), dtype=d_out.dtype)
    for i in range(kh):
        for j in range(kw_):
            dx[:, :, i : i + oh * s[0] : s[0], j : j + ow * s[1] : s[1]] += np.einsum("nohw,oi->nihw", d_out, w[:, :, i, j])
    return dx[:, :, pt : pt + h, pl : pl + wd]


def _op_conv2d_weight_grad(x, d_out, stride=(1, 1), padding="SAME", target_shape=None, **kw):
    # backends/numpy/eager/conv.py:699-764 (groups 1, dilation 1)
    s = _stride2(kw.get("strides", stride))
    o, ci, kh, kw_ = (int(v) for v in target_shape)
    h, wd = x.shape[2], x.shape[3]
    oh, ow = d_out.shape[2], d_out.shape[3]
    pt, pb, pl, pr = _conv_pads((h, wd), (kh, kw_), s, padding, (oh, ow))
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr))) if (pt or pb or pl or pr) else x
    dw = np.zeros((o, ci, kh, kw_), dtype=x.dtype)
    for i in range(kh):
        for j in range(kw_):
            patch = xp[:, :, i : i + oh * s[0] : s[0], j : j + ow * s[1] : s[1]]
            dw[:, :, i, j] = np.einsum("nohw,nihw->oi", d_out, patch)
    return dw


def _op_conv2d_bias_grad(d_out, **_):
    # backends/numpy/eager/conv.py:766-779
    return np.sum(d_out, axis=(0, 2, 3))


# ---- optimizer update steps (backends/numpy/eager/optimizers_ops.py) ----------------
# The numpy backend's own registry wins over the generic one for these names
# (numpy/eager/__init__.py:110-115), so its fixed hyperparameters apply: Adam with
# beta1 0.9, beta2 0.999, eps 1e-8 and no bias correction; Adagrad eps 1e-10; RMSProp rho
# 0.9, momentum 0, eps 1e-8; FTRL in its simplified numpy form. `lr` is a Python float,
# so numpy computes in the arrays' fp32 with one rounding per operation.
def _op_apply_adam(param, m, v, grad, lr=0.001, **_):
    # numpy/eager/optimizers_ops.py:11-35
    p, m_, v_, g = np.asarray(param), np.asarray(m), np.asarray(v), np.asarray(grad)
    beta1, beta2, eps = 0.9, 0.999, 1e-8
    m_new = m_ * beta1 + g * (1.0 - beta1)
    v_new = v_ * beta2 + (g * g) * (1.0 - beta2)
    p_new = p - float(lr) * (m_new / (np.sqrt(v_new) + eps))
    return p_new, m_new, v_new


def _op_apply_adagrad(param, accum, grad, lr=0.01, **_):
    # numpy/eager/optimizers_ops.py:38-59
    p, a, g = np.asarray(param), np.asarray(accum), np.asarray(grad)
    a_new = a + g * g
    p_new = p - float(lr) * (g / (np.sqrt(a_new) + 1e-10))
    return p_new, a_new


def _op_apply_ftrl(param, accum, linear, grad, lr=0.001, **_):
    # numpy/eager/optimizers_ops.py:62-83
    p, a, lin, g = np.asarray(param), np.asarray(accum), np.asarray(linear), np.asarray(grad)
    lr = float(lr)
    a_new = a + g * g
    sigma = (np.sqrt(a_new) - np.sqrt(a)) / lr
    l_new = lin - g + sigma * p
    p_new = p - lr * g
    return p_new, a_new, l_new


def _op_apply_rmsprop(param, ms, mom, grad, lr=0.001, **_):
    # numpy/eager/optimizers_ops.py:86-103
    p, m, mo, g = np.asarray(param), np.asarray(ms), np.asarray(mom), np.asarray(grad)
    rho, momentum, eps = 0.9, 0.0, 1e-8
    m_new = m * rho + (g * g) * (1.0 - rho)
    mo_new = mo * momentum + g / (np.sqrt(m_new) + eps)
    p_new = p - float(lr) * mo_new
    return p_new, m_new, mo_new


def _op_gather(*args, **kwargs):
    # backends/numpy/eager/indexing.py:312-332: take_along_axis(tensor, index, axis=dim),
    # arguments (tensor, dim, index) positionally or as keywords
    t = args[0] if len(args) > 0 else kwargs.get("tensor")
    dim = args[1] if len(args) > 1 else kwargs.get("dim")
    index = args[2] if len(args) > 2 else kwargs.get("index")
    dim = None if dim is None else int(np.asarray(dim).item())
    return np.take_along_axis(np.asarray(t), np.asarray(index), axis=dim)


def _op_one_hot(*args, **kwargs):
    # backends/numpy/eager/math_advanced/math_general.py:710-736
    indices = args[0] if args else None
    depth = args[1] if len(args) > 1 else kwargs.get("depth")
    if indices is None or depth is None:
        return None
    on_value = float(kwargs.get("on_value", 1))
    off_value = float(kwargs.get("off_value", 0))
    axis = kwargs.get("axis", -1)
    dtype = kwargs.get("dtype", float)
    out = np.eye(int(np.asarray(depth).item()), dtype=dtype)[indices]
    if axis != -1:
        out = np.moveaxis(out, -1, axis)
    out = out * (on_value - off_value) + off_value
    return out.astype(dtype)


# --- node types of the reference's fusion passes (no reference kernel exists; their
# meaning is the computation the pass folded into them) -----------------------------
_C_FUNCS = {"fmaxf": np.fmax, "fminf": np.fmin, "expf": np.exp, "logf": np.log, "sqrtf": np.sqrt, "tanhf": np.tanh,
            "fabsf": np.abs}


def _scalar_expr(expr: str, inputs):
    """Evaluate a FusedElementwise ``scalar_expr`` (transforms/passes/operator_fusion.py:
    619-715: a C float expression over in0..inN) in float32, left to right like C."""
    import ast
    import re

    text = re.sub(r"(\d+\.\d*|\.\d+|\d+)([eE][+-]?\d+)?[fF]\b", lambda m: m.group(1) + (m.group(2) or ""), expr)
    tree = ast.parse(text, mode="eval").body
    f32 = np.float32

    def ev(n):
        if isinstance(n, ast.BinOp):
            a, b = ev(n.left), ev(n.right)
            op = {ast.Add: np.add, ast.Sub: np.subtract, ast.Mult: np.multiply, ast.Div: np.true_divide}[type(n.op)]
            return op(a, b, dtype=f32)
        if isinstance(n, ast.UnaryOp):
            v = ev(n.operand)
            return np.negative(v, dtype=f32) if isinstance(n.op, ast.USub) else v
        if isinstance(n, ast.Constant):
            return f32(n.value)
        if isinstance(n, ast.Name):
            k = int(re.fullmatch(r"in_?(\d+)", n.id).group(1))
            return np.asarray(inputs[k]).astype(f32)
        if isinstance(n, ast.Call):
            return _C_FUNCS[n.func.id](*[ev(a) for a in n.args], dtype=f32)
        raise ValueError(f"scalar_expr: unsupported {ast.dump(n)}")

    return np.asarray(ev(tree), dtype=f32)


def _op_fused_elementwise(*inputs, scalar_expr="0.0f", **_):
    # transforms/passes/operator_fusion.py:673-715
    shape = np.broadcast_shapes(*[np.shape(x) for x in inputs]) if inputs else ()
    return np.broadcast_to(_scalar_expr(str(scalar_expr), inputs), shape).copy()


def _silu(x, **_):
    return x * (1.0 / (1.0 + np.exp(-x)))


_FUSION_ELEMS = ("Add", "Sub", "Mul", "Div", "TrueDivide", "Relu", "Sigmoid", "Neg", "Abs", "Exp", "Log", "Sqrt", "Gelu", "Silu",
                 "Tanh", "Pow", "Maximum", "Minimum")  # operator_fusion.py:596-615
_FUSION_ACTS = ("Relu", "Gelu", "Silu", "Sigmoid", "Tanh")  # operator_fusion.py:918


def _named(op):
    op = _ALIASES.get(op, op)
    if op == "Silu":
        return _silu
    return OPS[op]


def _elem_act(elem, act):
    # operator_fusion.py:906-945 (attributes fused_ops = [elem, act]); the YAML rule
    # ElementwiseFusion (fusion_patterns/ElementwiseFusion.yaml) builds AddRelu the same way
    def run(*inputs, fused_ops=None, **_):
        e, a = (list(fused_ops) if fused_ops else [elem, act])
        return _named(a)(_named(e)(*inputs))

    return run


def _conv_bias_act(act):
    # operator_fusion.py:851-890: act(Conv2D(x, w) + bias) with the conv's attributes;
    # the declarative rule (attribute fused_pattern) is the activation root alone
    def run(*inputs, activation=None, has_bias=True, fused_pattern=None, **kw):
        if fused_pattern is not None:
            return _named(act)(*inputs)
        x, w, b = inputs
        ck = {k: v for k, v in kw.items() if k in ("stride", "padding", "groups", "dilation")}
        return _named(activation or act)(np.add(_op_conv2d(x, w, **ck), b))

    return run


def _horizontal(*inputs, fused_ops=(), **_):
    # operator_fusion.py:992-1071: the siblings' ops on the shared inputs (their
    # attributes are not kept by the pass)
    return tuple(_named(op)(*inputs) for op in fused_ops)


_DECLARATIVE_ROOT = {  # transforms/fusion_patterns.yaml: rule name -> targets[-1]
    "ScaledDotProductAttention": "Matmul", "ConvBNActivation": "Relu", "LayerNorm": "Add", "MatMulBiasGelu": "Gelu",
    "Conv2DBatchNormFusion": "BatchNorm", "Conv2DBiasActivationFusion": "Relu", "DotGeluFusion": "Gelu",
    "DotReluFusion": "Relu", "FMAFusion": "Add", "MultiHeadAttentionFusion": "Matmul"}


def _declarative(default_root):
    # operator_fusion.py:464-482: the root node cloned under the fused name
    def run(*inputs, fused_pattern=None, **kw):
        root = _DECLARATIVE_ROOT.get(str(fused_pattern), default_root) if fused_pattern is not None else default_root
        return _named(root)(*inputs, **kw)

    return run


def _fused_layer_norm(x, eps, scale=None, shift=None, **_):
    # fusion_patterns/LayerNormFusion.yaml: (x - mean) / sqrt(var + eps) [* scale + shift]
    e = float(np.asarray(eps).item())
    mean = np.mean(x, axis=-1, keepdims=True)
    var = np.mean((x - mean) * (x - mean), axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + e)
    if scale is not None:
        y = y * scale + shift
    return y


OPS: dict[str, Any] = {
    "ApplyAdam": _op_apply_adam,
    "ApplyAdagrad": _op_apply_adagrad,
    "ApplyFtrl": _op_apply_ftrl,
    "ApplyRMSProp": _op_apply_rmsprop,
    "Matmul": _op_matmul,
    "BatchMatMul": _op_matmul,
    "Add": lambda a, b, **_: np.add(a, b),  # backends/numpy/eager/math_binary.py:9-20
    "Subtract": lambda a, b, **_: np.subtract(a, b),  # math_binary.py:23-36
    "Multiply": lambda a, b, **_: np.multiply(a, b),  # math_binary.py:39-51
    "TrueDivide": lambda a, b, **_: np.true_divide(a, b),  # math_binary.py:54-66
    "Negative": lambda a, **_: np.negative(a),  # np fallback (numpy/eager/__init__.py:114-125)
    "Exp": lambda a, **_: np.exp(a),  # numpy/eager/math_unary.py:11
    "Log": lambda a, **_: np.log(a),  # np fallback
    "Tanh": lambda a, **_: np.tanh(a),  # np fallback
    "Sqrt": lambda a, **_: np.sqrt(a),  # np fallback
    "Power": lambda a, b, **_: np.power(a, b),  # np fallback
    "Greater": lambda a, b, **_: np.greater(a, b),  # numpy/eager/math_logical.py:26
    "Where": lambda c, a, b, **_: np.where(c, a, b),  # math_logical.py:146
    "Relu": _op_relu,
    "Gelu": _op_gelu,
    "Softmax": _op_softmax,
    "LogSoftmax": _op_log_softmax,
    "LayerNorm": _op_layer_norm,
    "LayerNormInputGrad": _op_layer_norm_input_grad,
    "LayerNormGammaGrad": _op_layer_norm_gamma_grad,
    "LayerNormBetaGrad": _op_layer_norm_beta_grad,
    "ReduceSum": _op_reduce_sum,
    "ReduceMean": _op_reduce_mean,
    "ReduceMax": _op_reduce_max,
    "Numel": _op_numel,
    "BroadcastLike": _op_broadcast_like,
    "BroadcastReduce": _op_broadcast_reduce,
    "Argmax": _op_argmax,
    "Transpose": _op_transpose,
    "Reshape": _op_reshape,
    "TakeAlongAxis": _op_take_along_axis,
    "ScatterAdd": _op_scatter_add,
    "TensorScatterAdd": _op_tensor_scatter_add,
    "Take": _op_take,
    "ZerosLike": lambda a, **_: np.zeros_like(a),  # np fallback
    "Gather": _op_gather,
    "OneHot": _op_one_hot,
    "Clone": lambda a, *_, **__: np.copy(a),  # backends/numpy/eager/__init__.py:128-145
    "Maximum": lambda a, b, **_: np.maximum(a, b),
    "Minimum": lambda a, b, **_: np.minimum(a, b),
    "Abs": lambda a, **_: np.abs(a),
    "Sigmoid": lambda a, **_: 1.0 / (1.0 + np.exp(-a)),
    "Conv2D": _op_conv2d,
    "Conv2DInputGrad": _op_conv2d_input_grad,
    "Conv2DWeightGrad": _op_conv2d_weight_grad,
    "Conv2DBiasGrad": _op_conv2d_bias_grad,
}


OPS["FusedElementwise"] = _op_fused_elementwise
for _e in _FUSION_ELEMS:
    for _a in _FUSION_ACTS:
        OPS.setdefault(f"{_e}{_a}", _elem_act(_e, _a))
for _c in ("Conv2D", "Conv"):
    for _a in _FUSION_ACTS:
        OPS[f"Fused{_c}Bias{_a}"] = _conv_bias_act(_a)
OPS["HorizontalFusedOps"] = _horizontal
OPS["TupleGetItem"] = lambda t, index=0, **_: t[int(index)]
for _n, _r in (("FusedAttention", "Matmul"), ("FusedConv2D", "Relu"), ("FusedLinearGELU", "Gelu"), ("FusedLinearGelu", "Gelu"),
               ("FusedLinearRelu", "Relu"), ("ScaledDotProductAttention", "Matmul")):
    OPS[_n] = _declarative(_r)
OPS["FusedLayerNorm"] = lambda *a, fused_pattern=None, **k: (_declarative("Add")(*a, fused_pattern=fused_pattern, **k)
                                                             if fused_pattern else _fused_layer_norm(*a, **k))
OPS["FusedMultiplyAdd"] = lambda *a, fused_pattern=None, **k: (_declarative("Add")(*a, fused_pattern=fused_pattern, **k)
                                                               if fused_pattern else np.add(np.multiply(a[0], a[1]), a[2]))
OPS["FusedLayerNormAffine"] = lambda x, scale, shift, eps, **_: _fused_layer_norm(x, eps, scale, shift)
OPS["FusedLogExp"] = lambda x, **_: np.exp(np.log(x))
OPS["DotGelu"] = lambda a, b, **_: _op_gelu(np.dot(a, b))
OPS["DotRelu"] = lambda a, b, **_: _op_relu(np.dot(a, b))
OPS["Linear"] = lambda x, w, b, **_: np.add(np.matmul(x, w), b)
OPS["Dot"] = lambda a, b, **_: np.dot(a, b)  # backends/eager/core_math_ops/math_matrix.py:66-82


CONTRACTIONS = ("Matmul", "BatchMatMul", "Conv2D", "Conv2DInputGrad", "Conv2DWeightGrad")


def bf16_round(a):
    """Round to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


class UnimplementedOp(KeyError):
    """No restatement for this op (the reference raises UnimplementedMathError)."""


def execute_op(op: str, *args, contraction_rounding: str | None = None, **kwargs):
    """One op. ``contraction_rounding="bf16"`` rounds both operands of a contraction
    (Matmul / Conv2D and its VJPs) to bfloat16 first: the reference algorithm under the
    bf16-math policy of the bf16 workloads (fp32 accumulation, fp32 everything else)."""
    target = _ALIASES.get(op, op)
    fn = OPS.get(target)
    if fn is None:
        raise UnimplementedOp(target)
    if contraction_rounding == "bf16" and target in CONTRACTIONS:
        args = (bf16_round(args[0]), bf16_round(args[1])) + tuple(args[2:])
    return fn(*args, **kwargs)


def evaluate(graph: dict, inputs: dict[str, np.ndarray], contraction_rounding: str | None = None,
             blas_layout: bool = False, decisions: dict | None = None, decision_report: list | None = None) -> dict[str, Any]:
    """``evaluate_graph`` (evaluator.py:272-305): every node, in dependency order.
    ``blas_layout=True`` passes dense operands to np.matmul (see ``_BLAS_LAYOUT``).

    ``decisions`` (node id -> boolean array) replays another implementation's values for
    ``Greater`` nodes, the ReLU VJP's masks: a pre-activation within rounding of zero may be
    classified either way by two correct fp32 evaluations, and each such flip moves a
    whole row of a weight gradient by one discrete term. Every replayed mask is checked
    against this evaluation's own first: ``decision_report`` receives, per node, the
    number of elements where the two differ and the largest |x| / rms(x) among them (the
    comparison operand's magnitude there), so a caller can require that they differ only
    at the decision boundary."""
    global _BLAS_LAYOUT
    prev, _BLAS_LAYOUT = _BLAS_LAYOUT, bool(blas_layout)
    try:
        return _evaluate(graph, inputs, contraction_rounding, decisions, decision_report)
    finally:
        _BLAS_LAYOUT = prev


def _replay_decision(nid, own, given, x, report) -> np.ndarray:
    given = np.asarray(given).astype(bool).reshape(np.shape(own))
    diff = given != np.asarray(own)
    n = int(diff.sum())
    worst = 0.0
    if n:
        xa = np.abs(np.broadcast_to(np.asarray(x, dtype=np.float64), np.shape(own)))
        scale = float(np.sqrt(np.mean(xa * xa))) or 1.0
        worst = float(xa[diff].max() / scale)
    if report is not None:
        report.append((nid, n, worst))
    return given


def _evaluate(graph: dict, inputs: dict[str, np.ndarray], contraction_rounding: str | None, decisions: dict | None = None,
              decision_report: list | None = None) -> dict[str, Any]:
    env: dict[str, Any] = dict(inputs)
    for node in topo_order(graph):
        op, nid = node["op_type"], node["id"]
        if op == "Input":
            if nid not in env:
                raise ValueError(f"Missing input value for node '{nid}'")  # environment.py:33-48
            continue
        vals = [env[i] for i in node["inputs"] if i]
        if op == "Output":
            env[nid] = vals[0] if len(vals) == 1 else tuple(vals)
        elif op == "Identity":
            env[nid] = vals[0] if vals else None
        elif op == "Constant":
            env[nid] = np.array(node["attributes"]["value"], dtype=node.get("const_dtype"))
        elif op == "Recompute":
            # _evaluate_recompute_node (evaluator.py:720-735)
            attrs = node.get("attributes") or {}
            orig = _ALIASES.get(str(attrs.get("original_op", op)), str(attrs.get("original_op", op)))
            res_node = {"id": nid, "op_type": orig, "inputs": node["inputs"], "attributes": dict(attrs.get("original_attrs") or {})}
            env[nid] = _dispatch(res_node, orig, vals, contraction_rounding)
        else:
            target = _ALIASES.get(op, op)
            env[nid] = _dispatch(node, target, vals, contraction_rounding)
            if decisions is not None and nid in decisions and target == "Greater":
                env[nid] = _replay_decision(nid, env[nid], decisions[nid], vals[0], decision_report)
    out = {}
    for oid in graph["outputs"]:
        if oid not in env:
            raise RuntimeError(f"Output node '{oid}' was never evaluated.")
        out[oid] = env[oid]
    return out


def _parse_key(text):
    """_parse_slice_string (evaluator.py:308-425): the index key an attribute string denotes."""
    import ast
    import builtins

    def node(n):
        if isinstance(n, ast.Tuple):
            return tuple(node(e) for e in n.elts)
        if isinstance(n, ast.List):
            return [node(e) for e in n.elts]
        if isinstance(n, ast.Constant):
            return n.value.decode("utf-8", errors="replace") if isinstance(n.value, bytes) else n.value
        if isinstance(n, ast.Name):
            return {"None": None, "Ellipsis": Ellipsis, "False": False, "True": True}.get(n.id)
        if isinstance(n, ast.UnaryOp):
            if isinstance(n.op, ast.USub) and isinstance(n.operand, ast.Constant) and isinstance(n.operand.value, (int, float)):
                return -n.operand.value
            return None
        if isinstance(n, ast.Call) and isinstance(n.func, ast.Name):
            if n.func.id == "slice":
                return builtins.slice(*[v if isinstance((v := node(a)), (int, float, str)) else None for a in n.args])
            if n.func.id == "array":
                return node(n.args[0])
            return None
        raise ValueError(f"Unsupported slice expression node: {type(n)}")

    return node(ast.parse(str(text), mode="eval").body)


def _dispatch(node, target, vals, contraction_rounding):
    """_dispatch_op (evaluator.py:570-593): the interpreter's own indexing / checkpoint
    handlers, else the op kernel."""
    import builtins

    kw = _kwargs(node, target)
    if target == "Slice":  # _handle_slice, evaluator.py:428-463
        arr = np.asarray(vals[0])
        if "slices" in kw:
            return arr[_parse_key(kw["slices"])]
        dim = int(kw.get("dim", 0) or 0)
        sl = [builtins.slice(None)] * arr.ndim
        sl[dim] = builtins.slice(kw.get("start"), kw.get("end"), kw.get("step", 1))
        return arr[tuple(sl)]
    if target == "GetItem":  # _handle_getitem, :466-485
        return np.asarray(vals[0])[_parse_key(kw.get("key"))]
    if target in ("IndexPut", "SetItem"):  # _handle_index_put, :488-508
        arr = np.copy(vals[0])
        arr[_parse_key(kw.get("key", kw.get("index", 0)))] = vals[1]
        return arr
    if target == "Checkpoint":  # _handle_checkpoint, :511-545
        subs = node.get("subgraphs") or {}
        sg = subs.get("body") or subs.get("subgraph") or (node.get("attributes") or {}).get("subgraph")
        if not isinstance(sg, dict) or "inputs" not in sg or "outputs" not in sg:
            raise AttributeError("Checkpoint node is missing a valid subgraph")
        res = _evaluate(sg, dict(zip(sg["inputs"], vals)), contraction_rounding)
        outs = list(sg["outputs"]) if isinstance(sg["outputs"], list) else [sg["outputs"]]
        return res[outs[0]] if len(outs) == 1 else tuple(res[o] for o in outs)
    return execute_op(target, *vals, contraction_rounding=contraction_rounding, **kw)


def evaluate_roles(graph: dict, role_inputs: dict[str, np.ndarray], contraction_rounding: str | None = None,
                   blas_layout: bool = False, decisions: dict | None = None, decision_report: list | None = None) -> dict[str, Any]:
    """Evaluate with inputs keyed by workload role; outputs keyed by output name."""
    inputs = {nid: role_inputs[r] for r, nid in graph["roles"].items()}
    res = evaluate(graph, inputs, contraction_rounding=contraction_rounding, blas_layout=blas_layout, decisions=decisions,
                   decision_report=decision_report)
    return {name: res[nid] for name, nid in graph["output_names"].items()}

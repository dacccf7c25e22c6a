"""Per-op kernels of the b200 backend (the ``execute_op`` path).

Every op takes and returns ``torch.Tensor`` values on the current CUDA device (torch
allocates; all arithmetic runs in libb200.so) with the argument meaning of the
reference numpy-backend op of the same name (cited per op). Views (Transpose, Reshape
of contiguous data, BroadcastLike) stay views; consumers that need dense data
materialise it with the elementwise copy kernel.

Numeric policy: fp32 values are computed in fp32. numpy's float64 promotion from
Python-float constants is not reproduced: those constants are applied as fp32.
Contractions use ``matmul_dtype`` (``"f32"`` exact CUDA-core path, ``"bf16"`` tcgen05
tensor cores with fp32 accumulation).
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Any, Sequence

import torch

from . import _lib as L
from .errors import BackendNotSupportedError, UnimplementedMathError

_TORCH2CODE = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.int64: L.I64, torch.bool: L.BOOL, torch.int32: L.I32,
               torch.float64: L.F64}
_FLOATS = (torch.float32, torch.bfloat16)


class Config:
    """Backend-wide numeric policy (per process)."""

    matmul_dtype: str = "f32"  # "f32" | "bf16"
    conv_dtype: str = "f32"
    device: torch.device | None = None


def device() -> torch.device:
    if Config.device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("b200 backend: no CUDA device (there is no CPU fallback)")
        Config.device = torch.device("cuda", torch.cuda.current_device())
    return Config.device


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def code(t: torch.Tensor) -> int:
    c = _TORCH2CODE.get(t.dtype)
    if c is None:
        raise BackendNotSupportedError(f"dtype {t.dtype} has no b200 kernel")
    return c


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int) -> torch.Tensor | None:
    """Device scratch of `nbytes` for an entry point that takes a workspace (None if 0)."""
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device()) if nbytes > 0 else None


def to_device(x: Any, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Host value (numpy array, scalar, tensor) -> CUDA tensor (a copy, no compute)."""
    if isinstance(x, torch.Tensor):
        t = x
    else:
        import numpy as np

        a = np.asarray(x)
        if a.dtype == np.float64:
            a = a.astype(np.float32)
        t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None and t.dtype != dtype and not t.is_cuda:
        t = t.to(dtype)
    if not t.is_cuda:
        t = t.to(device(), non_blocking=False)
    elif dtype is not None and t.dtype != dtype:
        t = cast(t, dtype)
    return t


# ----------------------------------------------------------------------------------
# elementwise programs
# ----------------------------------------------------------------------------------


def _bshape(shapes: Sequence[Sequence[int]]) -> tuple[int, ...]:
    return tuple(torch.broadcast_shapes(*[tuple(s) for s in shapes]))


def _coalesce(shape: list[int], strides: list[list[int]]) -> tuple[list[int], list[list[int]]]:
    """Drop size-1 dims and merge adjacent dims that are jointly contiguous for every operand."""
    keep = [i for i, s in enumerate(shape) if s != 1]
    shape = [shape[i] for i in keep]
    strides = [[st[i] for i in keep] for st in strides]
    if not shape:
        return [], [[] for _ in strides]
    out_shape, out_strides = [shape[0]], [[st[0]] for st in strides]
    for d in range(1, len(shape)):
        if all(st[-1] == sd[d] * shape[d] for st, sd in zip(out_strides, strides)):
            out_shape[-1] *= shape[d]
            for st, sd in zip(out_strides, strides):
                st[-1] = sd[d]
        else:
            out_shape.append(shape[d])
            for st, sd in zip(out_strides, strides):
                st.append(sd[d])
    return out_shape, out_strides


class Prog:
    """Builder for one fused elementwise program (registers are SSA-allocated)."""

    def __init__(self) -> None:
        self.ins: list[tuple[int, int, int, int, int, float]] = []
        self.inputs: list[Any] = []  # torch tensors
        self.nreg = 0

    def reg(self) -> int:
        r = self.nreg
        self.nreg += 1
        if self.nreg > L.EW_MAX_REG:
            raise UnimplementedMathError("elementwise program needs more than 16 registers")
        return r

    def load(self, t: torch.Tensor) -> int:
        for i, u in enumerate(self.inputs):
            if u is t:
                idx = i
                break
        else:
            self.inputs.append(t)
            idx = len(self.inputs) - 1
        r = self.reg()
        self.ins.append((L.EW["LOAD"], r, idx, 0, 0, 0.0))
        return r

    def imm(self, v: float) -> int:
        r = self.reg()
        self.ins.append((L.EW["IMM"], r, 0, 0, 0, float(v)))
        return r

    def op(self, name: str, a: int, b: int = 0, c: int = 0) -> int:
        r = self.reg()
        self.ins.append((L.EW[name], r, a, b, c, 0.0))
        return r

    def value(self, x: Any) -> int:
        if isinstance(x, torch.Tensor):
            if x.dim() == 0 and not x.is_cuda:
                return self.imm(float(x))
            return self.load(x)
        return self.imm(float(x))

    def run(self, outs: list[tuple[int, torch.dtype]], shape: Sequence[int] | None = None) -> list[torch.Tensor]:
        tens = [t for t in self.inputs]
        if shape is None:
            shape = _bshape([t.shape for t in tens]) if tens else ()
        shape = list(shape)
        results = [torch.empty(shape, dtype=dt, device=device()) for _, dt in outs]
        n = 1
        for s in shape:
            n *= s
        if n == 0:
            return results
        strides = []
        for t in tens:
            e = t.expand(shape) if list(t.shape) != shape else t
            strides.append(list(e.stride()) if shape else [])
        cshape, cstrides = _coalesce(shape, strides + [list(results[0].stride()) if shape else []])
        cstrides = cstrides[:-1]
        if len(cshape) > L.EW_MAX_DIM:
            raise UnimplementedMathError(f"elementwise over {len(cshape)} non-mergeable dims")
        if len(tens) > L.EW_MAX_IN or len(outs) > L.EW_MAX_OUT:
            raise UnimplementedMathError("elementwise program with too many operands")
        ins = list(self.ins) + [(L.EW["STORE"], o, r, 0, 0, 0.0) for o, (r, _) in enumerate(outs)]
        if len(ins) > L.EW_MAX_INS:
            raise UnimplementedMathError("elementwise program longer than 48 instructions")
        p = L.EwProgram()
        p.ndim = len(cshape)
        p.n_in, p.n_out, p.n_ins = len(tens), len(outs), len(ins)
        for d, s in enumerate(cshape):
            p.shape[d] = s
        for j, st in enumerate(cstrides):
            for d, s in enumerate(st):
                p.in_strides[j][d] = s
            p.in_dtype[j] = code(tens[j])
        for o, r in enumerate(results):
            p.out_dtype[o] = code(r)
        for i, (op, dst, a, b, c, imm) in enumerate(ins):
            p.ins[i].op, p.ins[i].dst, p.ins[i].a, p.ins[i].b, p.ins[i].c, p.ins[i].imm = op, dst, a, b, c, imm
        inp = (C.c_void_p * max(1, len(tens)))(*[t.data_ptr() for t in tens])
        outp = (C.c_void_p * len(results))(*[r.data_ptr() for r in results])
        L.call("b200_ew_run", C.byref(p), inp, outp, stream_ptr())
        return results


def _result_float(*xs: Any) -> torch.dtype:
    for x in xs:
        if isinstance(x, torch.Tensor) and x.dtype == torch.float32:
            return torch.float32
    for x in xs:
        if isinstance(x, torch.Tensor) and x.dtype == torch.bfloat16:
            return torch.bfloat16
    return torch.float32


def _check_float_args(name: str, *xs: Any) -> None:
    for x in xs:
        if isinstance(x, torch.Tensor) and x.dtype in (torch.int64, torch.int32):
            raise UnimplementedMathError(f"{name} on integer tensors has no b200 kernel")


def _shape_of(x: Any) -> tuple[int, ...]:
    return tuple(x.shape) if isinstance(x, torch.Tensor) else ()


def ew_binary(name: str, a: Any, b: Any, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    _check_float_args(name, a, b)
    p = Prog()
    ra, rb = p.value(a), p.value(b)
    r = p.op(name, ra, rb)
    shape = _bshape([_shape_of(a), _shape_of(b)])
    return p.run([(r, out_dtype or _result_float(a, b))], shape)[0]


def ew_unary(name: str, a: Any, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    _check_float_args(name, a)
    p = Prog()
    r = p.op(name, p.value(a))
    return p.run([(r, out_dtype or _result_float(a))], _shape_of(a))[0]


def cast(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if x.dtype == dtype:
        return x
    p = Prog()
    r = p.load(x)
    return p.run([(r, dtype)], tuple(x.shape))[0]


def contiguous(x: torch.Tensor) -> torch.Tensor:
    """Dense row-major copy through the elementwise kernel (no torch compute)."""
    if x.is_contiguous():
        return x
    p = Prog()
    r = p.load(x)
    return p.run([(r, x.dtype)], tuple(x.shape))[0]


def copy(x: torch.Tensor) -> torch.Tensor:
    """Fresh dense copy through the elementwise kernel."""
    p = Prog()
    r = p.load(x)
    return p.run([(r, x.dtype)], tuple(x.shape))[0]


def full(shape: Sequence[int], value: float, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    p = Prog()
    r = p.imm(value)
    return p.run([(r, dtype)], tuple(shape))[0]


def op_add(a, b, **_):  # numpy/eager/math_binary.py:9-20
    return ew_binary("ADD", a, b)


def op_subtract(a, b, **_):  # math_binary.py:23-36
    return ew_binary("SUB", a, b)


def op_multiply(a, b, **_):  # math_binary.py:39-51
    return ew_binary("MUL", a, b)


def op_true_divide(a, b, **_):  # math_binary.py:54-66
    return ew_binary("DIV", a, b)


def op_power(a, b, **_):  # np.power fallback
    return ew_binary("POW", a, b)


def op_maximum(a, b, **_):
    return ew_binary("MAX", a, b)


def op_minimum(a, b, **_):
    return ew_binary("MIN", a, b)


def op_greater(a, b, **_):  # numpy/eager/math_logical.py:26
    return ew_binary("GT", a, b, out_dtype=torch.bool)


def op_greater_equal(a, b, **_):
    return ew_binary("GE", a, b, out_dtype=torch.bool)


def op_less(a, b, **_):
    return ew_binary("LT", a, b, out_dtype=torch.bool)


def op_equal(a, b, **_):
    return ew_binary("EQ", a, b, out_dtype=torch.bool)


def op_where(c, a, b, **_):  # numpy/eager/math_logical.py:146
    p = Prog()
    rc, ra, rb = p.value(c), p.value(a), p.value(b)
    r = p.op("WHERE", rc, ra, rb)
    shape = _bshape([_shape_of(c), _shape_of(a), _shape_of(b)])
    return p.run([(r, _result_float(a, b))], shape)[0]


def op_negative(a, **_):
    return ew_unary("NEG", a)


def op_exp(a, **_):  # numpy/eager/math_unary.py:11
    return ew_unary("EXP", a)


def op_log(a, **_):
    return ew_unary("LOG", a)


def op_tanh(a, **_):
    return ew_unary("TANH", a)


def op_sqrt(a, **_):
    return ew_unary("SQRT", a)


def op_abs(a, **_):
    return ew_unary("ABS", a)


def op_sigmoid(a, **_):
    return ew_unary("SIGMOID", a)


def op_erf(a, **_):
    return ew_unary("ERF", a)


def op_relu(a, **_):  # numpy/eager/activation_ops.py:12
    return ew_unary("RELU", a)


def op_gelu(a, **_):  # eager/core_math_ops/math_nn.py:184-199 (tanh approximation)
    return ew_unary("GELU", a)


def op_zeros_like(a, **_):
    return full(tuple(a.shape), 0.0, a.dtype if a.dtype in _FLOATS or a.dtype == torch.bool else a.dtype)


def op_ones_like(a, **_):
    return full(tuple(a.shape), 1.0, a.dtype)


def op_cast(x, dtype=None, **_):  # numpy/eager/variable_ops.py:26-43 (bfloat16 is computed as float32 there)
    name = str(dtype).replace("DType.", "").lower() if dtype is not None else "float32"
    table = {"float32": torch.float32, "bfloat16": torch.bfloat16, "int64": torch.int64, "bool": torch.bool,
             "int32": torch.int32, "float64": torch.float32}
    if name not in table:
        raise BackendNotSupportedError(f"Cast to {dtype}")
    return cast(x, table[name])


# ----------------------------------------------------------------------------------
# views
# ----------------------------------------------------------------------------------


def op_transpose(x, axes=None, **_):  # numpy/eager/array_manipulation.py:121
    if axes is None:
        axes = list(reversed(range(x.dim())))
    return x.permute(*[int(a) for a in axes])


def op_reshape(x, shape=None, newshape=None, **_):  # numpy/eager/array_manipulation.py:87
    tgt = tuple(int(d) for d in (shape if shape is not None else newshape))
    try:
        return x.view(tgt)
    except RuntimeError:
        return contiguous(x).view(tgt)


def op_broadcast_like(src, tgt, **_):  # eager/core_math_ops/math_reduction.py:227-249
    if not isinstance(src, torch.Tensor):
        return full(tuple(tgt.shape), float(src))
    if tuple(src.shape) == tuple(tgt.shape):
        return src
    return src.expand(tuple(tgt.shape))


def op_broadcast_to(x, shape=None, **_):  # eager/core_math_ops/math_manipulation.py:423
    return x.expand(tuple(int(d) for d in shape))


def op_identity(x, *_, **__):
    return x


# ----------------------------------------------------------------------------------
# reductions
# ----------------------------------------------------------------------------------


def _norm_axes(axis, ndim: int) -> list[int]:
    if axis is None:
        return list(range(ndim))
    axes = axis if isinstance(axis, (list, tuple)) else [axis]
    return sorted({int(a) % ndim for a in axes}) if ndim else []


def reduce(x: torch.Tensor, axis, keepdims: bool, op: int) -> torch.Tensor:
    """ReduceSum/Mean/Max over ``axis`` (eager/core_math_ops/math_reduction.py:37-114)."""
    if x.dtype not in _FLOATS:
        if x.dtype == torch.bool:
            x = cast(x, torch.float32)
        else:
            raise UnimplementedMathError(f"reduction over {x.dtype}")
    axes = _norm_axes(axis, x.dim())
    if not axes:
        return x if x.dtype == torch.float32 else cast(x, torch.float32)
    xc = contiguous(x)
    shape = list(xc.shape)
    # contiguous run of axes -> a single [outer, red, inner] pass
    if axes == list(range(axes[0], axes[-1] + 1)):
        outer = math.prod(shape[: axes[0]])
        red = math.prod(shape[axes[0] : axes[-1] + 1])
        inner = math.prod(shape[axes[-1] + 1 :])
        y = torch.empty(outer * inner, dtype=torch.float32, device=device())
        wn = int(L.lib().b200_reduce_workspace_bytes(outer, red, inner))
        ws = workspace(wn)
        L.call("b200_reduce", code(xc), xc.data_ptr(), y.data_ptr(), outer, red, inner, op, _ptr(ws), wn, stream_ptr())
        out_shape = [1 if i in axes else s for i, s in enumerate(shape)] if keepdims else [s for i, s in enumerate(shape) if i not in axes]
        return y.view(out_shape)
    # otherwise one axis at a time, last first (mean = sum / count at the end)
    sub_op = L.RED_MAX if op == L.RED_MAX else L.RED_SUM
    y = xc
    for a in reversed(axes):
        y = reduce(y, a, True, sub_op)
    if op == L.RED_MEAN:
        y = ew_binary("MUL", y, 1.0 / math.prod(shape[a] for a in axes))
    if not keepdims:
        y = y.view([s for i, s in enumerate(y.shape) if i not in axes])
    return y


def op_reduce_sum(x, axis=None, keepdims=False, **_):
    return reduce(x, axis, bool(keepdims), L.RED_SUM)


def op_reduce_mean(x, axis=None, keepdims=False, **_):
    return reduce(x, axis, bool(keepdims), L.RED_MEAN)


def op_reduce_max(x, axis=None, keepdims=False, **_):
    return reduce(x, axis, bool(keepdims), L.RED_MAX)


def op_broadcast_reduce(cot, tgt, **_):  # eager/core_math_ops/math_reduction.py:192-224
    cs, ts = tuple(cot.shape), tuple(tgt.shape)
    if cs == ts:
        return cot
    res = cot
    if len(cs) > len(ts):
        res = reduce(res, list(range(len(cs) - len(ts))), False, L.RED_SUM)
    axes = [i for i, (cd, td) in enumerate(zip(res.shape, ts)) if td == 1 and cd > 1]
    if axes:
        res = reduce(res, axes, True, L.RED_SUM)
    return res


def op_numel(x, **_):  # eager/core_math_ops/math_reduction.py:156-173 (Python float)
    return float(x.numel()) if isinstance(x, torch.Tensor) else 1.0


def op_argmax(x, axis=None, **_):  # numpy/eager/math_reductions.py:129-140
    xc = contiguous(x)
    if x.dtype not in _FLOATS:
        xc = cast(xc, torch.float32)
    if axis is None:
        outer, red, inner, out_shape = 1, xc.numel(), 1, ()
    else:
        a = int(axis) % xc.dim()
        shape = list(xc.shape)
        outer, red, inner = math.prod(shape[:a]), shape[a], math.prod(shape[a + 1 :])
        out_shape = tuple(shape[:a] + shape[a + 1 :])
    if red == 0:
        raise ValueError("attempt to get argmax of an empty sequence")
    y = torch.empty(out_shape, dtype=torch.int64, device=device())
    L.call("b200_argmax", code(xc), xc.data_ptr(), y.data_ptr(), outer, red, inner, stream_ptr())
    return y


def _last_axis(x: torch.Tensor, axis) -> bool:
    return axis is None or int(axis) % max(1, x.dim()) == x.dim() - 1


def _softmax(x, axis, log):
    if not _last_axis(x, axis):
        a = int(axis) % x.dim()
        perm = [i for i in range(x.dim()) if i != a] + [a]
        inv = [perm.index(i) for i in range(x.dim())]
        return _softmax(contiguous(x.permute(*perm)), -1, log).permute(*inv)
    xc = contiguous(cast(x, torch.float32))
    cols = xc.shape[-1] if xc.dim() else 1
    rows = xc.numel() // max(1, cols)
    y = torch.empty_like(xc)
    L.call("b200_softmax_rows", xc.data_ptr(), None, y.data_ptr(), None, rows, cols, 1 if log else 0, stream_ptr())
    return y


def op_softmax(x, axis=-1, **_):  # numpy/eager/math_advanced/math_signal.py:450-467
    return _softmax(x, axis, False)


def op_log_softmax(x, axis=-1, **_):  # numpy/eager/math_advanced/math_log_exp.py:87-104
    return _softmax(x, axis, True)


def _ln_args(x, axis):
    if not _last_axis(x, axis):
        raise UnimplementedMathError("LayerNorm over a non-last axis")
    xc = contiguous(cast(x, torch.float32))
    cols = xc.shape[-1]
    return xc, xc.numel() // cols, cols


def _opt(t):
    return None if t is None else contiguous(cast(t, torch.float32))


def layer_norm(x, gamma=None, beta=None, eps=1e-5, axis=-1, f32=True, bf16=False):
    """LayerNorm with fp32 and/or bf16 outputs: returns (y_f32 or None, y_bf16 or None)."""
    xc, rows, cols = _ln_args(x, axis)
    g, b = _opt(gamma), _opt(beta)
    y = torch.empty_like(xc) if f32 else None
    yb = torch.empty(xc.shape, dtype=torch.bfloat16, device=device()) if bf16 else None
    L.call("b200_layernorm_rows", xc.data_ptr(), _ptr(g), _ptr(b), _ptr(y), _ptr(yb), rows, cols, float(eps), stream_ptr())
    return y, yb


def op_layer_norm(x, gamma=None, beta=None, eps=1e-5, axis=-1, **kw):  # numpy/eager/nn_ops.py:219-241
    return layer_norm(x, gamma, beta, float(kw.get("epsilon", eps)), axis)[0]


def op_layer_norm_input_grad(dy, x, gamma=None, eps=1e-5, axis=-1, **kw):  # numpy/eager/nn_ops.py:244-273
    eps = float(kw.get("epsilon", eps))
    xc, rows, cols = _ln_args(x, axis)
    dyc = contiguous(cast(dy.expand(xc.shape), torch.float32))
    g = _opt(gamma)
    dx = torch.empty_like(xc)
    L.call("b200_layernorm_input_grad_rows", dyc.data_ptr(), xc.data_ptr(), _ptr(g), dx.data_ptr(), None, rows, cols, eps,
           stream_ptr())
    return dx


def _ln_param(dy, x, eps, axis, which):
    xc, rows, cols = _ln_args(x, axis)
    dyc = contiguous(cast(dy.expand(xc.shape), torch.float32))
    out = torch.empty(cols, dtype=torch.float32, device=device())
    dg = out if which == "gamma" else None
    db = out if which == "beta" else None
    wn = int(L.lib().b200_layernorm_param_grad_workspace_bytes(rows, cols))
    ws = workspace(wn)
    L.call("b200_layernorm_param_grad", dyc.data_ptr(), xc.data_ptr(), _ptr(dg), _ptr(db), rows, cols, float(eps), _ptr(ws), wn,
           stream_ptr())
    return out


def op_layer_norm_gamma_grad(dy, x, eps=1e-5, axis=-1, **kw):  # numpy/eager/nn_ops.py:276-297
    return _ln_param(dy, x, float(kw.get("epsilon", eps)), axis, "gamma")


def op_layer_norm_beta_grad(dy, axis=-1, **_):  # numpy/eager/nn_ops.py:300-318
    return reduce(dy, list(range(dy.dim() - 1)), False, L.RED_SUM) if dy.dim() > 1 else cast(dy, torch.float32)


# ----------------------------------------------------------------------------------
# indexing
# ----------------------------------------------------------------------------------


def _int_indices(indices: Any) -> torch.Tensor:
    """Indices as an int64 CUDA tensor (numpy accepts any integer dtype; floats raise)."""
    t = indices if isinstance(indices, torch.Tensor) else to_device(indices)
    if t.dtype == torch.int64:
        return t
    if t.dtype in (torch.int32, torch.int16, torch.int8, torch.uint8):
        return cast(t, torch.int64) if t.dtype == torch.int32 else cast(t.to(torch.int32), torch.int64)
    raise IndexError("arrays used as indices must be of integer type")


def gather_along_axis(x: torch.Tensor, indices: Any, axis: Any) -> torch.Tensor:
    """np.take_along_axis(x, indices, axis): the other axes of x and indices broadcast;
    axis=None gathers from x flattened (1-d indices). Any dtype, bits copied unchanged."""
    idx = _int_indices(indices)
    if axis is None:
        if idx.dim() != 1:
            raise ValueError("when axis=None, `indices` must have a single dimension.")
        x = contiguous(x).reshape(-1)
        axis = 0
    nd = x.dim()
    if nd == 0 or idx.dim() != nd:
        raise ValueError("`indices` and `arr` must have the same number of dimensions")
    ax = int(axis)
    if not -nd <= ax < nd:
        raise ValueError(f"axis {ax} is out of bounds for array of dimension {nd}")
    ax %= nd
    if nd > L.GATHER_MAX_DIM:
        raise UnimplementedMathError(f"Gather over {nd} dimensions (at most {L.GATHER_MAX_DIM})")
    shape = []
    for d in range(nd):
        if d == ax:
            shape.append(idx.shape[d])
        else:
            shape.append(tuple(torch.broadcast_shapes((x.shape[d],), (idx.shape[d],)))[0])
    xs = [x.stride(d) if (d == ax or x.shape[d] == shape[d]) else 0 for d in range(nd)]
    is_ = [idx.stride(d) if idx.shape[d] == shape[d] else 0 for d in range(nd)]
    y = torch.empty(tuple(shape), dtype=x.dtype, device=device())
    import ctypes as C

    A = C.c_int64 * nd
    L.call("b200_gather_axis", x.element_size(), x.data_ptr(), A(*xs), idx.data_ptr(), A(*is_), y.data_ptr(), A(*shape), nd,
           ax, int(x.shape[ax]), stream_ptr())
    return y


def op_take_along_axis(x, indices, axis=-1, **_):  # numpy/eager/advanced_indexing.py:163-177
    y = gather_along_axis(x, indices, axis)
    # bf16 graph values stand for the reference's fp32 values: the gathered result is fp32
    return cast(y, torch.float32) if y.dtype == torch.bfloat16 else y


def op_gather(*args, **kwargs):  # numpy/eager/indexing.py:312-332
    """Gather(tensor, dim, index) = np.take_along_axis(tensor, index, axis=dim), arguments
    positional in that order or as the keywords tensor / dim / index."""
    t = args[0] if len(args) > 0 else kwargs.get("tensor")
    dim = args[1] if len(args) > 1 else kwargs.get("dim")
    index = args[2] if len(args) > 2 else kwargs.get("index")
    if isinstance(dim, torch.Tensor):
        dim = int(dim.item())
    elif dim is not None:
        dim = int(dim)
    return op_take_along_axis(t, index, axis=dim)


_ONEHOT_DTYPES = {"float32": torch.float32, "float64": torch.float64, "float": torch.float64, "double": torch.float64,
                  "int64": torch.int64, "int": torch.int64, "int32": torch.int32, "bool": torch.bool}


def _one_hot_dtype(dtype: Any) -> torch.dtype:
    if dtype is None or dtype is float:
        return torch.float64
    if dtype is int:
        return torch.int64
    if dtype is bool:
        return torch.bool
    name = getattr(dtype, "__name__", None) if isinstance(dtype, type) else None
    key = str(name or dtype).replace("np.", "").replace("numpy.", "").replace("torch.", "").replace("<class '", "").rstrip("'>")
    if key not in _ONEHOT_DTYPES:
        raise UnimplementedMathError(f"OneHot to dtype {dtype!r} has no b200 kernel")
    return _ONEHOT_DTYPES[key]


def op_one_hot(*args, **kwargs):  # numpy/eager/math_advanced/math_general.py:710-736
    """OneHot(indices, depth, on_value=1, off_value=0, axis=-1, dtype=float):
    eye(depth)[indices] * (on - off) + off, the class axis moved to ``axis``. A float64
    result (the default dtype) is computed in fp64 and stored as fp32, the backend's
    floating-point type (host float64 arrays are uploaded as fp32 too)."""
    indices = args[0] if args else None
    depth = args[1] if len(args) > 1 else kwargs.get("depth")
    if indices is None or depth is None:
        return None
    on_value = float(kwargs.get("on_value", 1))
    off_value = float(kwargs.get("off_value", 0))
    axis = kwargs.get("axis", -1)
    want = _one_hot_dtype(kwargs.get("dtype", float))
    depth = int(depth.item()) if isinstance(depth, torch.Tensor) else int(depth)
    if depth < 0:
        raise ValueError("negative dimensions are not allowed")
    idx = contiguous(_int_indices(indices))
    nd = idx.dim() + 1
    pos = int(axis)
    if not -nd <= pos < nd:
        raise ValueError(f"destination {pos} is out of bounds for array of dimension {nd}")
    pos %= nd
    outer = 1
    for d in idx.shape[:pos]:
        outer *= int(d)
    inner = 1
    for d in idx.shape[pos:]:
        inner *= int(d)
    shape = tuple(idx.shape[:pos]) + (depth,) + tuple(idx.shape[pos:])
    kdt = torch.float64 if want == torch.float64 else want
    y = torch.empty(shape, dtype=kdt, device=device())
    L.call("b200_one_hot", idx.data_ptr(), y.data_ptr(), code(y), outer, depth, inner, on_value, off_value, stream_ptr())
    return cast(y, torch.float32) if kdt == torch.float64 else y


def op_scatter_add(inp, index, src, dim=0, **_):  # numpy/eager/advanced_indexing.py:309-326
    if int(dim) % inp.dim() != inp.dim() - 1:
        raise UnimplementedMathError("ScatterAdd on a non-last axis")
    base = contiguous(cast(inp, torch.float32))
    cols = base.shape[-1]
    rows = base.numel() // cols
    k = index.shape[-1]
    ic = contiguous(index)
    sc = contiguous(cast(src.expand(index.shape), torch.float32))
    y = torch.empty_like(base)
    L.call("b200_scatter_add_last", base.data_ptr(), ic.data_ptr(), sc.data_ptr(), y.data_ptr(), rows, cols, k, stream_ptr())
    return y


def op_take(a, indices, axis=None, **_):  # np.take fallback (numpy/eager/__init__.py:114-125)
    if axis is None or int(axis) != 0:
        raise UnimplementedMathError("Take supports axis=0 (row gather)")
    tc = contiguous(a)
    V = tc.shape[0]
    D = tc.numel() // max(1, V)
    ic = contiguous(indices)
    y = torch.empty(tuple(ic.shape) + tuple(tc.shape[1:]), dtype=tc.dtype, device=device())
    L.call("b200_take_rows", code(tc), tc.data_ptr(), ic.data_ptr(), y.data_ptr(), ic.numel(), V, D, stream_ptr())
    return y


def op_tensor_scatter_add(tensor, indices, updates, **_):  # numpy/eager/math_scatter.py:39-60
    if indices.dim() != 2 or indices.shape[-1] != 1:
        raise UnimplementedMathError("TensorScatterAdd supports [n, 1] row indices")
    y = copy(cast(tensor, torch.float32))
    V = y.shape[0]
    D = y.numel() // max(1, V)
    uc = contiguous(cast(updates, torch.float32))
    ic = contiguous(indices)
    wn = int(L.lib().b200_scatter_add_rows_workspace_bytes(ic.shape[0], V))
    ws = workspace(wn)
    L.call("b200_scatter_add_rows", uc.data_ptr(), ic.data_ptr(), y.data_ptr(), ic.shape[0], V, D, 1, _ptr(ws), wn,
           stream_ptr())
    return y


# ----------------------------------------------------------------------------------
# contractions
# ----------------------------------------------------------------------------------


# bf16 copies of fp32 GEMM operands made during one plan run, keyed by the source
# storage: two GEMMs reading the same value (e.g. dA and dB both read the masked
# cotangent) share one cast. Cleared by the executor at the start and end of each run.
_CAST_CACHE: dict = {}


def clear_cast_cache() -> None:
    _CAST_CACHE.clear()


def register_cast(src: torch.Tensor, dst: torch.Tensor) -> None:
    """Record ``dst`` (written by the kernel that produced ``src``) as the ``dst.dtype``
    copy of the dense tensor ``src``; ``cast_operand`` then reuses it."""
    _CAST_CACHE[(src.data_ptr(), src.numel(), src.dtype, dst.dtype)] = (src, dst)


def cast_operand(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Layout-preserving cast: a strided view of a dense tensor is cast in storage order
    (coalesced) and re-viewed, never materialised through the strided path."""
    if t.dtype == dtype:
        return t
    base = t._base if t._base is not None else t
    if not base.is_contiguous():
        return cast(t, dtype)
    key = (base.data_ptr(), base.numel(), base.dtype, dtype)
    hit = _CAST_CACHE.get(key)
    if hit is not None and hit[0] is base:
        cb = hit[1]
    else:
        cb = cast(base, dtype)
        # the entry keeps `base` alive, so its storage cannot be recycled under the key
        _CAST_CACHE[key] = (base, cb)
    return cb.as_strided(t.size(), t.stride(), t.storage_offset() - base.storage_offset())


def _tc_ok(t: torch.Tensor) -> bool:
    st = t.stride()
    return t.data_ptr() % 16 == 0 and (
        (st[-1] == 1 and (st[-2] * 2) % 16 == 0) or (st[-2] == 1 and (st[-1] * 2) % 16 == 0)
    )


def _gemm_operand(t: torch.Tensor, ab: torch.dtype) -> torch.Tensor:
    t = cast_operand(t, ab)
    if ab != torch.bfloat16 or _tc_ok(t):
        return t
    # tcgen05 path needs one unit stride and 16-byte aligned rows: try both dense layouts
    rm = contiguous(t)
    if _tc_ok(rm):
        return rm
    cm = contiguous(t.transpose(-1, -2)).transpose(-1, -2)
    if _tc_ok(cm):
        return cm
    return None  # no TMA-legal layout (e.g. N = 10): caller uses the CUDA-core kernel


def gemm(a: torch.Tensor, b: torch.Tensor, *, bias: torch.Tensor | None = None, epilogue: int = L.EPI_NONE,
         alpha: float = 1.0, out_dtype: torch.dtype = torch.float32, want_mask: bool = False,
         ab_dtype: torch.dtype | None = None, act_bf16: bool = False, resid: torch.Tensor | None = None):
    """numpy-style matmul of a [..., M, K] and b [..., K, N] with broadcast batch dims.

    Returns C = act(alpha a.b + bias) [, mask]. With ``act_bf16`` it returns
    (pre, act_in_bf16[, mask]): C holds the pre-activation and the activation is written
    in bf16 by the same epilogue. ``resid`` (fp32, C's shape; no activation, mask or
    alpha): C = (a.b + bias) + resid, the residual Add in the epilogue of the bf16 kernel,
    else as a separate Add."""
    if resid is not None:
        fused = (not act_bf16 and not want_mask and epilogue == L.EPI_NONE and alpha == 1.0 and out_dtype == torch.float32
                 and resid.dtype == torch.float32)
        if fused:
            y = _gemm_residual(a, b, bias, resid, ab_dtype)
            if y is not None:
                return y
        y = gemm(a, b, bias=bias, epilogue=epilogue, alpha=alpha, out_dtype=out_dtype, want_mask=want_mask,
                 ab_dtype=ab_dtype, act_bf16=act_bf16)
        if want_mask or act_bf16:
            raise UnimplementedMathError("gemm residual with a mask or a dual output")
        return op_add(y, resid)
    if act_bf16:
        return _gemm_dual(a, b, bias=bias, epilogue=epilogue, alpha=alpha, out_dtype=out_dtype, want_mask=want_mask,
                          ab_dtype=ab_dtype)
    if ab_dtype is None:
        ab_dtype = torch.bfloat16 if Config.matmul_dtype == "bf16" else torch.float32
    squeeze_m = squeeze_n = False
    if a.dim() == 1:
        a, squeeze_m = a.unsqueeze(0), True
    if b.dim() == 1:
        b, squeeze_n = b.unsqueeze(-1), True
    M, K = a.shape[-2], a.shape[-1]
    K2, N = b.shape[-2], b.shape[-1]
    if K != K2:
        raise ValueError(f"matmul: shapes {tuple(a.shape)} and {tuple(b.shape)} not aligned")
    batch_shape = _bshape([a.shape[:-2], b.shape[:-2]])
    Z = math.prod(batch_shape)
    # fold a batched A with a shared 2-D B into one tall GEMM
    if b.dim() == 2 and a.dim() > 2 and a.is_contiguous():
        y = gemm(a.reshape(-1, K), b, bias=bias, epilogue=epilogue, alpha=alpha, out_dtype=out_dtype,
                 want_mask=want_mask, ab_dtype=ab_dtype)
        ys = (y[0] if want_mask else y).view(*a.shape[:-1], N)
        res = (ys, y[1].view(*a.shape[:-1], N)) if want_mask else ys
        return res
    act_bf16 = None
    A = _gemm_operand(a, ab_dtype)
    B = _gemm_operand(b, ab_dtype) if A is not None else None
    if A is None or B is None:
        # TMA needs 16-byte aligned rows; tiny/odd GEMMs (e.g. a 128 -> 10 classifier) run
        # on the CUDA-core kernel in fp32, which is at least as precise as bf16 math
        ab_dtype = torch.float32
        A, B = cast(a, torch.float32), cast(b, torch.float32)
    if (ab_dtype == torch.bfloat16 and Z == 1 and bias is None and not want_mask and epilogue == L.EPI_NONE
            and alpha == 1.0):
        S = _split_k(M, N, K)
        if S > 1:
            return _gemm_split_k(A.reshape(M, K), B.reshape(K, N), S, out_dtype).view(*batch_shape, M, N)
    C_ = torch.empty(*batch_shape, M, N, dtype=out_dtype, device=device())
    mask = torch.empty(*batch_shape, M, N, dtype=torch.bool, device=device()) if want_mask else None
    bc = None if bias is None else contiguous(cast(bias, torch.float32))
    if bc is not None and bc.numel() != N:
        raise UnimplementedMathError("gemm bias must be a length-N vector")
    if not (Z and M and N):
        pass
    else:
        nb = len(batch_shape)
        sa = list(A.expand(*batch_shape, M, K).stride()[:nb]) if A.dim() > 2 else [0] * nb
        sb = list(B.expand(*batch_shape, K, N).stride()[:nb]) if B.dim() > 2 else [0] * nb
        sc = list(C_.stride()[:nb])
        # coalesce the batch dims jointly (drop size-1 dims, merge contiguous neighbours)
        dims = [(sz, x, y, z) for sz, x, y, z in zip(batch_shape, sa, sb, sc) if sz != 1]
        merged: list[list[int]] = []
        for sz, x, y, z in dims:
            if merged and merged[-1][1] == x * sz and merged[-1][2] == y * sz and merged[-1][3] == z * sz:
                merged[-1] = [merged[-1][0] * sz, x, y, z]
            else:
                merged.append([sz, x, y, z])
        if ab_dtype == torch.bfloat16 and len(merged) <= 2:
            while len(merged) < 2:
                merged.insert(0, [1, 0, 0, 0])
            (bo, sao, sbo, sco), (bi, sai, sbi, sci) = merged
            L.call("b200_gemm_batched2", code(A), code(C_), A.data_ptr(), B.data_ptr(), C_.data_ptr(), bo, bi, M, N, K, sao,
                   sai, A.stride(-2), A.stride(-1), sbo, sbi, B.stride(-2), B.stride(-1), sco, sci, N, float(alpha), _ptr(bc),
                   int(epilogue), _ptr(mask), _ptr(act_bf16), stream_ptr())
        else:
            if len(merged) > 1:
                A = contiguous(A.expand(*batch_shape, M, K))
                B = contiguous(B.expand(*batch_shape, K, N))
                sA = M * K if A.dim() > 2 else 0
                sB = K * N if B.dim() > 2 else 0
            else:
                sA = merged[0][1] if merged else 0
                sB = merged[0][2] if merged else 0
            L.call("b200_gemm", code(A), code(C_), A.data_ptr(), B.data_ptr(), C_.data_ptr(), Z, M, N, K, sA, A.stride(-2),
                   A.stride(-1), sB, B.stride(-2), B.stride(-1), M * N, N, float(alpha), _ptr(bc), int(epilogue), _ptr(mask),
                   stream_ptr())
    if squeeze_m:
        C_ = C_.squeeze(-2)
    if squeeze_n:
        C_ = C_.squeeze(-1)
    return (C_, mask) if want_mask else C_


def _batch2(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, batch_shape: tuple) -> list | None:
    """The batch dims of A, B (broadcast) and C coalesced into at most two levels:
    [(b_out, sA_out, sB_out, sC_out), (b_in, sA_in, sB_in, sC_in)], or None."""
    nb = len(batch_shape)
    M, K = A.shape[-2], A.shape[-1]
    N = B.shape[-1]
    sa = list(A.expand(*batch_shape, M, K).stride()[:nb]) if A.dim() > 2 else [0] * nb
    sb = list(B.expand(*batch_shape, K, N).stride()[:nb]) if B.dim() > 2 else [0] * nb
    sc = list(C.stride()[:nb])
    dims = [(sz, x, y, z) for sz, x, y, z in zip(batch_shape, sa, sb, sc) if sz != 1]
    merged: list[list[int]] = []
    for sz, x, y, z in dims:
        if merged and merged[-1][1] == x * sz and merged[-1][2] == y * sz and merged[-1][3] == z * sz:
            merged[-1] = [merged[-1][0] * sz, x, y, z]
        else:
            merged.append([sz, x, y, z])
    if len(merged) > 2:
        return None
    while len(merged) < 2:
        merged.insert(0, [1, 0, 0, 0])
    return merged


def gemm_softmax_rows(a: torch.Tensor, b: torch.Tensor, scale: torch.Tensor | None, f32: bool, bf16: bool):
    """softmax(scale * a.b) over the last axis, with the scores kept on chip (one tcgen05
    kernel: the GEMM's 128 x N accumulator in TMEM, the row softmax in its epilogue).
    Returns (y fp32 or None, y bf16 or None). Falls back to the GEMM + the row-softmax
    kernel when the operands' layout or sizes are outside the fused kernel."""
    A, B = _gemm_operand(a, torch.bfloat16), _gemm_operand(b, torch.bfloat16)
    M, K, N = a.shape[-2], a.shape[-1], b.shape[-1]
    batch_shape = _bshape([a.shape[:-2], b.shape[:-2]])
    shape = (*batch_shape, M, N)
    y = torch.empty(shape, dtype=torch.float32, device=device()) if f32 else None
    yb = torch.empty(shape, dtype=torch.bfloat16, device=device()) if bf16 else None
    sc = contiguous(cast(scale, torch.float32)) if scale is not None else None
    ref = y if y is not None else yb
    lv = _batch2(A, B, ref, batch_shape) if (A is not None and B is not None) else None
    if lv is not None and N <= 512 and K <= 128:
        (bo, sao, sbo, sco), (bi, sai, sbi, sci) = lv
        try:
            L.call("b200_gemm_softmax_rows", A.data_ptr(), B.data_ptr(), bo, bi, M, N, K, sao, sai, A.stride(-2), A.stride(-1),
                   sbo, sbi, B.stride(-2), B.stride(-1), _ptr(sc), _ptr(y), _ptr(yb), sco, sci, N, stream_ptr())
            return y, yb
        except UnimplementedMathError:
            pass
    x = gemm(a, b, ab_dtype=torch.bfloat16)
    xc = contiguous(x)
    L.call("b200_softmax_rows", xc.data_ptr(), _ptr(sc), _ptr(y), _ptr(yb), xc.numel() // N, N, 0, stream_ptr())
    return y, yb


def gemm_softmax_bwd_rows(a: torch.Tensor, b: torch.Tensor, y: torch.Tensor, scale: torch.Tensor | None, f32: bool, bf16: bool):
    """scale * y * (G - rowsum(G * y)) with G = a.b kept on chip (the softmax VJP in the
    epilogue of the tcgen05 GEMM that makes G). Returns (dx fp32 or None, dx bf16 or None);
    falls back to the GEMM + the softmax-VJP kernel outside the fused kernel's range."""
    A, B = _gemm_operand(a, torch.bfloat16), _gemm_operand(b, torch.bfloat16)
    M, K, N = a.shape[-2], a.shape[-1], b.shape[-1]
    batch_shape = _bshape([a.shape[:-2], b.shape[:-2]])
    shape = (*batch_shape, M, N)
    dx = torch.empty(shape, dtype=torch.float32, device=device()) if f32 else None
    dxb = torch.empty(shape, dtype=torch.bfloat16, device=device()) if bf16 else None
    sc = contiguous(cast(scale, torch.float32)) if scale is not None else None
    yc = contiguous(y) if y.dtype in (torch.float32, torch.bfloat16) else contiguous(cast(y, torch.float32))
    ref = dx if dx is not None else dxb
    lv = _batch2(A, B, ref, batch_shape) if (A is not None and B is not None) else None
    if lv is not None and N <= 512 and K <= 128 and tuple(yc.shape) == tuple(shape):
        (bo, sao, sbo, sco), (bi, sai, sbi, sci) = lv
        try:
            L.call("b200_gemm_softmax_bwd_rows", A.data_ptr(), B.data_ptr(), bo, bi, M, N, K, sao, sai, A.stride(-2),
                   A.stride(-1), sbo, sbi, B.stride(-2), B.stride(-1), _ptr(sc), code(yc), yc.data_ptr(), _ptr(dx), _ptr(dxb),
                   sco, sci, N, stream_ptr())
            return dx, dxb
        except UnimplementedMathError:
            pass
    g = contiguous(gemm(a, b, ab_dtype=torch.bfloat16))
    yf = contiguous(cast(yc, torch.float32))
    L.call("b200_softmax_bwd_rows", yf.data_ptr(), g.data_ptr(), _ptr(sc), _ptr(dx), _ptr(dxb), g.numel() // N, N, stream_ptr())
    return dx, dxb


_SMS: dict[int, int] = {}


def _num_sms() -> int:
    d = torch.cuda.current_device()
    if d not in _SMS:
        _SMS[d] = int(torch.cuda.get_device_properties(d).multi_processor_count)
    return _SMS[d]


def _split_k(M: int, N: int, K: int) -> int:
    """Number of K chunks for a GEMM whose output tiles cannot fill the GPU (weight
    gradients: small M x N, K = tokens). Chunks are equal, multiples of 64."""
    tiles = -(-M // 128) * -(-N // (256 if N > 128 else 128))
    sms = _num_sms()
    if tiles * 2 > sms or K < 4096:
        return 1
    want = max(1, min(sms // tiles, K // 2048))
    for S in range(want, 1, -1):
        if K % S == 0 and (K // S) % 64 == 0:
            return S
    return 1


def _gemm_split_k(A: torch.Tensor, B: torch.Tensor, S: int, out_dtype: torch.dtype) -> torch.Tensor:
    """C = A.B as S partial products over equal K chunks (one batched tcgen05 launch, the
    chunk index as the batch level) and a fixed-order sum of the partials."""
    M, K = A.shape
    N = B.shape[1]
    Kc = K // S
    part = torch.empty(S, M, N, dtype=torch.float32, device=device())
    # chunk s of A is columns [s Kc, (s+1) Kc), of B rows [s Kc, (s+1) Kc)
    L.call("b200_gemm_batched2", code(A), code(part), A.data_ptr(), B.data_ptr(), part.data_ptr(), 1, S, M, N, Kc, 0,
           Kc * A.stride(1), A.stride(0), A.stride(1), 0, Kc * B.stride(0), B.stride(0), B.stride(1), 0, M * N, N, 1.0, None,
           L.EPI_NONE, None, None, stream_ptr())
    C_ = torch.empty(M, N, dtype=torch.float32, device=device())
    # S chunks summed in order (M N columns fill the GPU: no further split)
    L.call("b200_reduce", code(part), part.data_ptr(), C_.data_ptr(), 1, S, M * N, L.RED_SUM, None, 0, stream_ptr())
    return C_ if out_dtype == torch.float32 else cast(C_, out_dtype)


def _gemm_residual(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None, resid: torch.Tensor,
                   ab_dtype: torch.dtype | None) -> torch.Tensor | None:
    """(a.b + bias) + resid for a [..., M, K] (contiguous or 2-D) and a 2-D b [K, N] on the
    tcgen05 kernel, or None when the operands do not fit it."""
    if ab_dtype is None:
        ab_dtype = torch.bfloat16 if Config.matmul_dtype == "bf16" else torch.float32
    if ab_dtype != torch.bfloat16 or a.dim() < 2 or b.dim() != 2 or (a.dim() > 2 and not a.is_contiguous()):
        return None
    K, N = b.shape
    if a.shape[-1] != K:
        raise ValueError(f"matmul: shapes {tuple(a.shape)} and {tuple(b.shape)} not aligned")
    out_shape = (*a.shape[:-1], N)
    if tuple(resid.shape) != out_shape or not resid.is_contiguous():
        return None
    a2 = a.reshape(-1, K)
    M = a2.shape[0]
    A = _gemm_operand(a2, torch.bfloat16)
    B = _gemm_operand(b, torch.bfloat16) if A is not None else None
    if A is None or B is None:
        return None
    bc = None if bias is None else contiguous(cast(bias, torch.float32))
    if bc is not None and bc.numel() != N:
        return None
    C_ = torch.empty(out_shape, dtype=torch.float32, device=device())
    if M and N:
        L.call("b200_gemm_batched2_residual", A.data_ptr(), B.data_ptr(), C_.data_ptr(), 1, 1, M, N, K, 0, 0, A.stride(-2),
               A.stride(-1), 0, 0, B.stride(-2), B.stride(-1), 0, 0, N, _ptr(bc), resid.data_ptr(), stream_ptr())
    return C_


def gemm_out(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, out2: torch.Tensor | None = None,
             ab_dtype: torch.dtype | None = None) -> bool:
    """a.b written into the preallocated view ``out`` (any batch / row strides, unit
    column stride) and optionally its bf16 twin ``out2`` (same element strides), by the
    tcgen05 kernel with <= 2 batch levels. Returns False, writing nothing, when the
    operands or ``out`` do not fit that path."""
    if ab_dtype is None:
        ab_dtype = torch.bfloat16 if Config.matmul_dtype == "bf16" else torch.float32
    if ab_dtype != torch.bfloat16 or a.dim() < 2 or b.dim() < 2:
        return False
    M, K = a.shape[-2], a.shape[-1]
    K2, N = b.shape[-2], b.shape[-1]
    if K != K2:
        raise ValueError(f"matmul: shapes {tuple(a.shape)} and {tuple(b.shape)} not aligned")
    batch_shape = _bshape([a.shape[:-2], b.shape[:-2]])
    if tuple(out.shape) != (*batch_shape, M, N) or out.stride(-1) != 1 or out.stride(-2) < N:
        return False
    if out2 is not None and (out2.dtype != torch.bfloat16 or out2.stride() != out.stride() or out2.shape != out.shape):
        return False
    A = _gemm_operand(a, torch.bfloat16)
    B = _gemm_operand(b, torch.bfloat16) if A is not None else None
    if A is None or B is None:
        return False
    nb = len(batch_shape)
    sa = list(A.expand(*batch_shape, M, K).stride()[:nb]) if A.dim() > 2 else [0] * nb
    sb = list(B.expand(*batch_shape, K, N).stride()[:nb]) if B.dim() > 2 else [0] * nb
    sc = list(out.stride()[:nb])
    merged: list[list[int]] = []
    for sz, x, y, z in zip(batch_shape, sa, sb, sc):
        if sz == 1:
            continue
        if merged and merged[-1][1] == x * sz and merged[-1][2] == y * sz and merged[-1][3] == z * sz:
            merged[-1] = [merged[-1][0] * sz, x, y, z]
        else:
            merged.append([sz, x, y, z])
    if len(merged) > 2:
        return False
    while len(merged) < 2:
        merged.insert(0, [1, 0, 0, 0])
    (bo, sao, sbo, sco), (bi, sai, sbi, sci) = merged
    if math.prod(batch_shape) and M and N:
        L.call("b200_gemm_batched2", code(A), code(out), A.data_ptr(), B.data_ptr(), out.data_ptr(), bo, bi, M, N, K, sao, sai,
               A.stride(-2), A.stride(-1), sbo, sbi, B.stride(-2), B.stride(-1), sco, sci, out.stride(-2), 1.0, None,
               L.EPI_NONE, None, _ptr(out2), stream_ptr())
    return True


def _gemm_dual(a, b, *, bias, epilogue, alpha, out_dtype, want_mask, ab_dtype):
    """pre = alpha a.b + bias and act(pre) in bf16 from one tcgen05 epilogue; other
    layouts compute pre first and apply the activation with an elementwise program."""
    if ab_dtype is None:
        ab_dtype = torch.bfloat16 if Config.matmul_dtype == "bf16" else torch.float32
    squeeze = a.dim() == 1 or b.dim() == 1
    A = _gemm_operand(a, ab_dtype) if ab_dtype == torch.bfloat16 and not squeeze else None
    B = _gemm_operand(b, ab_dtype) if A is not None else None
    if A is not None and B is not None and A.dim() == 2 and B.dim() == 2:
        M, K = A.shape
        N = B.shape[1]
        pre = torch.empty(M, N, dtype=out_dtype, device=device())
        act = torch.empty(M, N, dtype=torch.bfloat16, device=device())
        mask = torch.empty(M, N, dtype=torch.bool, device=device()) if want_mask else None
        bc = None if bias is None else contiguous(cast(bias, torch.float32))
        if bc is not None and bc.numel() != N:
            raise UnimplementedMathError("gemm bias must be a length-N vector")
        if M and N:
            L.call("b200_gemm_batched2", code(A), code(pre), A.data_ptr(), B.data_ptr(), pre.data_ptr(), 1, 1, M, N, K, 0, 0,
                   A.stride(0), A.stride(1), 0, 0, B.stride(0), B.stride(1), 0, 0, N, float(alpha), _ptr(bc), int(epilogue),
                   _ptr(mask), act.data_ptr(), stream_ptr())
        return (pre, act, mask) if want_mask else (pre, act)
    res = gemm(a, b, bias=bias, epilogue=L.EPI_NONE, alpha=alpha, out_dtype=torch.float32, ab_dtype=ab_dtype)
    fn = {L.EPI_RELU: op_relu, L.EPI_GELU: op_gelu}.get(int(epilogue))
    act = cast(fn(res) if fn else res, torch.bfloat16)
    if want_mask:
        return cast(res, out_dtype), act, op_greater(res, 0.0)
    return cast(res, out_dtype), act


def op_matmul(a, b, transpose_a=False, transpose_b=False, **_):  # eager/core_math_ops/math_matrix.py:21-44
    if transpose_a:
        a = a.transpose(-1, -2)
    if transpose_b:
        b = b.transpose(-1, -2)
    return gemm(a, b)


def _conv_pads(in_hw, k_hw, s_hw, padding, out_hw):
    # numpy/eager/conv.py:590-633 (_compute_conv2d_padding_values, dilation 1)
    if isinstance(padding, str) and padding.upper() == "SAME":
        ph = max(0, (out_hw[0] - 1) * s_hw[0] + k_hw[0] - in_hw[0])
        pw = max(0, (out_hw[1] - 1) * s_hw[1] + k_hw[1] - in_hw[1])
        return ph // 2, pw // 2
    if isinstance(padding, str) and padding.upper() == "VALID":
        return 0, 0
    raise UnimplementedMathError(f"Conv2D padding {padding!r}")


def _stride2(stride):
    if isinstance(stride, int):
        return stride, stride
    return int(stride[0]), int(stride[1])


def _conv_out_hw(in_hw, k_hw, s_hw, padding):
    if isinstance(padding, str) and padding.upper() == "SAME":
        return -(-in_hw[0] // s_hw[0]), -(-in_hw[1] // s_hw[1])
    return (in_hw[0] - k_hw[0]) // s_hw[0] + 1, (in_hw[1] - k_hw[1]) // s_hw[1] + 1


def _conv_dt() -> int:
    return L.BF16 if Config.conv_dtype == "bf16" else L.F32


def _conv_call(kind: int, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, dims: tuple, relu: bool = False,
               mask: torch.Tensor | None = None, fp32_out: bool = True) -> None:
    """fp32 math: exact CUDA-core kernels; bf16 math: tcgen05 implicit GEMMs (operand tiles
    gathered straight into shared memory), or tcgen05 GEMMs over staged operands for shapes
    the implicit GEMM does not take. ``relu`` (forward) and ``mask`` (input gradient:
    ``dx * (mask > 0)``) are epilogues of the implicit GEMM only. ``fp32_out=False`` (fused
    epilogues only, for results whose every reader takes the channels-last copy) leaves
    ``out`` unwritten and writes only the copy."""
    names = ("b200_conv2d_fwd", "b200_conv2d_dgrad", "b200_conv2d_wgrad")
    fused = relu or mask is not None
    if Config.conv_dtype != "bf16":
        if fused:
            raise UnimplementedMathError("fused convolution epilogues need bf16 convolution math")
        L.call(names[kind], L.F32, a.data_ptr(), b.data_ptr(), out.data_ptr(), *dims, stream_ptr())
        return
    if L.lib().b200_conv2d_igemm_supported(kind, *dims):
        N, Cc, H, W, O = dims[:5]
        # the packed weight image (fwd / dgrad) or the split partials (wgrad); the
        # channels-last copies come from channels_last() and are shared within a run
        ws_bytes = int(L.lib().b200_conv2d_igemm_workspace_bytes(kind, *dims))
        ws = torch.empty(max(256, ws_bytes), dtype=torch.uint8, device=device())
        ws_ptr = ws.data_ptr()
        # a planner-fused convolution (ReLU / mask epilogue) feeds the next convolution of
        # the chain: its epilogue also writes the result's channels-last copy, kept for it
        twin = None
        if fused and kind in (0, 1):
            cp = _rup(O if kind == 0 else Cc, 8)
            twin = torch.empty((out.shape[0], out.shape[2], out.shape[3], cp), dtype=torch.bfloat16, device=device())
        if not fp32_out and twin is None:
            raise UnimplementedMathError("a convolution result without fp32 output needs a fused epilogue")
        optr = out.data_ptr() if fp32_out else None
        if kind == 0:
            L.call("b200_conv2d_fwd_igemm", a.data_ptr(), channels_last(a, _rup(Cc, 8)).data_ptr(), b.data_ptr(),
                   optr, _ptr(twin), *dims, 1 if relu else 0, ws_ptr, ws_bytes, stream_ptr())
        elif kind == 1:
            # a ReLU output's own channels-last copy is the exact mask (nonzero where > 0)
            mcl = relu_copy(mask, _rup(Cc, 8)) if mask is not None else None
            L.call("b200_conv2d_dgrad_igemm", a.data_ptr(), channels_last(a, _rup(O, 8)).data_ptr(), b.data_ptr(),
                   None if mcl is not None else _ptr(mask), _ptr(mcl), int(mcl.shape[3]) if mcl is not None else 0,
                   optr, _ptr(twin), *dims, ws_ptr, ws_bytes, stream_ptr())
        if twin is not None:
            _CAST_CACHE[(out.data_ptr(), out.numel(), out.dtype, out._version, ("channels_last", twin.shape[3]))] = (
                out, twin, "relu" if (kind == 0 and relu) else "")
        if kind == 2:
            L.call("b200_conv2d_wgrad_igemm", a.data_ptr(), channels_last(a, _rup(Cc, 8)).data_ptr(), b.data_ptr(),
                   channels_last(b, _rup(O, 64)).data_ptr(), out.data_ptr(), *dims, ws_ptr, ws_bytes, stream_ptr())
        return
    if fused:
        raise UnimplementedMathError("fused convolution epilogue for a shape outside the implicit GEMM")
    ws_bytes = int(L.lib().b200_conv2d_tc_workspace_bytes(kind, *dims))
    ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=device())
    L.call(names[kind] + "_tc", a.data_ptr(), b.data_ptr(), out.data_ptr(), *dims, ws.data_ptr(), ws_bytes, stream_ptr())


def _rup(v: int, m: int) -> int:
    return (int(v) + m - 1) // m * m


def channels_last(t: torch.Tensor, cp: int) -> torch.Tensor:
    """bf16 channels-last copy [N, H, W, cp] (channels >= C zero) of a dense fp32 NCHW
    tensor, the layout the implicit-GEMM convolutions copy their tiles from. Within a plan
    run the copy is kept beside the bf16 operand casts, so the forward convolution and the
    weight gradient of the same activation (or the input and weight gradients of the same
    cotangent) share one."""
    key = (t.data_ptr(), t.numel(), t.dtype, t._version, ("channels_last", cp))
    hit = _CAST_CACHE.get(key)
    if hit is not None and hit[0] is t:
        return hit[1]
    N, Cc, H, W = (int(v) for v in t.shape)
    y = torch.empty((N, H, W, cp), dtype=torch.bfloat16, device=device())
    L.call("b200_conv2d_channels_last", t.data_ptr(), y.data_ptr(), N, Cc, H * W, cp, stream_ptr())
    _CAST_CACHE[key] = (t, y)
    return y


def relu_copy(t: torch.Tensor, cp: int) -> torch.Tensor | None:
    """The channels-last copy that a fused ReLU convolution wrote beside ``t`` in this run
    (nonzero exactly where ``t`` > 0), or None."""
    hit = _CAST_CACHE.get((t.data_ptr(), t.numel(), t.dtype, t._version, ("channels_last", cp)))
    if hit is not None and hit[0] is t and len(hit) > 2 and hit[2] == "relu":
        return hit[1]
    return None


def conv_fused_ok(kind: int, x_shape: tuple, w_shape: tuple, stride, padding, out_hw: tuple | None = None) -> bool:
    """Whether a fused conv epilogue (forward ReLU, input-gradient mask) has a kernel."""
    if Config.conv_dtype != "bf16" or len(x_shape) != 4 or len(w_shape) != 4:
        return False
    s = _stride2(stride)
    N, Cc, H, W = (int(v) for v in x_shape)
    O, _, KH, KW = (int(v) for v in w_shape)
    try:
        OH, OW = out_hw if out_hw is not None else _conv_out_hw((H, W), (KH, KW), s, padding)
        pt, pl = _conv_pads((H, W), (KH, KW), s, padding, (OH, OW))
    except UnimplementedMathError:
        return False
    return bool(L.lib().b200_conv2d_igemm_supported(kind, N, Cc, H, W, O, KH, KW, OH, OW, s[0], s[1], pt, pl))


def _check_conv_attrs(groups, dilation):
    if int(groups or 1) != 1:
        raise UnimplementedMathError("grouped Conv2D")
    d = _stride2(dilation or 1)
    if d != (1, 1):
        raise UnimplementedMathError("dilated Conv2D")


def op_conv2d(x, w, stride=(1, 1), padding="SAME", groups=1, dilation=1, relu=False, fp32_out=True,
              **kw):  # numpy/eager/conv.py:462-489
    """Conv2D; ``relu=True`` returns relu(Conv2D(x, w)) from the same kernel (the Relu node
    that follows it in the graph, fused). ``fp32_out=False`` (with ``relu``): the returned
    tensor is left unwritten and only its channels-last copy exists, for a planner that has
    checked that every reader takes that copy."""
    _check_conv_attrs(groups, kw.get("dilations", dilation))
    s = _stride2(kw.get("strides", stride))
    xc, wc = contiguous(cast(x, torch.float32)), contiguous(cast(w, torch.float32))
    N, Cc, H, W = xc.shape
    O, _, KH, KW = wc.shape
    OH, OW = _conv_out_hw((H, W), (KH, KW), s, padding)
    pt, pl = _conv_pads((H, W), (KH, KW), s, padding, (OH, OW))
    y = torch.empty(N, O, OH, OW, dtype=torch.float32, device=device())
    _conv_call(0, xc, wc, y, (N, Cc, H, W, O, KH, KW, OH, OW, s[0], s[1], pt, pl), relu=bool(relu), fp32_out=fp32_out)
    return y


def op_conv2d_input_grad(dy, w, stride=(1, 1), padding="SAME", target_shape=None, groups=1, dilation=1, mask=None,
                         fp32_out=True, **kw):
    """Conv2DInputGrad (numpy/eager/conv.py:634-697); with ``mask`` (fp32, the input's shape)
    it returns dx * (mask > 0): the Multiply by the ReLU VJP's Greater(pre, 0) mask, fused
    (read from the mask's own channels-last copy when a fused ReLU convolution wrote one).
    ``fp32_out=False`` (with ``mask``) as for op_conv2d."""
    _check_conv_attrs(groups, kw.get("dilations", dilation))
    s = _stride2(kw.get("strides", stride))
    dyc, wc = contiguous(cast(dy, torch.float32)), contiguous(cast(w, torch.float32))
    N, Cc, H, W = (int(v) for v in target_shape)
    O, _, KH, KW = wc.shape
    OH, OW = dyc.shape[2], dyc.shape[3]
    pt, pl = _conv_pads((H, W), (KH, KW), s, padding, (OH, OW))
    dx = torch.empty(N, Cc, H, W, dtype=torch.float32, device=device())
    if mask is not None:
        mask = contiguous(cast(mask, torch.float32))
        if tuple(mask.shape) != (N, Cc, H, W):
            raise ValueError(f"conv input-gradient mask shape {tuple(mask.shape)} != {(N, Cc, H, W)}")
    _conv_call(1, dyc, wc, dx, (N, Cc, H, W, O, KH, KW, OH, OW, s[0], s[1], pt, pl), mask=mask, fp32_out=fp32_out)
    return dx


def op_conv2d_weight_grad(x, dy, stride=(1, 1), padding="SAME", target_shape=None, groups=1, dilation=1, **kw):
    # numpy/eager/conv.py:699-764
    _check_conv_attrs(groups, kw.get("dilations", dilation))
    s = _stride2(kw.get("strides", stride))
    xc, dyc = contiguous(cast(x, torch.float32)), contiguous(cast(dy, torch.float32))
    O, Cc, KH, KW = (int(v) for v in target_shape)
    N, _, H, W = xc.shape
    OH, OW = dyc.shape[2], dyc.shape[3]
    pt, pl = _conv_pads((H, W), (KH, KW), s, padding, (OH, OW))
    dw = torch.empty(O, Cc, KH, KW, dtype=torch.float32, device=device())
    _conv_call(2, xc, dyc, dw, (N, Cc, H, W, O, KH, KW, OH, OW, s[0], s[1], pt, pl))
    return dw


def op_conv2d_bias_grad(dy, **_):  # numpy/eager/conv.py:766-779
    return reduce(dy, [0, 2, 3], False, L.RED_SUM)


# ----------------------------------------------------------------------------------
# collectives
# ----------------------------------------------------------------------------------


def op_all_reduce(x, op_type="sum", **_):  # numpy/eager/distributed.py:205-225
    import torch.distributed as dist

    if str(op_type).lower() not in ("sum", "add"):
        raise UnimplementedMathError(f"AllReduce op {op_type}")
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        y = copy(x)
        dist.all_reduce(y)
        return y
    return x


# ---- optimizer update steps ---------------------------------------------------------
_OPT_KIND = {"ApplyAdam": 0, "ApplyAdagrad": 1, "ApplyFtrl": 2, "ApplyRMSProp": 3}


def apply_optimizer(op: str, params, states, grads, lr=None, out=None):
    """One launch per 128 tensors of ``op`` (ApplyAdam / ApplyAdagrad / ApplyFtrl /
    ApplyRMSProp, the numpy backend's formulas, ``numpy/eager/optimizers_ops.py``).

    ``params`` / ``grads`` are lists of fp32 tensors, ``states`` a list of per-tensor
    tuples of state tensors (Adam: m, v; Adagrad: accum; FTRL: accum, linear; RMSProp: ms,
    mom). Results go to ``out`` (per-tensor tuples of param, states; the inputs themselves
    for an in-place step) or to new tensors. Returns the per-tensor result tuples."""
    kind = _OPT_KIND[op]
    if lr is None:
        lr = float(L.lib().b200_optimizer_default_lr(kind))
    nst = 1 if kind == 1 else 2
    ps = [contiguous(cast(to_device(p), torch.float32)) for p in params]
    gs = [contiguous(cast(to_device(g), torch.float32)) for g in grads]
    ss = [[contiguous(cast(to_device(x), torch.float32)) for x in st] for st in states]
    for p, g, st in zip(ps, gs, ss):
        if len(st) != nst or g.shape != p.shape or any(x.shape != p.shape for x in st):
            raise ValueError(f"{op}: param, states and grad must have one shape ({nst} state arrays)")
    if out is None:
        out = [tuple(torch.empty_like(p) for _ in range(1 + nst)) for p in ps]
    n = len(ps)
    P = C.c_void_p * n
    ptr = lambda ts: P(*[t.data_ptr() for t in ts])  # noqa: E731
    s2 = ptr([st[1] for st in ss]) if nst == 2 else None
    s2o = ptr([o[2] for o in out]) if nst == 2 else None
    sizes = (C.c_int64 * n)(*[p.numel() for p in ps])
    L.call("b200_apply_optimizer_f32", kind, n, ptr(ps), ptr([st[0] for st in ss]), s2, ptr(gs), ptr([o[0] for o in out]),
           ptr([o[1] for o in out]), s2o, sizes, float(lr), stream_ptr())
    return out


def _opt_op(op: str):
    def run(param, *rest, lr=None, **_):
        states, grad = rest[:-1], rest[-1]
        return tuple(apply_optimizer(op, [param], [states], [grad], lr=lr)[0])

    run.__name__ = "op_" + op
    return run


OPS: dict[str, Any] = {
    "ApplyAdam": _opt_op("ApplyAdam"),  # numpy/eager/optimizers_ops.py:11-35
    "ApplyAdagrad": _opt_op("ApplyAdagrad"),  # :38-59
    "ApplyFtrl": _opt_op("ApplyFtrl"),  # :62-83
    "ApplyRMSProp": _opt_op("ApplyRMSProp"),  # :86-103
    "Add": op_add,
    "Subtract": op_subtract,
    "Multiply": op_multiply,
    "TrueDivide": op_true_divide,
    "Power": op_power,
    "Maximum": op_maximum,
    "Minimum": op_minimum,
    "Greater": op_greater,
    "GreaterEqual": op_greater_equal,
    "Less": op_less,
    "Equal": op_equal,
    "Where": op_where,
    "Negative": op_negative,
    "Exp": op_exp,
    "Log": op_log,
    "Tanh": op_tanh,
    "Sqrt": op_sqrt,
    "Abs": op_abs,
    "Sigmoid": op_sigmoid,
    "Erf": op_erf,
    "Relu": op_relu,
    "Gelu": op_gelu,
    "GELU": op_gelu,
    "ZerosLike": op_zeros_like,
    "OnesLike": op_ones_like,
    "Cast": op_cast,
    "Transpose": op_transpose,
    "Reshape": op_reshape,
    "BroadcastLike": op_broadcast_like,
    "BroadcastTo": op_broadcast_to,
    "Identity": op_identity,
    "ReduceSum": op_reduce_sum,
    "ReduceMean": op_reduce_mean,
    "ReduceMax": op_reduce_max,
    "BroadcastReduce": op_broadcast_reduce,
    "Numel": op_numel,
    "Argmax": op_argmax,
    "Softmax": op_softmax,
    "LogSoftmax": op_log_softmax,
    "LayerNorm": op_layer_norm,
    "LayerNormInputGrad": op_layer_norm_input_grad,
    "LayerNormGammaGrad": op_layer_norm_gamma_grad,
    "LayerNormBetaGrad": op_layer_norm_beta_grad,
    "TakeAlongAxis": op_take_along_axis,
    "Gather": op_gather,
    "OneHot": op_one_hot,
    "ScatterAdd": op_scatter_add,
    "Take": op_take,
    "TensorScatterAdd": op_tensor_scatter_add,
    "Matmul": op_matmul,
    "BatchMatMul": op_matmul,
    "Conv2D": op_conv2d,
    "Conv2DInputGrad": op_conv2d_input_grad,
    "Conv2DWeightGrad": op_conv2d_weight_grad,
    "Conv2DBiasGrad": op_conv2d_bias_grad,
    "AllReduce": op_all_reduce,
    "NcclAllReduce": op_all_reduce,
    "Clone": lambda x, *_, **__: copy(x) if isinstance(x, torch.Tensor) else x,  # numpy/eager/__init__.py:128-145
}

from . import fused_nodes as _fused_nodes  # noqa: E402  (fusion-pass node types, registered into OPS)

_fused_nodes.register(OPS)

# reference aliases (interpreter/evaluator.py:771-791)
ALIASES = {"Sub": "Subtract", "Mul": "Multiply", "Div": "TrueDivide", "Neg": "Negative", "Pow": "Power", "MatMul": "Matmul",
           "Expand": "BroadcastTo", "Permute": "Transpose"}


def execute_op(op_type: str, *args, **kwargs):
    """Run one op on the GPU; unknown ops raise UnimplementedMathError (no fallback)."""
    name = ALIASES.get(op_type, op_type)
    fn = OPS.get(name)
    if fn is None:
        raise UnimplementedMathError(f"Operation {op_type} is not implemented in the b200 backend.")
    args = [to_device(a) if _is_array_like(a) else a for a in args]
    return fn(*args, **kwargs)


def _is_array_like(a: Any) -> bool:
    if isinstance(a, torch.Tensor):
        return not a.is_cuda
    try:
        import numpy as np

        return isinstance(a, np.ndarray)
    except Exception:  # noqa: BLE001
        return False

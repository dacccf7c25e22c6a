"""ctypes binding of libb200.so (the C ABI declared in include/b200.h).

The library is loaded from this package directory. There is no fallback: when the
shared object is missing or a CUDA device is absent, ``lib()`` raises, and every op of
the backend fails loudly instead of computing anywhere else.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

from .errors import BackendNotSupportedError, UnimplementedMathError

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libb200.so")

F32, BF16, I64, BOOL, I32, F64 = 0, 1, 2, 3, 4, 5
GATHER_MAX_DIM = 8
OK, ERR_ARG, ERR_DTYPE, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED = 0, 1, 2, 3, 4, 5

EW_MAX_IN, EW_MAX_OUT, EW_MAX_DIM, EW_MAX_INS, EW_MAX_REG = 8, 4, 6, 48, 16
EPI_NONE, EPI_RELU, EPI_GELU = 0, 1, 2
RED_SUM, RED_MEAN, RED_MAX = 0, 1, 2

# elementwise opcodes (enum b200_ew_op)
EW = {
    name: i
    for i, name in enumerate(
        "LOAD STORE IMM ADD SUB MUL DIV NEG EXP LOG TANH SQRT POW MAX MIN GT GE LT EQ WHERE RELU GELU ABS SIGMOID ERF MOV RECIP FMA".split()
    )
}


class EwIns(C.Structure):
    _fields_ = [
        ("op", C.c_uint8),
        ("dst", C.c_uint8),
        ("a", C.c_uint8),
        ("b", C.c_uint8),
        ("c", C.c_uint8),
        ("pad0", C.c_uint8),
        ("pad1", C.c_uint8),
        ("pad2", C.c_uint8),
        ("imm", C.c_float),
    ]


class EwProgram(C.Structure):
    _fields_ = [
        ("ndim", C.c_int32),
        ("n_in", C.c_int32),
        ("n_out", C.c_int32),
        ("n_ins", C.c_int32),
        ("shape", C.c_int64 * EW_MAX_DIM),
        ("in_strides", (C.c_int64 * EW_MAX_DIM) * EW_MAX_IN),
        ("in_dtype", C.c_int32 * EW_MAX_IN),
        ("out_dtype", C.c_int32 * EW_MAX_OUT),
        ("ins", EwIns * EW_MAX_INS),
    ]


_P, _I64, _I32, _F32 = C.c_void_p, C.c_int64, C.c_int, C.c_float

SIGNATURES = {
    "b200_abi_version": ([], C.c_int),
    "b200_last_error": ([], C.c_char_p),
    "b200_launch_count": ([], C.c_uint64),
    "b200_check_device_error": ([_P], C.c_int),
    "b200_ew_run": ([C.POINTER(EwProgram), C.POINTER(_P), C.POINTER(_P), _P], C.c_int),
    "b200_reduce": ([_I32, _P, _P, _I64, _I64, _I64, _I32, _P, C.c_size_t, _P], C.c_int),
    "b200_reduce_workspace_bytes": ([_I64, _I64, _I64], C.c_size_t),
    "b200_argmax": ([_I32, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_softmax": ([_P, _P, _I64, _I64, _I32, _P], C.c_int),
    "b200_gelu_bwd_colsum_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_gelu_bwd_colsum": ([_P, _P, _P, _P, _P, _I64, _I64, _P, C.c_size_t, _P], C.c_int),
    "b200_layernorm_bwd_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_layernorm_bwd_rows": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _F32, _P, C.c_size_t, _P], C.c_int),
    "b200_layernorm_rows": ([_P, _P, _P, _P, _P, _I64, _I64, _F32, _P], C.c_int),
    "b200_layernorm_input_grad_rows": ([_P, _P, _P, _P, _P, _I64, _I64, _F32, _P], C.c_int),
    "b200_softmax_rows": ([_P, _P, _P, _P, _I64, _I64, _I32, _P], C.c_int),
    "b200_softmax_bwd_rows": ([_P, _P, _P, _P, _P, _I64, _I64, _P], C.c_int),
    "b200_layernorm": ([_P, _P, _P, _P, _I64, _I64, _F32, _P], C.c_int),
    "b200_layernorm_input_grad": ([_P, _P, _P, _P, _I64, _I64, _F32, _P], C.c_int),
    "b200_layernorm_param_grad": ([_P, _P, _P, _P, _I64, _I64, _F32, _P, C.c_size_t, _P], C.c_int),
    "b200_layernorm_param_grad_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_take_along_last": ([_P, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_scatter_add_last": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_take_rows": ([_I32, _P, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_gather_axis": ([_I32, _P, C.POINTER(_I64), _P, C.POINTER(_I64), _P, C.POINTER(_I64), _I32, _I32, _I64, _P], C.c_int),
    "b200_copy_strided": ([_I32, _P, C.POINTER(_I64), _P, C.POINTER(_I64), C.POINTER(_I64), _I32, _P], C.c_int),
    "b200_one_hot": ([_P, _P, _I32, _I64, _I64, _I64, C.c_double, C.c_double, _P], C.c_int),
    "b200_gemm_softmax_rows": ([_P, _P] + [_I64] * 13 + [_P, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_gemm_softmax_bwd_rows": ([_P, _P] + [_I64] * 13 + [_P, _I32, _P, _P, _P, _I64, _I64, _I64, _P], C.c_int),
    "b200_scatter_add_rows": ([_P, _P, _P, _I64, _I64, _I64, _I32, _P, C.c_size_t, _P], C.c_int),
    "b200_scatter_add_rows_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_gemm": (
        [_I32, _I32, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F32, _P, _I32, _P, _P],
        C.c_int,
    ),
    "b200_gemm_batched2": (
        [_I32, _I32, _P, _P, _P] + [_I64] * 16 + [_F32, _P, _I32, _P, _P, _P],
        C.c_int,
    ),
    "b200_rowfused_fwd_bwd_noalloc": ([_P] * 13 + [_I64, _I64, _F32, _P], C.c_int),
    "b200_peer_allreduce_blocks": ([_I64], C.c_int),
    "b200_peer_allreduce_f32": ([_P, _I64, _P, _I64, C.c_int, C.c_int, _P, _P, _I64, _F32, _P], C.c_int),
    "b200_memset_async": ([_P, C.c_int, C.c_size_t, _P], C.c_int),
    "b200_peer_allreduce_tensors_f32": ([C.c_int, _P, _P, _P, _I64, C.c_int, C.c_int, _P, _P, _I64, _F32, C.c_int, _P, _P, _P,
                                         _F32, _P], C.c_int),
    "b200_optimizer_default_lr": ([C.c_int], C.c_double),
    "b200_apply_optimizer_f32": ([C.c_int, C.c_int, _P, _P, _P, _P, _P, _P, _P, _P, _F32, _P], C.c_int),
    "b200_peer_allreduce_apply_f32": ([_P, _I64, _P, _I64, C.c_int, C.c_int, _P, _P, _I64, _F32, C.c_int, C.c_int, _P, _P,
                                       _P, _P, _F32, _P], C.c_int),
    "b200_rowfused_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_rowfused_fwd_bwd": ([_P] * 13 + [_I64, _I64, _F32, _P, C.c_size_t, _P], C.c_int),
    "b200_mask_mul_colsum_workspace_bytes": ([_I64, _I64], C.c_size_t),
    "b200_mask_mul_colsum": ([_P, _P, _P, _P, _P, _I64, _I64, _P, C.c_size_t, _P], C.c_int),
    "b200_logsoftmax_pick": ([_I32, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _P], C.c_int),
    "b200_conv2d_tc_workspace_bytes": ([_I32] + [_I64] * 13, C.c_size_t),
    "b200_conv2d_fwd_tc": ([_P, _P, _P] + [_I64] * 13 + [_P, C.c_size_t, _P], C.c_int),
    "b200_conv2d_dgrad_tc": ([_P, _P, _P] + [_I64] * 13 + [_P, C.c_size_t, _P], C.c_int),
    "b200_conv2d_wgrad_tc": ([_P, _P, _P] + [_I64] * 13 + [_P, C.c_size_t, _P], C.c_int),
    "b200_conv2d_igemm_supported": ([_I32] + [_I64] * 13, C.c_int),
    "b200_conv2d_igemm_workspace_bytes": ([_I32] + [_I64] * 13, C.c_size_t),
    "b200_conv2d_channels_last": ([_P, _P] + [_I64] * 4 + [_P], C.c_int),
    "b200_conv2d_fwd_igemm": ([_P, _P, _P, _P, _P] + [_I64] * 13 + [_I32, _P, C.c_size_t, _P], C.c_int),
    "b200_gemm_batched2_residual": ([_P, _P, _P] + [_I64] * 16 + [_P, _P, _P], C.c_int),
    "b200_conv2d_dgrad_igemm": ([_P, _P, _P, _P, _P, _I64, _P, _P] + [_I64] * 13 + [_P, C.c_size_t, _P], C.c_int),
    "b200_conv2d_wgrad_igemm": ([_P, _P, _P, _P, _P] + [_I64] * 13 + [_P, C.c_size_t, _P], C.c_int),
    "b200_conv2d_fwd": ([_I32, _P, _P, _P] + [_I64] * 13 + [_P], C.c_int),
    "b200_conv2d_dgrad": ([_I32, _P, _P, _P] + [_I64] * 13 + [_P], C.c_int),
    "b200_conv2d_wgrad": ([_I32, _P, _P, _P] + [_I64] * 13 + [_P], C.c_int),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """dlopen libb200.so and attach the C signatures (no CUDA work happens here)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libb200.so not found at {path}: build it with `python -m b200.build` "
                    "(the b200 backend has no CPU fallback)"
                )
            lib = C.CDLL(path)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
        return _lib


def lib() -> C.CDLL:
    return _lib if _lib is not None else load()


def last_error() -> str:
    msg = lib().b200_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str = "") -> None:
    """Map a C-ABI status to the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc == ERR_ARG:
        raise ValueError(msg)
    if rc == ERR_DTYPE:
        raise BackendNotSupportedError(msg)
    if rc == ERR_UNSUPPORTED:
        raise UnimplementedMathError(msg)
    if rc == ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def launch_count() -> int:
    return int(lib().b200_launch_count())

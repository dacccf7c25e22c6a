"""The interpreter's own indexing nodes on device values: Slice, GetItem, IndexPut /
SetItem (``interpreter/evaluator.py:428-508``).

The reference applies ``arr[key]`` / ``arr[key] = v`` to backend values, with ``key``
parsed from the node's ``slices`` / ``key`` attribute string by a small AST reader
(``evaluator.py:308-425``: tuples, lists, constants, ``None`` / ``Ellipsis`` /
``True`` / ``False``, unary minus, ``slice(...)`` and ``array(...)`` calls). Here the same
keys become views of the device tensor (no kernel), or one gather kernel:

* integers, ``slice`` with a positive step, ``None`` and ``...`` are views
  (``narrow`` / ``select`` / ``as_strided`` / ``unsqueeze``: metadata only);
* a slice with a negative step, and one integer list / array (numpy advanced indexing
  on a single axis), go through ``b200_gather_axis``;
* IndexPut clones the base with the copy kernel (``execute_op("Clone")``, as the
  reference does at ``evaluator.py:506``), then writes the value, broadcast and cast to
  the base's dtype, into the view of the key with ``b200_copy_strided``.

Keys with several advanced indices or boolean masks raise ``UnimplementedMathError``.
"""

from __future__ import annotations

import ast
import builtins
import ctypes as C
from typing import Any

import torch

from . import _lib as L
from .errors import UnimplementedMathError


# ------------------------------------------------------------------------------------
# key parsing (the grammar of evaluator.py:308-425)
# ------------------------------------------------------------------------------------
def _node(n: ast.AST) -> Any:
    if isinstance(n, ast.Tuple):
        return tuple(_node(e) for e in n.elts)
    if isinstance(n, ast.List):
        return [_node(e) for e in n.elts]
    if isinstance(n, ast.Constant):
        v = n.value
        return v.decode("utf-8", errors="replace") if isinstance(v, bytes) else v
    if isinstance(n, ast.Name):
        return {"None": None, "Ellipsis": Ellipsis, "False": False, "True": True}.get(n.id)
    if isinstance(n, ast.UnaryOp):
        if isinstance(n.op, ast.USub) and isinstance(n.operand, ast.Constant) and isinstance(n.operand.value, (int, float)):
            return -n.operand.value
        return None
    if isinstance(n, ast.Call):
        if not isinstance(n.func, ast.Name):
            return None
        if n.func.id == "slice":
            args = [v if isinstance((v := _node(a)), (int, float, str)) else None for a in n.args]
            return builtins.slice(*args)
        if n.func.id == "array":
            return _node(n.args[0])
        return None
    raise ValueError(f"Unsupported slice expression node: {type(n)}")


def parse_key(s: Any) -> Any:
    """The key a Slice / GetItem / IndexPut attribute string denotes."""
    return _node(ast.parse(str(s), mode="eval").body)


def _as_index(v: Any, what: str) -> int | None:
    if v is None:
        return None
    if isinstance(v, bool):
        raise UnimplementedMathError(f"boolean {what} in an index key")
    if isinstance(v, (int, float)):
        if isinstance(v, float) and not v.is_integer():
            raise TypeError("slice indices must be integers or None or have an __index__ method")
        return int(v)
    if isinstance(v, str):
        try:
            return int(v)
        except ValueError as e:
            raise TypeError("slice indices must be integers or None or have an __index__ method") from e
    raise TypeError(f"unsupported {what} {v!r}")


# ------------------------------------------------------------------------------------
# applying a key
# ------------------------------------------------------------------------------------
def _expand_key(key: Any, ndim: int) -> list[Any]:
    items = list(key) if isinstance(key, tuple) else [key]
    n_ell = sum(1 for k in items if k is Ellipsis)
    if n_ell > 1:
        raise IndexError("an index can only have a single ellipsis ('...')")
    consumed = sum(1 for k in items if k is not None and k is not Ellipsis)
    if consumed > ndim:
        raise IndexError(f"too many indices for array: array is {ndim}-dimensional, but {consumed} were indexed")
    out: list[Any] = []
    for k in items:
        if k is Ellipsis:
            out.extend([builtins.slice(None)] * (ndim - consumed))
        else:
            out.append(k)
    out.extend([builtins.slice(None)] * (ndim - sum(1 for k in out if k is not None)))
    return out


def _index_tensor(values: list[int]) -> torch.Tensor:
    from . import ops

    return ops.to_device(torch.tensor(values, dtype=torch.int64))


def _gather_dim(t: torch.Tensor, d: int, idx: torch.Tensor) -> torch.Tensor:
    """t with axis d replaced by t.take(idx, axis=d) (idx of any shape)."""
    from . import ops

    k = idx.numel()
    shape = list(t.shape)
    view_shape = [1] * t.dim()
    view_shape[d] = k
    flat = ops.contiguous(idx).reshape(view_shape)
    expand = list(shape)
    expand[d] = k
    y = ops.gather_along_axis(t, flat.expand(expand), d)
    return y.reshape(shape[:d] + list(idx.shape) + shape[d + 1 :])


def _basic_view(t: torch.Tensor, items: list[Any]) -> tuple[torch.Tensor, list[tuple[int, Any]]]:
    """Apply ints, positive-step slices and None as views; returns the view and the
    deferred gathers (output axis, slice with negative step or integer list)."""
    out = t
    d = 0  # current axis in `out`
    deferred: list[tuple[int, Any]] = []
    for k in items:
        if k is None:
            out = out.unsqueeze(d)
            d += 1
            continue
        n = out.shape[d]
        if isinstance(k, builtins.slice):
            start, stop, step = (_as_index(k.start, "slice start"), _as_index(k.stop, "slice stop"),
                                 _as_index(k.step, "slice step"))
            if step == 0:
                raise ValueError("slice step cannot be zero")
            s0, s1, st = builtins.slice(start, stop, step).indices(n)
            length = len(range(s0, s1, st))
            if st > 0:
                out = out.narrow(d, s0, length) if length else out.narrow(d, 0, 0)
                if st > 1 and length:
                    sizes = list(out.shape)
                    strides = list(out.stride())
                    strides[d] *= st
                    out = out.as_strided(sizes, strides, out.storage_offset())
            else:
                deferred.append((d, list(range(s0, s1, st))))
            d += 1
            continue
        if isinstance(k, (list, tuple)) or isinstance(k, torch.Tensor):
            vals = k.tolist() if isinstance(k, torch.Tensor) else list(k)
            if any(isinstance(v, bool) for v in vals):
                raise UnimplementedMathError("boolean mask keys have no b200 kernel")
            deferred.append((d, vals))
            d += 1
            continue
        i = _as_index(k, "index")
        if not -n <= i < n:
            raise IndexError(f"index {i} is out of bounds for axis {d} with size {n}")
        out = out.select(d, i % n)
    return out, deferred


def get_item(x: torch.Tensor, key: Any, cache: dict | None = None) -> torch.Tensor:
    """numpy-style ``x[key]`` on a device tensor (views where numpy makes views).
    ``cache`` keeps the device index arrays of the key between calls, so a plan step
    uploads them once (outside any CUDA graph capture) and replays without copies."""
    if not isinstance(x, torch.Tensor):
        raise UnimplementedMathError("indexing a non-tensor value")
    items = _expand_key(key, x.dim())
    n_adv = sum(1 for k in items if isinstance(k, (list, tuple, torch.Tensor)))
    if n_adv > 1:
        raise UnimplementedMathError("keys with more than one advanced index have no b200 kernel")
    if n_adv and any(isinstance(k, (int, float, str)) and not isinstance(k, bool) for k in items):
        # numpy broadcasts integer indices together with the array index and may move the
        # result axes to the front; not supported here
        raise UnimplementedMathError("keys mixing an integer index with an array index have no b200 kernel")
    out, deferred = _basic_view(x, items)
    for d, vals in deferred:
        n = out.shape[d]
        norm = []
        for v in vals:
            v = _as_index(v, "index")
            if not -n <= v < n:
                raise IndexError(f"index {v} is out of bounds for axis {d} with size {n}")
            norm.append(v % n)
        ck = (d, n, tuple(norm))
        idx = cache.get(ck) if cache is not None else None
        if idx is None:
            idx = _index_tensor(norm) if norm else torch.empty(0, dtype=torch.int64, device=out.device)
            if cache is not None:
                cache[ck] = idx
        out = _gather_dim(out, d, idx)
    return out


def slice_node(x: torch.Tensor, kwargs: dict[str, Any], cache: dict | None = None) -> torch.Tensor:
    """_handle_slice (evaluator.py:428-463): ``slices`` string, else dim / start / end / step."""
    if "slices" in kwargs:
        return get_item(x, parse_key(kwargs["slices"]), cache)
    raw_dim = kwargs.get("dim", 0)
    dim = int(raw_dim) if raw_dim is not None else 0
    start, end, step = kwargs.get("start"), kwargs.get("end"), kwargs.get("step", 1)
    start = start if isinstance(start, (int, float, str)) else None
    end = end if isinstance(end, (int, float, str)) else None
    step = step if isinstance(step, (int, float, str)) else None
    rank = x.dim() if isinstance(x, torch.Tensor) else 1
    sl: list[Any] = [builtins.slice(None)] * rank
    sl[dim] = builtins.slice(start, end, step)
    return get_item(x, tuple(sl), cache)


def index_put(x: torch.Tensor, key: Any, value: Any) -> torch.Tensor:
    """_handle_index_put (evaluator.py:488-508): a clone of x with ``value`` written at
    ``key`` (basic keys: ints, slices with a positive step, None, ...)."""
    from . import ops

    arr = ops.copy(x)
    items = _expand_key(key, arr.dim())
    if any(isinstance(k, (list, tuple, torch.Tensor)) for k in items):
        raise UnimplementedMathError("IndexPut with an advanced index has no b200 kernel")
    view, deferred = _basic_view(arr, items)
    if deferred:
        raise UnimplementedMathError("IndexPut with a negative-step slice has no b200 kernel")
    v = value if isinstance(value, torch.Tensor) else ops.to_device(torch.tensor(value))
    v = ops.cast(v, arr.dtype) if v.dtype != arr.dtype else v
    shape = tuple(view.shape)
    src = v.expand(shape) if tuple(v.shape) != shape else v
    copy_strided(src, view)
    return arr


def copy_strided(src: torch.Tensor, dst: torch.Tensor) -> None:
    """dst[...] = src for two views of the same shape and dtype (src may broadcast)."""
    from . import ops

    if src.dtype != dst.dtype or tuple(src.shape) != tuple(dst.shape):
        raise ValueError("copy_strided: shapes and dtypes must match")
    nd = dst.dim()
    if dst.numel() == 0:
        return
    if nd == 0:
        src, dst = src.reshape(1), dst.reshape(1)
        nd = 1
    if nd > L.GATHER_MAX_DIM:
        raise UnimplementedMathError(f"strided copy over {nd} dimensions")
    A = C.c_int64 * nd
    L.call("b200_copy_strided", dst.element_size(), src.data_ptr(), A(*src.stride()), dst.data_ptr(), A(*dst.stride()),
           A(*dst.shape), nd, ops.stream_ptr())

"""Weight I/O for device tensors: safetensors and npz files in the reference's layouts.

The reference reads and writes parameters through ``serialization/formats``:

* safetensors (``safetensors.py:109-185``): an 8-byte little-endian header length, the
  header as compact JSON (``separators=(",", ":")``, tensors in insertion order, no
  ``__metadata__``) padded with spaces to a multiple of 8 bytes, then the raw tensor bytes
  end to end. Its loader hands each tensor's bytes to the active backend's
  ``from_buffer(buffer, dtype, shape)`` (``safetensors.py:118-129``).
* npz (``npz.py:62-115``, ``serialization/utils.py:424-447``): a ZIP_STORED archive of
  ``<name>.npy`` entries, each an NPY 1.0 header written as
  ``{'descr': '<f4', 'fortran_order': False, 'shape': (..), }`` padded with spaces to a
  multiple of 16 bytes (magic and lengths included) plus ``\\n``, then the data. A backend
  may take over with ``load_npz(path)`` / ``save_npz(weights, path)`` (``npz.py:84-115``).

``B200Backend`` implements those three hooks with the functions here, so the
reference's own format classes load straight into HBM and save from it. The files are
the same bytes the reference writes (safetensors in full; npz entry by entry, the zip
timestamps aside). Loading reads the file once into pinned host memory and moves it to
the device with one copy per file (safetensors) or per tensor (npz); saving copies each
tensor back once.
"""

from __future__ import annotations

import io
import json
import struct
import zipfile
from collections.abc import Mapping
from typing import Any

import numpy as np
import torch

# safetensors dtype names (the reference's map, serialization_schema.yaml, plus BF16)
_ST_OF_TORCH = {
    torch.float32: "F32", torch.float64: "F64", torch.float16: "F16", torch.bfloat16: "BF16",
    torch.int32: "I32", torch.int64: "I64", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8", torch.bool: "BOOL",
}
_TORCH_OF_ST = {v: k for k, v in _ST_OF_TORCH.items()}
# NPY descr strings (little-endian)
_DESCR_OF_TORCH = {
    torch.float32: "<f4", torch.float64: "<f8", torch.float16: "<f2", torch.int32: "<i4", torch.int64: "<i8",
    torch.int16: "<i2", torch.int8: "|i1", torch.uint8: "|u1", torch.bool: "|b1",
}


def _device() -> torch.device:
    from . import ops

    return ops.device()


def _c_order(a: np.ndarray) -> np.ndarray:
    """C-contiguous, keeping 0-d arrays 0-d (np.ascontiguousarray returns at least 1-d)."""
    a = np.asarray(a)
    return a if a.flags.c_contiguous else a.copy(order="C")


def _as_tensor(v: Any) -> torch.Tensor:
    if isinstance(v, torch.Tensor):
        return v
    return torch.from_numpy(_c_order(v))


def _host_views(tensors: list[torch.Tensor]) -> list[memoryview]:
    """Raw little-endian bytes of each tensor as memoryviews of host memory (device
    tensors: one copy each into pinned memory, one synchronisation for all)."""
    hosts = []
    for t in tensors:
        t = t.contiguous()
        if t.is_cuda:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t, non_blocking=True)
            hosts.append(h)
        else:
            hosts.append(t)
    if any(t.is_cuda for t in tensors):
        torch.cuda.synchronize()
    return [memoryview(h.reshape(-1).view(torch.uint8).numpy()) for h in hosts]




# ---- safetensors ----------------------------------------------------------------------
def _safetensors_parts(weights: Mapping[str, Any]) -> tuple[bytes, list[memoryview]]:
    """Length prefix + padded header, and the tensors' bytes in file order
    (safetensors.py:130-185)."""
    items = [(str(k), _as_tensor(v)) for k, v in weights.items()]
    for k, t in items:
        if t.dtype not in _ST_OF_TORCH:
            raise TypeError(f"safetensors: unsupported dtype {t.dtype} for {k!r}")
    blobs = _host_views([t for _, t in items])
    header: dict[str, Any] = {}
    offset = 0
    for (k, t), b in zip(items, blobs):
        header[k] = {"dtype": _ST_OF_TORCH[t.dtype], "shape": list(t.shape), "data_offsets": [offset, offset + b.nbytes]}
        offset += b.nbytes
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((8 - len(hb) % 8) % 8)
    return struct.pack("<Q", len(hb)) + hb, blobs


def safetensors_bytes(weights: Mapping[str, Any]) -> bytes:
    """The file contents the reference's saver writes for ``weights``."""
    head, blobs = _safetensors_parts(weights)
    return head + b"".join(blobs)


def save_safetensors(weights: Mapping[str, Any], path: str) -> None:
    head, blobs = _safetensors_parts(weights)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:  # straight from the pinned copies, no intermediate join
            f.write(b)


def load_safetensors(path: str, device: torch.device | None = None) -> dict[str, torch.Tensor]:
    """All tensors of a safetensors file on the device: the data section goes to HBM in one
    copy; each tensor is a view of it (or a copy, where its offset does not fit its dtype's
    alignment)."""
    import os

    with open(path, "rb") as f:
        pre = f.read(8)
        if len(pre) < 8:
            return {}
        (hlen,) = struct.unpack("<Q", pre)
        header = json.loads(f.read(hlen).decode("utf-8"))
        entries = [(k, v) for k, v in header.items() if k != "__metadata__"]
        if not entries:
            return {}
        size = os.fstat(f.fileno()).st_size - 8 - hlen
        pinned = torch.empty(size, dtype=torch.uint8, pin_memory=True)
        got = f.readinto(memoryview(pinned.numpy()))  # the data section straight into pinned memory
        if got != size:
            raise OSError(f"{path}: short read ({got} of {size} bytes)")
    dev = device or _device()
    blob = pinned.to(dev, non_blocking=True)
    out = {}
    for k, v in entries:
        dt = _TORCH_OF_ST[v["dtype"]]
        lo, hi = v["data_offsets"]
        seg = blob[lo:hi]
        item = torch.empty((), dtype=dt).element_size()
        if lo % item:
            seg = seg.clone()
        out[k] = seg.view(dt).reshape(v["shape"])
    return out


def from_buffer(buffer: bytes, dtype: str, shape: Any, device: torch.device | None = None) -> torch.Tensor:
    """One tensor from its raw bytes (the backend hook the reference's loader calls)."""
    dt = _TORCH_OF_ST[dtype]
    host = torch.frombuffer(bytearray(buffer), dtype=dt).reshape(list(shape)) if len(buffer) else torch.empty(list(shape), dtype=dt)
    return host.to(device or _device())


# ---- npz ------------------------------------------------------------------------------
def npy_bytes(tensor: Any) -> bytes:
    """One ``.npy`` entry as the reference writes it (serialization/utils.py:424-447)."""
    t = _as_tensor(tensor)
    if t.dtype not in _DESCR_OF_TORCH:
        raise TypeError(f"npy: unsupported dtype {t.dtype}")
    shape = tuple(t.shape)
    shape_str = f"({shape[0]},)" if len(shape) == 1 else str(shape)
    d = "{'descr': '" + _DESCR_OF_TORCH[t.dtype] + "', 'fortran_order': False, 'shape': " + shape_str + ", }"
    d += " " * (16 - (len(d) + 10) % 16) + "\n"
    return b"\x93NUMPY" + struct.pack("<BBH", 1, 0, len(d)) + d.encode("ascii") + bytes(_host_views([t])[0])


def save_npz(weights: Mapping[str, Any], path: str) -> None:
    with zipfile.ZipFile(path, "w", compression=zipfile.ZIP_STORED) as zf:
        for k, v in weights.items():
            name = str(k) if str(k).endswith(".npy") else f"{k}.npy"
            zf.writestr(name, npy_bytes(v))


def load_npz(path: str, device: torch.device | None = None) -> dict[str, torch.Tensor]:
    """All arrays of an ``.npz`` archive on the device (stored or deflated entries)."""
    dev = device or _device()
    out = {}
    with zipfile.ZipFile(path, "r") as zf:
        for name in zf.namelist():
            arr = np.lib.format.read_array(io.BytesIO(zf.read(name)), allow_pickle=False)
            key = name[:-4] if name.endswith(".npy") else name
            host = torch.from_numpy(_c_order(arr))
            out[key] = host.pin_memory().to(dev, non_blocking=True) if host.numel() else host.to(dev)
    return out

"""Weight I/O into and out of HBM: the reference's own files (tests/golden/ops) load into
device tensors with the exact values, through b200's loaders and through the backend
hooks the reference's format classes call (from_buffer, load_npz); device tensors save to
the same bytes the reference wrote; a 64 MB file round-trips."""

import os
import zipfile

import numpy as np
import pytest
import torch

from gpu_helpers import to_np

pytestmark = pytest.mark.gpu

OPS = os.path.join(os.path.dirname(__file__), "golden", "ops")
NAMES = ["layer0.W", "layer0.b", "embed.ids", "half", "bytes", "scale", "big"]


def _arrays():
    z = np.load(os.path.join(OPS, "weights_arrays.npz"))
    return {k: z[k] for k in NAMES}


def test_reference_files_load_into_hbm(cuda):
    from b200 import weights as W
    from b200.backend import B200Backend

    ref = _arrays()
    st = W.load_safetensors(os.path.join(OPS, "weights.safetensors"))
    nz = B200Backend.load_npz(os.path.join(OPS, "weights.npz"))
    assert list(st) == NAMES and sorted(nz) == sorted(NAMES)
    for k, v in ref.items():
        for got in (st[k], nz[k]):
            assert got.is_cuda and tuple(got.shape) == v.shape
            np.testing.assert_array_equal(to_np(got), v)
    # the per-tensor hook the reference's safetensors loader calls
    t = B200Backend.from_buffer(ref["big"].tobytes(), dtype="F32", shape=[64, 33])
    assert t.is_cuda
    np.testing.assert_array_equal(to_np(t), ref["big"])


def test_device_tensors_save_to_reference_bytes(cuda, tmp_path):
    from b200 import weights as W
    from b200.backend import B200Backend

    dev = {k: torch.from_numpy(v).cuda() for k, v in _arrays().items()}
    p = tmp_path / "w.safetensors"
    W.save_safetensors(dev, str(p))
    with open(os.path.join(OPS, "weights.safetensors"), "rb") as f:
        assert p.read_bytes() == f.read()
    q = tmp_path / "w.npz"
    B200Backend.save_npz(dev, str(q))
    ref = zipfile.ZipFile(os.path.join(OPS, "weights.npz"))
    mine = zipfile.ZipFile(q)
    for n in ref.namelist():
        assert mine.read(n) == ref.read(n)


def test_large_roundtrip_bf16_and_f32(cuda, tmp_path):
    from b200 import weights as W

    g = torch.Generator(device="cpu").manual_seed(3)
    w = {"a": torch.randn(4096, 4096, generator=g).cuda(), "b": torch.randn(1000, 7, generator=g).to(torch.bfloat16).cuda(),
         "c": torch.arange(11, dtype=torch.int64).cuda()}
    p = tmp_path / "big.safetensors"
    W.save_safetensors(w, str(p))
    back = W.load_safetensors(str(p))
    for k in w:
        assert back[k].dtype == w[k].dtype and torch.equal(back[k], w[k]), k

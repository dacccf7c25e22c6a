"""Weight files: the b200 writers produce the bytes the reference's own savers wrote for
the same arrays (tests/golden/make_weights_golden.py): the whole safetensors file, and
every .npy entry of the npz archive (the zip's timestamps aside)."""

import os
import zipfile

import numpy as np
import torch

OPS = os.path.join(os.path.dirname(__file__), "golden", "ops")
NAMES = ["layer0.W", "layer0.b", "embed.ids", "half", "bytes", "scale", "big"]


def _arrays():
    z = np.load(os.path.join(OPS, "weights_arrays.npz"))
    return {k: z[k] for k in NAMES}


def test_safetensors_writer_matches_reference_bytes():
    from b200 import weights as W

    w = {k: torch.from_numpy(v) for k, v in _arrays().items()}
    with open(os.path.join(OPS, "weights.safetensors"), "rb") as f:
        assert W.safetensors_bytes(w) == f.read()


def test_npz_entries_match_reference_bytes(tmp_path):
    from b200 import weights as W

    w = _arrays()
    ref = zipfile.ZipFile(os.path.join(OPS, "weights.npz"))
    assert ref.namelist() == [k + ".npy" for k in NAMES]
    for k, v in w.items():
        assert W.npy_bytes(torch.from_numpy(v)) == ref.read(k + ".npy"), k
    out = tmp_path / "mine.npz"
    W.save_npz({k: torch.from_numpy(v) for k, v in w.items()}, str(out))
    mine = zipfile.ZipFile(out)
    assert mine.namelist() == ref.namelist()
    for n in ref.namelist():
        assert mine.read(n) == ref.read(n)
        assert mine.getinfo(n).compress_type == zipfile.ZIP_STORED


def test_writers_take_numpy_arrays_and_keep_0d_shapes():
    from b200 import weights as W

    w = _arrays()
    with open(os.path.join(OPS, "weights.safetensors"), "rb") as f:
        assert W.safetensors_bytes(w) == f.read()  # numpy inputs, 0-d "scale" included
    assert W.npy_bytes(w["scale"]) == zipfile.ZipFile(os.path.join(OPS, "weights.npz")).read("scale.npy")

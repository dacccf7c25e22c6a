"""Generate weight-file fixtures with the REFERENCE's own savers.

Test infrastructure: imports the reference (``ml_switcheroo_compiler``) read-only from the
source tree named by ``--reference-src`` or ``$ML_SWITCHEROO_REFERENCE_SRC``, with the
``ml_switcheroo_ir`` stand-in under ``oracle/standin``, activates its numpy backend and writes, for one seeded weights dictionary (several dtypes,
0-d / 1-d / n-d shapes):

* ``tests/golden/ops/weights.safetensors`` with ``SafetensorsWeightFormat().save``
  (``serialization/formats/safetensors.py:130-185``);
* ``tests/golden/ops/weights.npz`` with ``NpzWeightFormat().save`` (``npz.py:95-115``);
* ``tests/golden/ops/weights_arrays.npz``, the same arrays through numpy, for comparison.

Usage: ``python tests/golden/make_weights_golden.py --reference-src PATH``.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from refpath import add_reference_to_path  # noqa: E402

add_reference_to_path()

from ml_switcheroo_compiler.core.config import config  # noqa: E402
from ml_switcheroo_compiler.serialization.formats.npz import NpzWeightFormat  # noqa: E402
from ml_switcheroo_compiler.serialization.formats.safetensors import SafetensorsWeightFormat  # noqa: E402


def weights() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(17)
    return {
        "layer0.W": rng.standard_normal((3, 5)).astype(np.float32),
        "layer0.b": rng.standard_normal(7).astype(np.float32),
        "embed.ids": rng.integers(-5, 5, size=4).astype(np.int64),
        "half": rng.standard_normal((2, 2, 2)).astype(np.float16),
        "bytes": rng.integers(0, 255, size=5).astype(np.uint8),
        "scale": np.array(0.125, dtype=np.float64),
        "big": rng.standard_normal((64, 33)).astype(np.float32),
    }


def main() -> None:
    config.backend = "numpy"
    out = os.path.join(HERE, "ops")
    os.makedirs(out, exist_ok=True)
    w = weights()
    SafetensorsWeightFormat().save(w, os.path.join(out, "weights.safetensors"))
    NpzWeightFormat().save(w, os.path.join(out, "weights.npz"))
    np.savez(os.path.join(out, "weights_arrays.npz"), **w)
    print("wrote", sorted(os.listdir(out)))


if __name__ == "__main__":
    main()

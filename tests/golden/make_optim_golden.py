"""Generate golden vectors for the optimizer update ops from the REFERENCE itself.

Test infrastructure: imports the reference (``ml_switcheroo_compiler``) read-only from the
source tree named by ``--reference-src`` or ``$ML_SWITCHEROO_REFERENCE_SRC``, with the usage-derived ``ml_switcheroo_ir`` stand-in under
``oracle/standin``, runs the numpy backend's ``execute_op`` (``backends/numpy/generator.py:134``
-> ``numpy/eager/__init__.py:90-125``, which resolves ``ApplyAdam`` / ``ApplyAdagrad`` /
``ApplyFtrl`` / ``ApplyRMSProp`` to ``numpy/eager/optimizers_ops.py``) on seeded fp32
inputs, and writes ``tests/golden/ops/optim.npz``:

* ``<op>/<k>/in<j>``: the j-th array operand of case k,
* ``<op>/<k>/out<j>``: the j-th returned array,
* ``<op>/<k>/lr``: the learning rate passed (absent: the op's default).

Cases cover the default learning rate and another one, zero accumulators (the first
step), negative and zero gradients, and a ragged length. Usage:
``python tests/golden/make_optim_golden.py --reference-src PATH``.
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

from ml_switcheroo_compiler.backends.registry import BackendRegistry  # noqa: E402

# operand count (param + states + grad) of each op
ARITY = {"ApplyAdam": 4, "ApplyAdagrad": 3, "ApplyFtrl": 4, "ApplyRMSProp": 4}
# which operands must be non-negative (second moments / accumulators)
NONNEG = {"ApplyAdam": (2,), "ApplyAdagrad": (1,), "ApplyFtrl": (1,), "ApplyRMSProp": (1,)}


def make_case(op: str, n: int, seed: int, zero_state: bool) -> list[np.ndarray]:
    rng = np.random.default_rng(seed)
    arrs = []
    for j in range(ARITY[op]):
        a = rng.standard_normal(n).astype(np.float32)
        if j in NONNEG[op]:
            a = np.abs(a) * np.float32(0.01)
        if zero_state and 0 < j < ARITY[op] - 1:
            a[:] = 0
        arrs.append(a)
    g = arrs[-1]
    g[:: 17] = 0  # zero gradients
    return arrs


def main() -> None:
    backend = BackendRegistry.get("numpy")
    out: dict[str, np.ndarray] = {}
    for op in ARITY:
        cases = [(515, 1, False, None), (1029, 2, True, None), (2048, 3, False, 0.05), (5, 4, True, 0.3)]
        for k, (n, seed, zero_state, lr) in enumerate(cases):
            ins = make_case(op, n, seed + 10 * list(ARITY).index(op), zero_state)
            kw = {} if lr is None else {"lr": float(lr)}
            res = backend.execute_op(op, *[a.copy() for a in ins], **kw)
            for j, a in enumerate(ins):
                out[f"{op}/{k}/in{j}"] = a
            for j, r in enumerate(res):
                r = np.asarray(r)
                assert r.dtype == np.float32, (op, k, j, r.dtype)
                out[f"{op}/{k}/out{j}"] = r
            if lr is not None:
                out[f"{op}/{k}/lr"] = np.float64(lr)
    np.savez_compressed(os.path.join(HERE, "ops", "optim.npz"), **out)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()

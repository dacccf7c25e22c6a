"""The five fwd+bwd graph workloads: named inputs, seeded synthetic data, sizes.

Each workload is a traced forward function of the reference's op vocabulary plus its
graph-AD backward (the graph itself is produced once by the reference's tracer and AD
and stored as JSON; see ``graphs.py``). This module only knows the *data*: the role of
each graph input, how the synthetic values are drawn (``numpy.random.default_rng``,
one generator per workload, roles drawn in the order listed) and the sizes used by
the benchmark and by the parity cases. No public dataset is involved: every input is
seeded synthetic data with the shapes and distributions of the workload definitions.
"""

from __future__ import annotations

import numpy as np

WORKLOADS: dict[str, dict] = {
    # 2-layer MLP, fp32: x[B,D] -> Linear D->H + ReLU -> Linear H->C -> softmax CE (int64 labels)
    "mlp": {
        "forward": "mlp",
        "inputs": ["x", "W1", "b1", "W2", "b2", "labels"],
        "wrt": ["W1", "b1", "W2", "b2"],
        "fwd_output": "loss",
        "full": {"B": 64, "D": 784, "H": 256, "C": 10},
        "dtype": "f32",
    },
    # fused bandwidth-bound row graph, fp32: y = softmax(LN(gelu_tanh(x*a+b))), argmax(y)
    "rowfused": {
        "forward": "rowfused",
        "inputs": ["x", "a", "b", "gamma", "beta"],
        "wrt": ["x", "a", "b"],
        "fwd_output": "y",
        "argmax_of_output": True,
        "full": {"R": 8192, "C": 4096},
        "dtype": "f32",
    },
    # batched dense contraction, bf16 in / fp32 accumulate: relu(A@B + bias)
    "bmm": {
        "forward": "bmm",
        "inputs": ["A", "B", "bias"],
        "wrt": ["A", "B", "bias"],
        "fwd_output": "out",
        "full": {"Z": 16, "M": 2048, "K": 2048, "N": 2048},
        "dtype": "bf16",
    },
    # small CNN, fp32 activations / bf16 conv math
    "cnn": {
        "forward": "cnn",
        "inputs": ["X", "w1", "w2", "w3", "Wl", "bl", "labels"],
        "wrt": ["w1", "w2", "w3", "Wl", "bl"],
        "fwd_output": "loss",
        "full": {"N": 512},
        "dtype": "bf16",
    },
}


def transformer_roles(L: int) -> list[str]:
    """Graph input roles of the transformer workload, in trace order."""
    roles = ["ids", "labels", "wmask", "attn_scale", "tok_emb", "pos_emb"]
    for i in range(L):
        roles += [f"l{i}_{k}" for k in ("ln1_g", "ln1_b", "Wq", "bq", "Wk", "bk", "Wv", "bv", "Wo", "bo", "ln2_g", "ln2_b", "W1", "b1", "W2", "b2")]
    return roles + ["lnf_g", "lnf_b", "Whead"]


def transformer_params(L: int) -> list[str]:
    return [r for r in transformer_roles(L) if r not in ("ids", "labels", "wmask", "attn_scale")]


# pre-LN transformer encoder stack, bf16 GEMMs with fp32 reductions
WORKLOADS["transformer"] = {
    "forward": "transformer",
    "inputs": lambda dims: transformer_roles(dims["L"]),
    "wrt": lambda dims: transformer_params(dims["L"]),
    "fwd_output": "loss",
    "full": {"L": 4, "d": 1024, "H": 16, "F": 4096, "S": 512, "B": 64, "V": 32000},
    "dtype": "bf16",
}

# Workload graphs stored for the benchmark / DP runs (per-rank batch for DP).
GRAPH_CASES: dict[str, tuple[str, dict]] = {
    "mlp_full": ("mlp", dict(WORKLOADS["mlp"]["full"])),
    "rowfused_full": ("rowfused", dict(WORKLOADS["rowfused"]["full"])),
    "bmm_full": ("bmm", dict(WORKLOADS["bmm"]["full"])),
    "bmm_z8": ("bmm", {"Z": 8, "M": 2048, "K": 2048, "N": 2048}),
    "bmm_z4": ("bmm", {"Z": 4, "M": 2048, "K": 2048, "N": 2048}),
    "bmm_z2": ("bmm", {"Z": 2, "M": 2048, "K": 2048, "N": 2048}),
    "cnn_full": ("cnn", {"N": 512}),
    "cnn_n256": ("cnn", {"N": 256}),
    "cnn_n128": ("cnn", {"N": 128}),
    "cnn_n64": ("cnn", {"N": 64}),
    "transformer_full": ("transformer", dict(WORKLOADS["transformer"]["full"])),
    "transformer_b32": ("transformer", dict(WORKLOADS["transformer"]["full"], B=32)),
    "transformer_b16": ("transformer", dict(WORKLOADS["transformer"]["full"], B=16)),
    "transformer_b8": ("transformer", dict(WORKLOADS["transformer"]["full"], B=8)),
    # one sequence at full width: the bounded CPU sample of the transformer step
    "transformer_b1": ("transformer", dict(WORKLOADS["transformer"]["full"], B=1)),
}

# Small cases with reference-evaluated golden outputs.
GOLDEN_CASES: dict[str, tuple[str, dict]] = {
    "mlp_small": ("mlp", {"B": 64, "D": 784, "H": 256, "C": 10}),
    "mlp_ragged": ("mlp", {"B": 7, "D": 33, "H": 19, "C": 5}),
    "rowfused_small": ("rowfused", {"R": 64, "C": 4096}),
    "rowfused_ragged": ("rowfused", {"R": 9, "C": 1000}),
    "bmm_small": ("bmm", {"Z": 2, "M": 256, "K": 192, "N": 256}),
    "cnn_small": ("cnn", {"N": 4}),
    "transformer_small": ("transformer", {"L": 2, "d": 64, "H": 4, "F": 256, "S": 32, "B": 2, "V": 512}),
}


def _bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returned as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def make_inputs(workload: str, dims: dict, seed: int = 0) -> dict[str, np.ndarray]:
    """Seeded synthetic inputs for ``workload`` at ``dims`` (role -> array).

    The cotangent (upstream gradient) of the forward output is included as role
    ``"cotangent"``: 1.0 for scalar losses, N(0,1) for tensor outputs.
    """
    rng = np.random.default_rng(seed)
    f32 = np.float32
    out: dict[str, np.ndarray] = {}
    if workload == "mlp":
        B, Din, H, C = dims["B"], dims["D"], dims["H"], dims["C"]
        out["x"] = rng.standard_normal((B, Din), dtype=f32)
        out["W1"] = (rng.uniform(-1, 1, (Din, H)) * np.sqrt(6.0 / Din)).astype(f32)
        out["b1"] = np.zeros(H, f32)
        out["W2"] = (rng.uniform(-1, 1, (H, C)) * np.sqrt(6.0 / H)).astype(f32)
        out["b2"] = np.zeros(C, f32)
        out["labels"] = rng.integers(0, C, (B, 1), dtype=np.int64)
        out["cotangent"] = np.array(1.0, f32)
    elif workload == "rowfused":
        R, C = dims["R"], dims["C"]
        out["x"] = rng.standard_normal((R, C), dtype=f32)
        out["a"] = rng.uniform(0.5, 1.5, C).astype(f32)
        out["b"] = (rng.standard_normal(C) * 0.1).astype(f32)
        out["gamma"] = np.ones(C, f32)
        out["beta"] = np.zeros(C, f32)
        out["cotangent"] = rng.standard_normal((R, C), dtype=f32)
    elif workload == "bmm":
        Z, M, K, N = dims["Z"], dims["M"], dims["K"], dims["N"]
        s = np.sqrt(1.0 / 2048.0)
        out["A"] = _bf16_round((rng.standard_normal((Z, M, K), dtype=f32) * s).astype(f32))
        out["B"] = _bf16_round((rng.standard_normal((Z, K, N), dtype=f32) * s).astype(f32))
        out["bias"] = (rng.standard_normal(N) * 0.02).astype(f32)
        out["cotangent"] = rng.standard_normal((Z, M, N), dtype=f32)
    elif workload == "cnn":
        N = dims["N"]

        def he(*shape):
            fan_in = int(np.prod(shape[1:]))
            return (rng.standard_normal(shape) * np.sqrt(2.0 / fan_in)).astype(f32)

        out["X"] = rng.standard_normal((N, 3, 32, 32), dtype=f32)
        out["w1"] = _bf16_round(he(64, 3, 3, 3))
        out["w2"] = _bf16_round(he(64, 64, 3, 3))
        out["w3"] = _bf16_round(he(128, 64, 3, 3))
        out["Wl"] = (rng.standard_normal((128, 10)) * np.sqrt(2.0 / 128)).astype(f32)
        out["bl"] = np.zeros(10, f32)
        out["labels"] = rng.integers(0, 10, (N, 1), dtype=np.int64)
        out["cotangent"] = np.array(1.0, f32)
    elif workload == "transformer":
        L, d, H, F, S, B, V = (dims[k] for k in ("L", "d", "H", "F", "S", "B", "V"))
        T = B * S

        def w(*shape):
            return _bf16_round((rng.standard_normal(shape, dtype=f32) * 0.02).astype(f32))

        ids = rng.integers(0, V, (B, S), dtype=np.int64)
        out["ids"] = ids.reshape(T)
        nxt = np.zeros((B, S), np.int64)
        nxt[:, :-1] = ids[:, 1:]
        out["labels"] = nxt.reshape(T, 1)
        wm = np.full((B, S), -1.0 / (B * (S - 1)), f32)
        wm[:, -1] = 0.0
        out["wmask"] = wm.reshape(T, 1)
        out["attn_scale"] = np.array(1.0 / np.sqrt(d // H), f32)
        out["tok_emb"] = w(V, d)
        out["pos_emb"] = w(S, d)
        for i in range(L):
            out[f"l{i}_ln1_g"] = np.ones(d, f32)
            out[f"l{i}_ln1_b"] = np.zeros(d, f32)
            for nm in ("Wq", "Wk", "Wv", "Wo"):
                out[f"l{i}_{nm}"] = w(d, d)
                out[f"l{i}_b{nm[1].lower()}"] = np.zeros(d, f32)
            out[f"l{i}_ln2_g"] = np.ones(d, f32)
            out[f"l{i}_ln2_b"] = np.zeros(d, f32)
            out[f"l{i}_W1"] = w(d, F)
            out[f"l{i}_b1"] = np.zeros(F, f32)
            out[f"l{i}_W2"] = w(F, d)
            out[f"l{i}_b2"] = np.zeros(d, f32)
        out["lnf_g"] = np.ones(d, f32)
        out["lnf_b"] = np.zeros(d, f32)
        out["Whead"] = w(d, V)
        out["cotangent"] = np.array(1.0, f32)
    else:
        raise KeyError(workload)
    return out

"""Helpers shared by the -m gpu tests."""

import numpy as np
import torch

from conftest import load_golden

BF16_WORKLOADS = {"bmm", "cnn", "transformer"}


def set_policy(workload: str) -> None:
    from b200 import ops

    bf = workload in BF16_WORKLOADS
    ops.Config.matmul_dtype = "bf16" if bf else "f32"
    ops.Config.conv_dtype = "bf16" if bf else "f32"


def to_np(v):
    if isinstance(v, torch.Tensor):
        v = v.detach()
        if v.dtype == torch.bfloat16:
            v = v.float()
        return v.cpu().numpy()
    return np.asarray(v)


def rms(a) -> float:
    """Root mean square over the entries that are not exactly zero (0 if all are)."""
    a = np.asarray(a, dtype=np.float64)
    nz = a[a != 0]
    return float(np.sqrt(np.mean(nz * nz))) if nz.size else 0.0


BF16_REALIZATIONS = 2.0  # the GPU's bf16 rounding and the oracle's emulation of it


def bf16_noise(ref_bf16, ref_fp32) -> tuple[float, float]:
    """(largest |difference|, RMS difference) that bf16 operand rounding itself makes to one
    output of a bf16-math graph: the oracle evaluated with and without rounding every
    contraction operand to bf16 (fp32 accumulation both times)."""
    a = np.asarray(ref_bf16, dtype=np.float64) - np.asarray(ref_fp32, dtype=np.float64)
    if not a.size:
        return 0.0, 0.0
    return float(np.abs(a).max()), float(np.sqrt(np.mean(a * a)))


def bf16_report(name, got, ref_bf16, ref_fp32, rtol, floor=0.0) -> str | None:
    """None when ``got`` (the backend under the bf16 policy) is as close to the oracle's
    bf16 emulation ``ref_bf16`` as a second bf16 evaluation can be, else a description.

    Two correct bf16 evaluations (this backend and the oracle's emulation) differ only in
    fp32 summation order before each rounding, but a difference of one fp32 ulp there can
    move a rounded operand by a whole bf16 ulp. A difference d before a rounding thus
    becomes about sqrt(d x ulp) after it, and through a deep graph the two evaluations
    drift apart until they differ like two independent roundings (measured on the
    transformer step: the ratio RMS(backend - emulation) / RMS(emulation - fp32) grows
    0.005, 0.04, 0.18, 0.43, 0.67, ... through the first layer's GEMMs and settles near 1).
    Rounding noise in a gradient is also heavy-tailed: its largest element is tens of times
    its RMS. So each evaluation is held to the rounding's own size, measured on the oracle:
    if both lie within M = max |emulation - fp32| of the exact result, they lie within 2M of
    each other (and within 2 x RMS(emulation - fp32) in RMS):

    * elementwise |got - ref_bf16| <= rtol * |ref_bf16| + atol, atol = the larger of
      rtol * rms(ref_bf16) (``close_report``'s floor) and 2M;
    * RMS(got - ref_bf16) <= 2 x RMS(ref_bf16 - ref_fp32) + 1e-5 x rms(ref_bf16), so a
      systematic error cannot hide under the tails' allowance.
    """
    big, spread = bf16_noise(ref_bf16, ref_fp32)
    msg = close_report(name, got, ref_bf16, rtol, floor=floor, atol_floor=BF16_REALIZATIONS * big)
    if msg:
        return msg
    g = to_np(got).astype(np.float64)
    e = np.asarray(ref_bf16, dtype=np.float64)
    d = float(np.sqrt(np.mean((g - e) ** 2))) if e.size else 0.0
    lim = BF16_REALIZATIONS * spread + 1e-5 * rms(e)
    if d > lim:
        return (f"{name}: RMS(got - oracle) {d:.3g} above {BF16_REALIZATIONS:g} x RMS of the bf16 rounding's own effect "
                f"({spread:.3g}) + 1e-5 x rms")
    return None


def close_report(name, got, ref, rtol, floor=0.0, atol_floor=0.0) -> str | None:
    """None when ``got`` matches ``ref`` elementwise, else a one-line description:
    |got - ref| <= rtol * |ref| + atol for every element, with the absolute floor
    atol = rtol * max(rms(ref), floor), rms over ref's non-zero entries.

    Why a floor at all: an entry much smaller than its output's typical magnitude is a sum
    whose terms cancelled, so its absolute rounding error is set by the size of those
    terms, which is the typical magnitude of the output's entries (their RMS), not by the
    entry itself. The floor bounds that error at rtol of the RMS. Entries that are exactly
    zero in the reference (embedding rows of tokens absent from the batch) do not set the
    scale. ``floor`` covers outputs that are zero in exact arithmetic (pure rounding
    noise): the caller derives it from a related output. ``atol_floor`` is an absolute
    floor in the output's units (``bf16_report``). Integer / bool outputs (argmax,
    labels, gathers) must be bit-exact."""
    got = to_np(got)
    ref = np.asarray(ref)
    if got.shape != ref.shape:
        return f"{name}: shape {got.shape} != {ref.shape}"
    if ref.dtype.kind in "iub":
        n = int((got != ref).sum())
        return None if n == 0 else f"{name}: {n} of {ref.size} integer elements differ"
    g64, r64 = got.astype(np.float64), ref.astype(np.float64)
    scale = rms(r64)
    atol = max(rtol * max(scale, float(floor), 1e-30), float(atol_floor))
    err = np.abs(g64 - r64)
    lim = atol + rtol * np.abs(r64)
    bad = ~(err <= lim)
    if not bad.any():
        return None
    k = int(np.argmax(np.where(bad, err / lim, 0)))
    return (f"{name}: {int(bad.sum())} of {ref.size} elements outside rtol {rtol} (atol {atol:.3g}, rms {scale:.3g}); "
            f"worst at flat index {k}: got {g64.flat[k]:.6g}, ref {r64.flat[k]:.6g}, |diff| / limit = "
            f"{float(err.flat[k] / lim.flat[k]):.3g}; max |diff| / rms = {float(err.max() / max(scale, 1e-30)):.3g}")


def assert_close(name, got, ref, rtol, floor=0.0, atol_floor=0.0):
    """``close_report`` as an assertion."""
    msg = close_report(name, got, ref, rtol, floor, atol_floor)
    if msg:
        raise AssertionError(msg)


def run_case(case: str, mode: str = "graph"):
    """Evaluate a golden case on the b200 backend; returns ({name: value}, golden outs, graph)."""
    from b200 import graph as G
    from b200.backend import B200Backend
    from b200.executor import GraphRunner

    ins, outs = load_golden(case)
    g = G.load(case)
    set_policy(g.meta["workload"])
    inputs = {nid: torch.from_numpy(np.ascontiguousarray(ins[r])).cuda() for r, nid in g.roles.items()}
    if mode == "graph":
        res = B200Backend.execute_graph(g, inputs)
    elif mode == "pernode":
        res = GraphRunner(g, fuse=False)(inputs)
    elif mode == "compiled":
        fn = B200Backend.compile_graph(g)
        fn(inputs)
        res = fn(inputs)
    elif mode == "compiled_host":  # replays fed from pinned host tensors (copied into the static buffers)
        fn = B200Backend.compile_graph(g)
        fn(inputs)
        host = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        fn(host)
        res = {k: v.clone() for k, v in fn(host).items()}
    else:
        raise ValueError(mode)
    return {name: res[nid] for name, nid in g.output_names.items()}, outs, g


def gpu_decisions(g, inputs) -> dict:
    """The backend's own ReLU VJP masks (every ``Greater`` node of the graph): node id ->
    bool array. Each mask is taken from the fused plan the backend runs, where the kernel
    that produces it (a GEMM or convolution epilogue, a fused elementwise step) publishes
    it; a mask that stays inside a fused kernel is taken from an unfused run of the same
    graph on the same inputs instead."""
    from b200.executor import GraphRunner

    ids = {n.id: None for n in g.nodes.values() if n.op_type == "Greater"}
    if not ids:
        return {}
    for fuse in (True, False):
        want = {k: None for k, v in ids.items() if v is None}
        if not want:
            break
        r = GraphRunner(g, fuse=fuse)
        d = r.device_inputs(inputs)
        r.plan_for(d).run(d, capture=want)
        ids.update({k: v for k, v in want.items() if v is not None})
    return {k: to_np(v).astype(bool) for k, v in ids.items() if v is not None}


def check_decisions(report, limit=1e-2) -> None:
    """Replayed masks may differ from the oracle's own only at the decision boundary:
    where they differ, |pre-activation| <= ``limit`` x its RMS."""
    for nid, n, worst in report:
        assert worst <= limit, f"mask {nid}: {n} decisions differ, one at |x| = {worst:.3g} x rms (not at the boundary)"

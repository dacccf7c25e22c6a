"""Benchmark: fwd+bwd graph steps/sec of the b200 backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl b200|reference]

A step is one evaluation of a workload's fwd+bwd LogicalGraph (the graph the reference's
tracer + AD produced, stored under tests/golden/graphs) on one batch of seeded synthetic
inputs. The headline workload (default) is the pre-LN transformer encoder stack (4 x
d 1024, 16 heads, FFN 4096, seq 512, vocab 32000, global batch 64): the configuration
with a data-parallel split and a multi-GPU target. The other four workloads (fused
bandwidth-bound row graph, MLP, batched contraction, small CNN) are timed in the same run
and reported in the line's ``configs`` block.

Multi-GPU (torchrun, one process per GPU, NCCL): workloads with per-rank graphs split the
global batch over the ranks (strong scaling: transformer, CNN, batched contraction); the
others run one full batch per rank (weak scaling). Replicated-parameter gradients are
all-reduced. ``value`` = global batches processed by all ranks / max-over-ranks device
time.

``--impl reference`` times the reference algorithm on the host CPU: the numpy
restatement of the reference's evaluate_graph + numpy kernels (pinned to the reference's
own evaluation by tests/test_oracle.py), on bounded samples of the same workload, scaled
to a full step. Only the evaluation is timed.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "ml-switcheroo-compiler_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

# workload -> graph at the global batch, per-rank graphs for a batch split, dtype, the
# replicated parameters whose gradients are exchanged, and the CPU sample
WORKLOADS = {
    "transformer": {"graph": "transformer_full", "dtype": "bf16", "params": "all", "reduce": "mean",
                    "dp_graphs": {2: "transformer_b32", 4: "transformer_b16", 8: "transformer_b8"},
                    "cpu_sample": ("transformer_b1", 64),
                    "desc": "pre-LN transformer encoder 4x(d1024,h16,ffn4096) seq 512, global batch 64, next-token CE fwd+bwd"},
    "rowfused": {"graph": "rowfused_full", "dtype": "f32", "params": ["a", "b"], "reduce": "sum",
                 "desc": "fused bandwidth-bound graph x[8192,4096]: gelu_tanh(x*a+b) -> LayerNorm -> softmax + argmax, fwd+bwd wrt x,a,b"},
    "mlp": {"graph": "mlp_full", "dtype": "f32", "params": ["W1", "b1", "W2", "b2"], "reduce": "mean",
            "desc": "2-layer MLP x[64,784] 784->256->10 softmax CE fwd+bwd"},
    "bmm": {"graph": "bmm_full", "dtype": "bf16", "params": ["bias"], "bf16_inputs": ["A", "B"], "reduce": "sum",
            "dp_graphs": {2: "bmm_z8", 4: "bmm_z4", 8: "bmm_z2"},
            "desc": "batched contraction A,B[16,2048,2048] bf16: relu(A@B+bias) fwd+bwd (dA, dB, dbias)"},
    "cnn": {"graph": "cnn_full", "dtype": "bf16", "params": ["w1", "w2", "w3", "Wl", "bl"], "reduce": "mean",
            "dp_graphs": {2: "cnn_n256", 4: "cnn_n128", 8: "cnn_n64"},
            "desc": "small CNN [512,3,32,32] 3 conv3x3 (VALID) + GAP + linear, softmax CE fwd+bwd"},
}
CONFIG_ORDER = ["transformer", "rowfused", "mlp", "bmm", "cnn"]


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained") or d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------------
# CPU reference (the oracle port of the reference's numpy evaluation)
# ----------------------------------------------------------------------------------
_ROW_STATE: dict = {}


def _row_worker_init(case: str, lo: int, hi: int) -> None:
    """Pool initializer: import, load the graph and draw this worker's rows (untimed)."""
    from oracle import evaluator as O

    _ROW_STATE["g"] = O.load_graph(case)
    _ROW_STATE["arrays"] = _row_slice_inputs(_ROW_STATE["g"], lo, hi)


def _row_worker_eval(_) -> float:
    """One evaluation of this worker's rows; returns its duration."""
    from oracle import evaluator as O

    t0 = time.perf_counter()
    O.evaluate_roles(_ROW_STATE["g"], _ROW_STATE["arrays"])
    return time.perf_counter() - t0


def _row_slice_inputs(g, lo, hi):
    rng = np.random.default_rng(1000 + lo)
    C = g["dims"]["C"]
    n = hi - lo
    f32 = np.float32
    return {"x": rng.standard_normal((n, C), dtype=f32), "a": rng.uniform(0.5, 1.5, C).astype(f32),
            "b": (rng.standard_normal(C) * 0.1).astype(f32), "gamma": np.ones(C, f32), "beta": np.zeros(C, f32),
            "cotangent": rng.standard_normal((n, C), dtype=f32)}


class CpuReference:
    """Timed CPU evaluations of a workload by the oracle. Everything but the evaluation
    (process start, imports, graph loading, input generation, one warm-up evaluation)
    happens in ``prepare``; ``sample()`` times one evaluation and returns the full-step
    time it stands for."""

    def __init__(self, workload: str) -> None:
        self.workload = workload
        self.spec = WORKLOADS[workload]
        self.cores = os.cpu_count() or 1
        self.pool = None

    def prepare(self, budget_s: float = 20.0) -> None:
        from oracle import evaluator as O

        if self.workload == "rowfused":
            import multiprocessing as mp

            R = 8192
            self.R = R
            # one worker per core, each evaluating its own contiguous rows (rows are independent)
            g = O.load_graph("rowfused_full")
            probe_in = _row_slice_inputs(g, 0, 16)
            O.evaluate_roles(g, probe_in)
            t0 = time.perf_counter()
            O.evaluate_roles(g, probe_in)
            per_row = max((time.perf_counter() - t0) / 16, 1e-5)
            rows_total = int(min(R, max(self.cores * 8, budget_s * self.cores / per_row / 2)))
            self.rows = rows_total
            chunk = max(8, -(-rows_total // self.cores))
            self.shards = [(lo, min(rows_total, lo + chunk)) for lo in range(0, rows_total, chunk)]
            ctx = mp.get_context("spawn")
            self.pool = [ctx.Pool(1, initializer=_row_worker_init, initargs=("rowfused_full", lo, hi)) for lo, hi in self.shards]
            self._map()  # warm-up evaluation in every worker (untimed)
            self.desc = f"{rows_total} of {R} rows in {len(self.shards)} processes (one evaluation each), scaled to {R} rows"
            self.used_cores = len(self.shards)
            return
        case, scale = self.spec.get("cpu_sample", (self.spec["graph"], 1))
        self.scale = scale
        self.g = O.load_graph(case)
        from b200.workloads import make_inputs

        self.arrays = make_inputs(self.g["workload"], self.g["dims"], seed=0)
        self._eval()  # warm-up evaluation (untimed)
        # fp32 numpy on the operands' own layouts, as the reference evaluates these graphs
        # (its numpy Cast to bfloat16 is fp32, numpy/eager/variable_ops.py:42-43)
        self.desc = (f"one fwd+bwd evaluation of {case}" + (f" (1/{scale} of the global batch), scaled x{scale}" if scale > 1 else "")
                     + f"; fp32 numpy as the reference runs it, BLAS threads = {self.cores}")
        self.used_cores = self.cores

    def _eval(self) -> None:
        from oracle import evaluator as O

        O.evaluate_roles(self.g, self.arrays)

    def _map(self) -> float:
        rs = [p.apply_async(_row_worker_eval, (0,)) for p in self.pool]
        return max(r.get() for r in rs)

    def sample(self) -> float:
        """Seconds of one full step, from one timed evaluation of the sample."""
        if self.workload == "rowfused":
            t0 = time.perf_counter()
            self._map()
            return (time.perf_counter() - t0) * self.R / self.rows
        t0 = time.perf_counter()
        self._eval()
        return (time.perf_counter() - t0) * self.scale

    def close(self) -> None:
        for p in self.pool or []:
            p.terminate()

    def baseline(self, value: float, samples: int) -> dict:
        return {"value": value, "unit": "steps/s", "cores": self.used_cores, "kind": "port",
                "sample": f"{self.desc}; {samples} timed sample(s)"}


def cpu_baseline(workload: str, max_samples: int = 3, budget_s: float = 45.0) -> dict:
    """The oracle on the host cores, beside the GPU number: at most ``max_samples`` timed
    evaluations, stopped once ``budget_s`` seconds of them have run."""
    ref = CpuReference(workload)
    try:
        ref.prepare()
        times, t_start = [], time.perf_counter()
        while len(times) < max_samples:
            times.append(ref.sample())
            if time.perf_counter() - t_start > budget_s:
                break
        return ref.baseline(1.0 / statistics.median(times), len(times))
    finally:
        ref.close()


# ----------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------
def algorithmic_bytes_rowfused(R: int, C: int) -> int:
    # read x, cot; write y, dx (fp32) + argmax int64 + da, db (+ a, b, gamma, beta read)
    return 4 * R * C * 4 + R * 8 + 2 * C * 4 + 4 * C * 4


def cnn_flops(N: int) -> float:
    """Conv FLOPs of one fwd+bwd step of the small CNN (VALID padding, the shapes the
    reference's tracer infers): forward and weight gradient of the three convs, input
    gradient of the last two (the first conv's is dead)."""
    f1 = 2.0 * 64 * 30 * 30 * 3 * 9
    f2 = 2.0 * 64 * 14 * 14 * 64 * 9
    f3 = 2.0 * 128 * 6 * 6 * 64 * 9
    return N * (2 * (f1 + f2 + f3) + f2 + f3)


class GemmTimer:
    """CUDA events around every bf16 tcgen05 GEMM launch of one eager plan run, on the
    launching stream: algorithmic FLOPs (2 M N K per batch matrix) / event time."""

    NAMES = ("b200_gemm", "b200_gemm_batched2")

    def __init__(self) -> None:
        self.recs: list = []

    def run(self, plan, inputs) -> dict:
        import torch

        from b200 import _lib as L

        orig = L.call

        def call(name, *a):
            if name in self.NAMES and a[0] == L.BF16:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                orig(name, *a)
                e1.record()
                fl = 2.0 * a[5] * a[6] * a[7] * a[8] * (a[9] if name == "b200_gemm_batched2" else 1)
                self.recs.append((fl, e0, e1))
            else:
                orig(name, *a)

        L.call = call
        try:
            plan.run(dict(inputs))
            torch.cuda.synchronize()
        finally:
            L.call = orig
        fl = sum(r[0] for r in self.recs)
        ms = sum(r[1].elapsed_time(r[2]) for r in self.recs)
        return {"launches": len(self.recs), "flops": fl, "ms": ms}


def _sync_fn(dist, sync, grads):
    if dist is None:
        return lambda out: None
    return lambda out: sync([out[g] for g in grads])


def measure(name: str, args, world: int, rank: int, dist, dev, headline: bool) -> dict:
    """Time one workload: CUDA-graph replays of its fused plan on resident inputs (plus the
    gradient exchange at N > 1), then the same steps end to end through the public
    ``compile_graph`` call with pinned host inputs and every output copied back."""
    import torch

    from b200 import _lib
    from b200 import graph as G
    from b200 import ops
    from b200.backend import B200Backend
    from b200.dp import GradAllReduce
    from b200.executor import CompiledGraph
    from b200.workloads import make_inputs

    spec = WORKLOADS[name]
    ops.Config.matmul_dtype = "bf16" if spec["dtype"] == "bf16" else "f32"
    ops.Config.conv_dtype = ops.Config.matmul_dtype
    strong = world > 1 and world in spec.get("dp_graphs", {})
    gname = spec["dp_graphs"][world] if strong else spec["graph"]
    if headline and args.graph:
        gname = args.graph  # a smaller per-rank graph of the same workload (profiling captures)
    g = G.load(gname)
    arrays = make_inputs(g.meta["workload"], g.meta["dims"], seed=rank)  # each rank: its own shard
    params = [k[2:] for k in g.output_names if k.startswith("d_")] if spec["params"] == "all" else spec["params"]
    grad_ids = [g.output_names["d_" + r] for r in params]
    sync = GradAllReduce("mean" if (strong and spec["reduce"] == "mean") else "sum")
    allreduce = _sync_fn(dist, sync, grad_ids)

    bf16_roles = set(spec.get("bf16_inputs", []))
    dinputs = {nid: torch.from_numpy(np.ascontiguousarray(arrays[r])).to(dev) for r, nid in g.roles.items()}
    for r in bf16_roles:
        dinputs[g.roles[r]] = dinputs[g.roles[r]].to(torch.bfloat16)
    stream = torch.cuda.current_stream()
    overlap = dist is not None and strong and not args.no_overlap
    exchange = ov = cg = None
    if overlap:
        # gradient buckets all-reduced on a side stream while the backward computes
        from b200.dp import OverlappedStep

        ov = OverlappedStep(g, dinputs, grad_ids, sync)
        static_in, plan = ov.static_in, ov.plan
    else:
        cg = CompiledGraph(g)
        out = cg(dinputs)  # plan + capture
        torch.cuda.synchronize()
        static_in = cg.static_in  # resident in the graph's static buffers from here on
        plan = cg.runner.plan_for(cg.static_in)
    n0 = _lib.launch_count()
    if args.profile and headline:
        # the profiler range (ncu --profile-from-start off) covers exactly this one eager step
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
    plan.run(dict(static_in))  # one eager run of the plan: count its kernels
    torch.cuda.synchronize()
    if args.profile and headline:
        torch.cuda.profiler.stop()
    launches_per_step = int(_lib.launch_count() - n0)

    sync_launches = 0
    for i in range(args.warmup):
        if ov is not None:
            n1 = _lib.launch_count()
            ov()
            if i == args.warmup - 1:
                sync_launches = max(0, int(_lib.launch_count() - n1))  # exchange kernels (graph replays do not count)
            continue
        out = cg(static_in)
        n1 = _lib.launch_count()
        allreduce(out)
        if i == args.warmup - 1:
            sync_launches = int(_lib.launch_count() - n1)
    torch.cuda.synchronize()
    if cg is not None and dist is not None and sync.graph_safe([out[gid] for gid in grad_ids]):
        exchange = torch.cuda.CUDAGraph()
        with torch.cuda.graph(exchange):
            allreduce(out)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(env_int("LOCAL_RANK", 0)) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            if ov is not None:
                ov()
                continue
            out = cg(static_in)
            if exchange is not None:
                exchange.replay()
            else:
                allreduce(out)
        ev1.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    sync.check()  # collective: a peer wait that gave up raises here on every rank
    t = torch.tensor([ms], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    value = (1 if strong else world) * args.steps / (ms_max / 1000.0)
    res = {"value": round(value, 3), "unit": "steps/s", "ms_per_step": round(ms_step, 4),
           "scaling": "strong" if strong else "weak", "graph": gname, "dims": g.meta["dims"],
           "launches_per_step": launches_per_step + sync_launches, "gpu_launches": (launches_per_step + sync_launches) * args.steps,
           "plan_steps": len(plan.steps), "clocks": clk.summary(),
           "grad_exchange": ((("overlapped with the backward: " + json.dumps(ov.describe())) if ov is not None else "after the step")
                             + "; " + (("peer-memory kernel" + (", CUDA graph" if exchange is not None else " + NCCL buckets"))
                                       if sync.peer is not None else "NCCL buckets")) if world > 1 else None}
    if headline:
        res["plan"] = plan.describe()

    # roofline of the dominant kernel
    pk = peaks()
    roof = None
    if name in ("transformer", "bmm"):
        gt = GemmTimer().run(plan, static_in)
        ach = gt["flops"] / (gt["ms"] / 1000.0) / 1e12
        peak = pk["bf16_tflops_sustained"]
        roof = {"bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05, every bf16 GEMM launch of one step)", "achieved": round(ach, 1),
                "peak": peak, "peak_kind": "sustained (GEMMs timed inside a long step)", "unit": "TFLOP/s",
                "frac": round(ach / peak, 4), "peak_source": pk["source"], "launches": gt["launches"],
                "algorithmic_flops": gt["flops"], "kernel_ms": round(gt["ms"], 4), "traffic": None,
                "step_tflops": round(gt["flops"] / (ms_step / 1000.0) / 1e12, 1)}
    elif name == "rowfused":
        R, C = g.meta["dims"]["R"], g.meta["dims"]["C"]
        bytes_ = algorithmic_bytes_rowfused(R, C)
        ach = bytes_ / (ms_step / 1000.0) / 1e9
        roof = {"bound": "hbm", "kernel": "rowfused (fused row kernel + column-sum kernel: the whole replayed step)",
                "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(ach / pk["hbm_gbs"], 4),
                "peak_source": pk["source"], "algorithmic_bytes": bytes_, "kernel_ms": round(ms_step, 4), "traffic": args.traffic}
    elif name == "cnn":
        fl = cnn_flops(g.meta["dims"]["N"])
        ach = fl / (ms_step / 1000.0) / 1e12
        roof = {"bound": "tensor", "kernel": "whole step (conv FLOPs / step time)", "achieved": round(ach, 2),
                "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s", "frac": round(ach / pk["bf16_tflops_sustained"], 4),
                "peak_source": pk["source"], "algorithmic_flops": fl, "traffic": None}
    res["roofline"] = roof

    # end to end through the public API: pinned host inputs in, every output back to pinned host
    if not args.no_e2e:
        host = {nid: torch.from_numpy(np.ascontiguousarray(arrays[r])) for r, nid in g.roles.items()}
        for r in bf16_roles:
            host[g.roles[r]] = host[g.roles[r]].to(torch.bfloat16)
        host = {k: v.pin_memory() for k, v in host.items()}
        out_ids = list(dict.fromkeys(g.output_names.values()))
        ref_out = ov.static_out if ov is not None else out
        host_out = {k: torch.empty(ref_out[k].shape, dtype=ref_out[k].dtype).pin_memory() for k in out_ids}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        d2h = sum(v.numel() * v.element_size() for v in host_out.values())
        del cg, ov, plan, ref_out
        out = None
        gc.collect()
        torch.cuda.empty_cache()
        fn = B200Backend.compile_graph(g)

        def e2e_step():
            o = fn(host)  # pinned host inputs copied by the call straight into its static buffers
            allreduce(o)
            for k in out_ids:
                host_out[k].copy_(o[k], non_blocking=True)

        for _ in range(max(2, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        et = torch.tensor([a.elapsed_time(b)], device=dev)
        if dist is not None:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        res["e2e"] = {"value": round((1 if strong else world) * args.steps / (float(et.item()) / 1000.0), 3), "unit": "steps/s",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                      "outputs_copied": f"all {len(out_ids)} graph outputs"}
        del fn
    gc.collect()
    torch.cuda.empty_cache()
    return res


def run_gpu(args) -> None:
    import torch

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from b200 import _lib

    _lib.load()
    head = args.workload
    others = [] if args.only else [w for w in CONFIG_ORDER if w != head]
    results = {head: measure(head, args, world, rank, dist, dev, headline=True)}
    for w in others:
        results[w] = measure(w, args, world, rank, dist, dev, headline=False)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(head)
    if rank == 0:
        h = results[head]
        spec = WORKLOADS[head]
        line = {
            "metric": "fwd+bwd graph steps/sec",
            "value": h["value"],
            "unit": "steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": h["ms_per_step"],
            "higher_is_better": True,
            "scaling": h["scaling"],
            "vs_baseline": None,
            "dtype": spec["dtype"],
            "data": "synthetic (seeded numpy, per-rank seed)",
            "config": {"workload": spec["desc"], "graph": h["graph"], "dims": h["dims"],
                       "parallelism": f"dp{world}" if world > 1 else "single",
                       "l2": "inputs and the step's working set larger than the 126 MB L2 (no flush needed)",
                       "replay": "CUDA graph of the fused plan", "grad_exchange": h["grad_exchange"]},
            "gpu_launches": sum(r["gpu_launches"] for r in results.values()),
            "launches_per_step": h["launches_per_step"],
            "plan_steps": h["plan_steps"],
            "plan": h.get("plan"),
            "clocks": h["clocks"],
            "roofline": h["roofline"],
            "cpu_baseline": cpu,
            "e2e": h.get("e2e"),
            "configs": {w: {k: v for k, v in r.items() if k not in ("plan",)} for w, r in results.items() if w != head},
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args) -> None:
    """The reference algorithm on the host CPU (the oracle port), for the same workload,
    metric and unit as the GPU arm: one untimed warm-up evaluation, then timed samples
    (at most --steps, stopped once ~90 s of samples have run); only evaluations are timed."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    spec = WORKLOADS[args.workload]
    ref = CpuReference(args.workload)
    try:
        ref.prepare()
        times: list[float] = []
        spent = 0.0
        while len(times) < max(1, args.steps):
            t0 = time.perf_counter()
            times.append(ref.sample())
            spent += time.perf_counter() - t0
            if spent > 90.0:
                break
    finally:
        ref.close()
    v = 1.0 / statistics.median(times)
    line = {"impl": "reference", "metric": "fwd+bwd graph steps/sec", "value": v, "unit": "steps/s",
            "n_gpus": env_int("WORLD_SIZE", 1), "steps": len(times), "warmup": 1,
            "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic (seeded numpy)",
            "config": {"workload": spec["desc"], "graph": spec["graph"]},
            "timed_region_s": round(spent, 2),
            "cpu_baseline": ref.baseline(v, len(times)),
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gemm_micro(args) -> None:
    """Dominant-kernel microbenchmark: the bf16 tcgen05 GEMM in the three operand layouts
    of the batched-contraction graph (forward NN with bias+ReLU+mask epilogue, dA = G B^T,
    dB = A^T G), 16 x 2048^3 each, CUDA events on the launching stream."""
    import torch

    from b200 import _lib
    from b200 import ops

    torch.cuda.set_device(0)
    Z, M, N, K = 16, 2048, 2048, 2048
    gen = torch.Generator(device="cpu").manual_seed(0)
    A = (torch.randn(Z, M, K, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    B = (torch.randn(Z, K, N, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    G = torch.randn(Z, M, N, generator=gen).to(torch.bfloat16).cuda()
    bias = torch.zeros(N).cuda()
    cases = {
        "fwd_nn_bias_relu_mask": lambda: ops.gemm(A, B, bias=bias, epilogue=_lib.EPI_RELU, want_mask=True, ab_dtype=torch.bfloat16),
        "dA_nt": lambda: ops.gemm(G, B.transpose(-1, -2), ab_dtype=torch.bfloat16),
        "dB_tn": lambda: ops.gemm(A.transpose(-1, -2), G, ab_dtype=torch.bfloat16),
    }
    pk = peaks()
    res = {}
    for name, fn in cases.items():
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        tf = 2.0 * Z * M * N * K / (ms / 1000.0) / 1e12
        res[name] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / pk["bf16_tflops"], 4)}
    print(json.dumps({"microbench": "gemm_bf16_tcgen05", "shape": [Z, M, N, K], "peak_tflops": pk["bf16_tflops"],
                      "peak_source": pk["source"], "cases": res}), flush=True)


def run_optimizer_micro(args) -> None:
    """Optimizer-step microbenchmark: ApplyAdam (the reference numpy backend's formula,
    bit-exact) over every parameter of the pre-LN transformer workload (4 x (d 1024, FFN
    4096), vocab 32000: one launch per 128 tensors, in place), CUDA events on the launching
    stream, against the HBM roofline at 28 bytes per element (read param, m, v, grad;
    write param, m, v). The oracle's numpy step over the same tensors is timed on the host
    cores beside it."""
    import time

    import torch

    from b200 import graph as G
    from b200 import ops
    from oracle import evaluator as O

    torch.cuda.set_device(0)
    g = G.load("transformer_full")
    from b200.workloads import make_inputs

    arrays = make_inputs(g.meta["workload"], g.meta["dims"], seed=0)
    names = [k[2:] for k in g.output_names if k.startswith("d_") and k[2:] in arrays]
    gen = torch.Generator(device="cpu").manual_seed(0)
    params = [torch.from_numpy(np.ascontiguousarray(arrays[r], dtype=np.float32)).cuda() for r in names]
    grads = [torch.randn(p.shape, generator=gen).cuda() * 1e-3 for p in params]
    states = [(torch.zeros_like(p), torch.zeros_like(p)) for p in params]
    out = [(p,) + st for p, st in zip(params, states)]
    n = sum(p.numel() for p in params)

    def step():
        ops.apply_optimizer("ApplyAdam", params, states, grads, lr=1e-3, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pk = peaks()
    gbs = 28.0 * n / (ms / 1000.0) / 1e9
    # the oracle on the host: a bounded sample of the tensors, scaled to all of them
    hp = [p.cpu().numpy() for p in params]
    hg = [x.cpu().numpy() for x in grads]
    done, t0 = 0, time.perf_counter()
    for p, gr in zip(hp, hg):
        m = np.zeros_like(p)
        O.execute_op("ApplyAdam", p, m, m, gr, lr=1e-3)
        done += p.size
        if time.perf_counter() - t0 > 10.0:
            break
    cpu_s = (time.perf_counter() - t0) * n / max(1, done)
    print(json.dumps({"microbench": "apply_adam_f32", "tensors": len(params), "elements": n, "ms": round(ms, 4),
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                   "frac": round(gbs / pk["hbm_gbs"], 4), "bytes_per_element": 28},
                      "cpu_baseline": {"value": round(1.0 / cpu_s, 3), "unit": "steps/s", "cores": 1, "kind": "port",
                                       "sample": f"{done} of {n} elements, scaled"},
                      "peak_source": pk["source"]}), flush=True)


def run_weights_micro(args) -> None:
    """Weight I/O microbenchmark: the pre-LN transformer workload's parameters (116.4 M fp32,
    466 MB) saved from HBM to a safetensors file in the reference's layout and loaded back
    into HBM (file in the page cache after the first pass), wall-clock around each call
    with the device synchronised. Host-side file I/O plus one PCIe copy per direction."""
    import os
    import tempfile
    import time

    import torch

    from b200 import graph as G
    from b200 import weights as W
    from b200.workloads import make_inputs

    torch.cuda.set_device(0)
    g = G.load("transformer_full")
    arrays = make_inputs(g.meta["workload"], g.meta["dims"], seed=0)
    names = [k[2:] for k in g.output_names if k.startswith("d_") and k[2:] in arrays]
    w = {r: torch.from_numpy(np.ascontiguousarray(arrays[r], dtype=np.float32)).cuda() for r in names}
    nbytes = sum(t.numel() * 4 for t in w.values())
    path = os.path.join(tempfile.gettempdir(), "b200_bench_weights.safetensors")
    save_s, load_s = [], []
    try:
        for i in range(max(2, args.steps // 5) + 1):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            W.save_safetensors(w, path)
            t1 = time.perf_counter()
            back = W.load_safetensors(path)
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            if i:  # first pass warms the page cache and the pinned allocator
                save_s.append(t1 - t0)
                load_s.append(t2 - t1)
        ok = all(torch.equal(back[k], w[k]) for k in w)
    finally:
        if os.path.exists(path):
            os.remove(path)
    print(json.dumps({"microbench": "weights_safetensors", "tensors": len(w), "bytes": nbytes, "roundtrip_exact": ok,
                      "save": {"s": round(min(save_s), 4), "GB/s": round(nbytes / min(save_s) / 1e9, 2)},
                      "load": {"s": round(min(load_s), 4), "GB/s": round(nbytes / min(load_s) / 1e9, 2)}}), flush=True)



def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="transformer", choices=sorted(WORKLOADS) + ["gemm", "adam", "weights"])
    ap.add_argument("--only", action="store_true", help="time the --workload alone (no configs block)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-overlap", action="store_true", help="all-reduce after the step instead of during the backward")
    ap.add_argument("--profile", action="store_true",
                    help="bracket one eager step of the headline plan with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    ap.add_argument("--graph", default=None,
                    help="run the headline workload on another of its stored graphs (e.g. transformer_b8, cnn_n64) "
                         "for small profiling captures; its numbers are not the benchmark's")
    # dram__bytes_read.sum + dram__bytes_write.sum of one rowfused2_kernel launch at
    # [8192, 4096] (ncu capture summarised in profiles/rowfused_kernel_8192x4096.md)
    ap.add_argument("--traffic", type=float, default=488077312.0, help="ncu dram bytes per launch of the row kernel")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "gemm":
        run_gemm_micro(args)
    elif args.workload == "adam":
        run_optimizer_micro(args)
    elif args.workload == "weights":
        run_weights_micro(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()

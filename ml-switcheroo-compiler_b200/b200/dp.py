"""Data-parallel execution: one process per GPU, the batch split across ranks, parameter
gradients exchanged with one all-reduce step (NCCL over NVLink on the GPUs).

This is the exchange the reference expresses as ``AllReduce`` / ``NcclAllReduce`` nodes
(``backends/numpy/eager/distributed.py:205-225``, ``all_reduce_ring`` ``:105``) after the
SPMD pass splits the batch (``transforms/passes/spmd.py:636``). Parameters are
replicated, each rank evaluates the fwd+bwd graph on its shard, and the gradients are
combined:

* ``"sum"``  when each shard's graph already divides by the global batch (a graph traced
  at the global batch and evaluated on a shard), or the loss is a sum;
* ``"mean"`` when each rank's graph was traced at its own batch (a mean over the shard):
  the global mean is the average of the shard means.

Small gradients are packed into buckets (contiguous device-to-device copies, no compute)
so a step issues a few large collectives instead of one per parameter. On GPUs, fp32
buckets up to ``peer_below`` bytes skip NCCL: ``PeerAllReduce`` adds the ranks' values
with one kernel over peer-mapped memory (NVLink P2P loads), where a collective's fixed
latency would dominate (the fused row graph's column gradients are 32 KB).
"""

from __future__ import annotations

import os
from typing import Sequence

import torch


def shard_rows(n: int, rank: int, world: int) -> slice:
    """Contiguous share of ``n`` batch rows for ``rank`` (earlier ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    per, rem = divmod(n, world)
    lo = rank * per + min(rank, rem)
    return slice(lo, lo + per + (1 if rank < rem else 0))


class PeerAllReduce:
    """All-reduce of small fp32 buffers through peer-mapped memory
    (``b200_peer_allreduce_f32``): one kernel pushes each value, tagged with its call
    number in one 64-bit word, into every peer's receive area, then adds the words it
    receives in rank order, so all ranks hold bit-identical sums.

    Construction is collective (symmetric-memory rendezvous on ``group``) and must be
    followed by one more collective on ``group`` before the first call, so that every
    receive area is clear. Every rank must then make the same calls with the same sizes,
    and issue all of them on one stream in call order (CUDA graph replays included): the
    receive area is double-buffered by call parity, which is safe only while call e - 2 of
    a rank has finished before its call e starts.

    A wait that gives up sets a status word, and from then on every call on that rank
    returns at once without sending, summing or updating anything; its peers' next waits
    then give up too. ``check()`` turns the status into ``TimeoutError``; ``reset()``
    (collective) clears the receive areas, call counters and status on every rank.
    """

    SPIN_LIMIT = 1 << 24  # polls per thread (backing off to ~256 ns sleeps): seconds, not forever
    MAX_NUMEL = 64 * 4096  # values per call (64 blocks of 4096)

    def __init__(self, group, max_numel: int, device: torch.device) -> None:
        import torch.distributed as dist

        # plain peer mappings only: no NVLink multicast object behind the buffer
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm

        from . import _lib as L
        from . import ops

        self.group, self.device = group, device
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.max_numel = min(int(max_numel), self.MAX_NUMEL)
        # receive area: [2 halves][world sources][max_numel] 64-bit words
        self.buf = symm.empty(2 * self.world * self.max_numel, dtype=torch.int64, device=device)
        self.handle = symm.rendezvous(self.buf, group if group is not None else dist.group.WORLD)
        self.epoch = torch.zeros(64, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        L.call("b200_memset_async", self.buf.data_ptr(), 0, self.buf.numel() * 8, ops.stream_ptr())
        torch.cuda.synchronize(device)
        # the first call must wait until every rank has cleared its area: the caller follows
        # construction with a collective on `group` (GradAllReduce agrees on success)

    MAX_SEGMENTS = 64  # parameter tensors of one fused optimizer epilogue

    def __call__(self, flat: torch.Tensor, scale: float = 1.0, step: "OptimizerStep | None" = None,
                 indices: Sequence[int] = ()) -> None:
        """Sum ``flat`` over the ranks (times ``scale``). With ``step``, the same kernel then
        applies ``step``'s optimizer to its parameters ``indices``, whose gradients are laid
        end to end in ``flat``."""
        import ctypes as C

        from . import _lib as L
        from . import ops

        if flat.dtype != torch.float32 or not flat.is_contiguous() or flat.numel() > self.max_numel:
            raise ValueError("PeerAllReduce takes contiguous fp32 buffers of at most max_numel values")
        n = flat.numel()
        head = (flat.data_ptr(), n, int(self.handle.buffer_ptrs_dev), self.max_numel, self.rank, self.world,
                self.epoch.data_ptr(), self.status.data_ptr(), self.SPIN_LIMIT, float(scale))
        if step is None:
            L.call("b200_peer_allreduce_f32", *head, ops.stream_ptr())
            return
        if not 1 <= len(indices) <= self.MAX_SEGMENTS:
            raise ValueError(f"a fused optimizer epilogue takes 1..{self.MAX_SEGMENTS} tensors")
        offs = [0]
        for i in indices:
            step.check_matches(i)
            offs.append(offs[-1] + step.params[i].numel())
        if offs[-1] != n:
            raise ValueError("the gradients of `indices` must fill `flat` exactly")
        if any(step.params[i].device != flat.device for i in indices):
            raise ValueError("parameters and gradients must be on the same device")
        P = C.c_void_p * len(indices)
        s2 = P(*[step.states[i][1].data_ptr() for i in indices]) if step.nstates == 2 else None
        L.call("b200_peer_allreduce_apply_f32", *head, step.kind, len(indices), (C.c_int64 * len(offs))(*offs),
               P(*[step.params[i].data_ptr() for i in indices]), P(*[step.states[i][0].data_ptr() for i in indices]), s2,
               float(step.lr), ops.stream_ptr())

    def tensors(self, ts: Sequence[torch.Tensor], scale: float = 1.0, step: "OptimizerStep | None" = None,
                indices: Sequence[int] = ()) -> None:
        """Sum each of the contiguous fp32 tensors ``ts`` over the ranks in place (times
        ``scale``) in one kernel, without packing them into one buffer. With ``step``, the
        same kernel applies ``step``'s optimizer to its parameters ``indices`` (one per
        tensor, in order)."""
        import ctypes as C

        from . import _lib as L
        from . import ops

        if not 1 <= len(ts) <= self.MAX_SEGMENTS:
            raise ValueError(f"PeerAllReduce.tensors takes 1..{self.MAX_SEGMENTS} tensors")
        offs = [0]
        for t in ts:
            if t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("PeerAllReduce.tensors takes contiguous fp32 tensors")
            offs.append(offs[-1] + t.numel())
        if offs[-1] > self.max_numel:
            raise ValueError("PeerAllReduce.tensors: more values than the receive capacity")
        P = C.c_void_p * len(ts)
        kind, par, st1, st2, lr = -1, None, None, None, 0.0
        if step is not None:
            if len(indices) != len(ts):
                raise ValueError("one parameter index per tensor")
            for t, i in zip(ts, indices):
                step.check_matches(i, t)
            kind, lr = step.kind, float(step.lr)
            par = P(*[step.params[i].data_ptr() for i in indices])
            st1 = P(*[step.states[i][0].data_ptr() for i in indices])
            st2 = P(*[step.states[i][1].data_ptr() for i in indices]) if step.nstates == 2 else None
        L.call("b200_peer_allreduce_tensors_f32", len(ts), (C.c_int64 * len(offs))(*offs), P(*[t.data_ptr() for t in ts]),
               int(self.handle.buffer_ptrs_dev), self.max_numel, self.rank, self.world, self.epoch.data_ptr(),
               self.status.data_ptr(), self.SPIN_LIMIT, float(scale), kind, par, st1, st2, lr, ops.stream_ptr())

    def failed(self) -> bool:
        """True if a wait for a peer gave up on this rank since construction or the last
        ``reset()`` (reads the device status word: synchronises with the stream)."""
        return int(self.status.item()) != 0

    def check(self) -> None:
        """Raise TimeoutError if a wait for a peer gave up on this rank."""
        code = int(self.status.item())
        if code:
            raise TimeoutError(f"peer all-reduce: a peer's values did not arrive (status {code}); the exchange is "
                               "stopped on this rank until a collective reset()")

    def reset(self) -> None:
        """Collective: clear this rank's receive area, call counters and status, then wait
        for every rank to have done the same, so the next call starts from call 1 on all
        ranks. Every rank of the group must call it, with no exchange in flight."""
        import torch.distributed as dist

        from . import _lib as L
        from . import ops

        torch.cuda.synchronize(self.device)
        L.call("b200_memset_async", self.buf.data_ptr(), 0, self.buf.numel() * 8, ops.stream_ptr())
        self.epoch.zero_()
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


class OptimizerStep:
    """Device optimizer for a list of fp32 parameter tensors, updated in place: ApplyAdam,
    ApplyAdagrad, ApplyFtrl or ApplyRMSProp with the reference numpy backend's formulas
    (``numpy/eager/optimizers_ops.py``), states starting at zero. ``GradAllReduce(grads,
    step)`` applies it after the gradient exchange, fused into the peer-memory kernel for
    the buckets that take that path."""

    def __init__(self, op: str, params: Sequence[torch.Tensor], lr: float | None = None) -> None:
        from . import _lib as L
        from . import ops

        if op not in ops._OPT_KIND:
            raise ValueError(f"unknown optimizer op {op!r}")
        for p in params:
            if p.dtype != torch.float32 or not p.is_cuda or not p.is_contiguous():
                raise ValueError("OptimizerStep updates contiguous fp32 CUDA tensors in place")
        self.op, self.kind = op, ops._OPT_KIND[op]
        self.lr = float(L.lib().b200_optimizer_default_lr(self.kind)) if lr is None else float(lr)
        self.params = list(params)
        self.nstates = 1 if op == "ApplyAdagrad" else 2
        self.states = [tuple(torch.zeros_like(p) for _ in range(self.nstates)) for p in self.params]

    def check_matches(self, i: int, grad: torch.Tensor | None = None) -> None:
        """Raise ValueError unless parameter ``i``, its state arrays and (when given)
        ``grad`` have the same number of elements and device: the kernels index all of them
        with the gradient's offsets and cannot check their extents."""
        p = self.params[i]
        ts = [p, *self.states[i]] + ([grad] if grad is not None else [])
        for t in ts:
            if t.numel() != p.numel() or t.device != p.device:
                raise ValueError(f"optimizer tensor {i}: parameter {tuple(p.shape)} on {p.device}, but a state or "
                                 f"gradient has {t.numel()} elements on {t.device}")

    def apply(self, indices: Sequence[int], grads: Sequence[torch.Tensor]) -> None:
        """One launch: parameters ``indices`` take one step with ``grads`` (same order)."""
        from . import ops

        if not indices:
            return
        ps = [self.params[i] for i in indices]
        sts = [self.states[i] for i in indices]
        ops.apply_optimizer(self.op, ps, sts, list(grads), lr=self.lr, out=[(p,) + st for p, st in zip(ps, sts)])


class GradAllReduce:
    """In-place all-reduce of a list of gradient tensors across the process group, and,
    when given an ``OptimizerStep`` over the matching parameters, the optimizer step."""

    def __init__(self, op: str = "sum", group=None, bucket_bytes: int = 32 << 20, pack_below: int = 4 << 20,
                 peer_below: int = 1 << 20) -> None:
        if op not in ("sum", "mean"):
            raise ValueError(f"op must be 'sum' or 'mean', not {op!r}")
        self.op, self.group = op, group
        self.bucket_bytes, self.pack_below = bucket_bytes, pack_below
        self.peer_below = peer_below if os.environ.get("B200_PEER_ALLREDUCE", "1") != "0" else 0
        self._flat: dict[tuple, torch.Tensor] = {}
        self.peer: PeerAllReduce | None = None
        self._peer_failed = False

    def _peer_for(self, t: torch.Tensor, numel: int | None = None) -> PeerAllReduce | None:
        """The peer-memory path for ``numel`` (default ``t.numel()``) contiguous fp32 values
        on ``t``'s device, set up on first use, or None where it does not apply."""
        import torch.distributed as dist

        numel = t.numel() if numel is None else numel
        if (not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous()
                or numel * 4 > self.peer_below or dist.get_backend(self.group) != "nccl"):
            return None
        if self.peer is None and not self._peer_failed:
            # collective set-up; every rank reports success, and the peer path is used only
            # when all ranks have it (otherwise every rank keeps NCCL for these buckets)
            err = None
            try:
                peer = PeerAllReduce(self.group, self.peer_below // 4, t.device)
            except Exception as e:  # noqa: BLE001 - reported below, ranks agree on the outcome
                peer, err = None, e
            ok = torch.tensor([0 if peer is None else 1], dtype=torch.int32, device=t.device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
            if int(ok.item()) == 1:
                self.peer = peer
            else:
                self._peer_failed = True
                import warnings

                warnings.warn(f"peer-memory all-reduce unavailable on this group, NCCL only ({err!r})")
        return self.peer

    def graph_safe(self, grads: Sequence[torch.Tensor]) -> bool:
        """True when every bucket of ``grads`` goes through the peer-memory kernel (set up
        by an earlier call): no NCCL call and no host synchronisation, so the exchange can
        be captured in a CUDA graph and replayed (its call counters live on the device)."""
        import torch.distributed as dist

        if dist.get_world_size(self.group) == 1:
            return True
        if self.peer is None:
            return False
        for b in self.buckets(grads):
            t = grads[b[0]]
            n = sum(grads[i].numel() for i in b)
            if t.dtype != torch.float32 or not t.is_cuda or n > self.peer.max_numel:
                return False
        return True

    def check(self) -> None:
        """Collective: raise TimeoutError if a peer-memory exchange gave up waiting on any
        rank. The ranks agree on the outcome (one small all-reduce), and after a failure
        every rank drops the peer path and exchanges through NCCL from then on, so no rank
        keeps using an exchange whose call numbers have diverged. Parameters updated by a
        fused optimizer epilogue may differ across ranks after a failure: re-broadcast them
        before continuing. Call it on every rank at the same point (for instance once per
        step or every few steps)."""
        import torch.distributed as dist

        if self.peer is None:
            return
        bad = torch.tensor([1 if self.peer.failed() else 0], dtype=torch.int32, device=self.peer.device)
        if dist.get_world_size(self.group) > 1:
            dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=self.group)
        if int(bad.item()):
            self.peer, self._peer_failed = None, True
            raise TimeoutError("peer all-reduce: a wait for a peer gave up on some rank; the peer path is off and "
                               "later exchanges use NCCL. Parameters stepped by the fused optimizer may differ "
                               "across ranks: re-broadcast them.")

    def _reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        world = dist.get_world_size(self.group)
        if world == 1:
            return
        peer = self._peer_for(t)
        if peer is not None:
            peer(t.reshape(-1), 1.0 / world if self.op == "mean" else 1.0)
            return
        if self.op == "mean" and dist.get_backend(self.group) == "nccl":
            dist.all_reduce(t, op=dist.ReduceOp.AVG, group=self.group)
            return
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        if self.op == "mean":
            t.div_(world)  # host-side reduction on CPU process groups (gloo has no AVG)

    def buckets(self, grads: Sequence[torch.Tensor]) -> list[list[int]]:
        """Indices of the gradients reduced together: large ones alone, small ones packed
        in order up to ``bucket_bytes`` per bucket (same dtype and device)."""
        out: list[list[int]] = []
        cur: list[int] = []
        size = 0
        for i, g in enumerate(grads):
            nb = g.numel() * g.element_size()
            if nb >= self.pack_below or not g.is_contiguous():
                out.append([i])
                continue
            if cur and (size + nb > self.bucket_bytes or grads[cur[0]].dtype != g.dtype or grads[cur[0]].device != g.device):
                out.append(cur)
                cur, size = [], 0
            cur.append(i)
            size += nb
        if cur:
            out.append(cur)
        return out

    def __call__(self, grads: Sequence[torch.Tensor], step: OptimizerStep | None = None) -> None:
        import torch.distributed as dist

        if step is not None:
            if len(step.params) != len(grads):
                raise ValueError("the optimizer step must cover the same tensors as the gradients")
            for i, g in enumerate(grads):
                step.check_matches(i, g)
        world = dist.get_world_size(self.group)
        for b in self.buckets(grads):
            if len(b) == 1:
                g = grads[b[0]]
                peer = self._peer_for(g) if world > 1 and step is not None else None
                if peer is not None:  # exchange and step in one kernel
                    peer(g.reshape(-1), 1.0 / world if self.op == "mean" else 1.0, step, b)
                    continue
                self._reduce(g)
                if step is not None:
                    step.apply(b, [g])
                continue
            ts = [grads[i] for i in b]
            n = sum(t.numel() for t in ts)
            if (world > 1 and len(b) <= PeerAllReduce.MAX_SEGMENTS and ts[0].dtype == torch.float32
                    and all(t.is_contiguous() for t in ts)):
                peer = self._peer_for(ts[0], n)
                if peer is not None:  # one kernel over the tensors themselves: no packing copies
                    peer.tensors(ts, 1.0 / world if self.op == "mean" else 1.0, step, b if step is not None else ())
                    continue
            key = (ts[0].dtype, str(ts[0].device), n)
            flat = self._flat.get(key)
            if flat is None:
                flat = torch.empty(n, dtype=ts[0].dtype, device=ts[0].device)
                self._flat[key] = flat
            off = 0
            for t in ts:  # contiguous copies: device-to-device memcpy, no kernel
                flat[off : off + t.numel()].copy_(t.reshape(-1))
                off += t.numel()
            peer = (self._peer_for(flat) if world > 1 and step is not None and len(b) <= PeerAllReduce.MAX_SEGMENTS
                    else None)
            if peer is not None:
                peer(flat, 1.0 / world if self.op == "mean" else 1.0, step, b)
            else:
                self._reduce(flat)
            off = 0
            for t in ts:
                t.reshape(-1).copy_(flat[off : off + t.numel()])
                off += t.numel()
            if step is not None and peer is None:
                step.apply(b, ts)


class OverlappedStep:
    """One data-parallel fwd+bwd step with the gradient all-reduce overlapped with the
    backward pass.

    The reference puts its ``AllReduce`` nodes after the whole backward
    (``transforms/passes/spmd.py:636``); here each gradient is exchanged as soon as the
    step that writes it (and every step that reads it) has run. The fused plan is captured
    as a few CUDA graphs, split where a bucket of gradients becomes final: gradients are
    grouped in the order the backward finishes them, ``bucket_bytes`` or more per bucket.
    A replay runs the segments on the current (compute) stream; after each one an event
    releases that segment's buckets to a communication stream, which all-reduces them with
    ``GradAllReduce`` (NCCL, or the peer-memory kernel for small fp32 buckets) while the
    next segment computes. The compute stream waits for the communication stream at the
    end, so the returned gradients are the all-reduced ones.

    The segments share one CUDA graph memory pool and always replay in capture order, so
    memory one segment frees can be reused by a later one exactly as inside one graph.
    Gradients are graph outputs and are never freed, so the communication stream can read
    and write them while later segments run."""

    def __init__(self, graph, inputs: dict, grad_ids: Sequence[str], sync: "GradAllReduce",
                 bucket_bytes: int = 48 << 20, max_segments: int = 8) -> None:
        from . import ops
        from .executor import GraphRunner

        self.runner = GraphRunner(graph)
        self.sync = sync
        self.static_in = {k: (ops.copy(v) if isinstance(v, torch.Tensor) else v) for k, v in inputs.items()}
        plan = self.runner.plan_for(self.static_in)
        self.plan = plan
        last = plan.last_use()
        n = len(plan.steps)
        ready = sorted((last.get(gid, n - 1), k, gid) for k, gid in enumerate(grad_ids))
        # warm-up run (eager, side stream): allocations settle, output shapes known
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            out = plan.run(dict(self.static_in))
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        sizes = {gid: out[gid].numel() * out[gid].element_size() for gid in grad_ids}
        del out
        # buckets in finishing order; a bucket is released after its last gradient's step
        buckets: list[tuple[int, list[str]]] = []
        cur: list[str] = []
        acc = 0
        for pos, _, gid in ready:
            cur.append(gid)
            acc += sizes[gid]
            if acc >= bucket_bytes:
                buckets.append((pos, cur))
                cur, acc = [], 0
        if cur:
            buckets.append((ready[-1][0], cur))
        # at most max_segments segments: merge the earliest buckets when there are more
        while len(buckets) > max_segments:
            (p0, b0), (p1, b1) = buckets[0], buckets[1]
            buckets[0:2] = [(max(p0, p1), b0 + b1)]
        self.buckets = buckets
        cuts = sorted({p + 1 for p, _ in buckets} | {n})
        self.bounds = list(zip([0] + cuts[:-1], cuts))
        self.release = {}  # segment index -> bucket lists released after it
        for p, b in buckets:
            seg = next(i for i, (lo, hi) in enumerate(self.bounds) if lo <= p < hi)
            self.release.setdefault(seg, []).append(b)
        # capture the segments into graphs sharing one memory pool
        pool = torch.cuda.graph_pool_handle()
        self.graphs: list[torch.cuda.CUDAGraph] = []
        env = plan.begin(self.static_in)
        try:
            for lo, hi in self.bounds:
                cg = torch.cuda.CUDAGraph()
                with torch.cuda.graph(cg, pool=pool):
                    plan.run_steps(env, lo, hi)
                self.graphs.append(cg)
        finally:
            self.static_out = plan.finish(env)
        self.comm = torch.cuda.Stream()
        self.events = [torch.cuda.Event() for _ in self.bounds]

    def __call__(self, inputs: dict | None = None) -> dict:
        """Replay one step (inputs, when given, are copied into the static buffers first)
        and return the graph's outputs with the gradients all-reduced."""
        if inputs:
            for k, v in inputs.items():
                dst = self.static_in[k]
                if isinstance(dst, torch.Tensor) and v is not dst:
                    dst.copy_(v, non_blocking=True)
        compute = torch.cuda.current_stream()
        for i, g in enumerate(self.graphs):
            g.replay()
            if i in self.release:
                self.events[i].record(compute)
                self.comm.wait_event(self.events[i])
                with torch.cuda.stream(self.comm):
                    for b in self.release[i]:
                        self.sync([self.static_out[gid] for gid in b])
        compute.wait_stream(self.comm)
        return self.static_out

    def describe(self) -> dict:
        return {"segments": len(self.graphs), "buckets": [len(b) for _, b in self.buckets],
                "released_after_steps": [p for p, _ in self.buckets]}

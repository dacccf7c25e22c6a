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
so a step issues a few large collectives instead of one per parameter.
"""

from __future__ import annotations

from typing import Sequence

import torch


def shard_rows(n: int, rank: int, world: int) -> slice:
    """Contiguous share of ``n`` batch rows for ``rank`` (earlier ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    per, rem = divmod(n, world)
    lo = rank * per + min(rank, rem)
    return slice(lo, lo + per + (1 if rank < rem else 0))


class GradAllReduce:
    """In-place all-reduce of a list of gradient tensors across the process group."""

    def __init__(self, op: str = "sum", group=None, bucket_bytes: int = 32 << 20, pack_below: int = 4 << 20) -> None:
        if op not in ("sum", "mean"):
            raise ValueError(f"op must be 'sum' or 'mean', not {op!r}")
        self.op, self.group = op, group
        self.bucket_bytes, self.pack_below = bucket_bytes, pack_below
        self._flat: dict[tuple, torch.Tensor] = {}

    def _reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        world = dist.get_world_size(self.group)
        if world == 1:
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

    def __call__(self, grads: Sequence[torch.Tensor]) -> None:
        for b in self.buckets(grads):
            if len(b) == 1:
                self._reduce(grads[b[0]])
                continue
            ts = [grads[i] for i in b]
            n = sum(t.numel() for t in ts)
            key = (ts[0].dtype, str(ts[0].device), n)
            flat = self._flat.get(key)
            if flat is None:
                flat = torch.empty(n, dtype=ts[0].dtype, device=ts[0].device)
                self._flat[key] = flat
            off = 0
            for t in ts:  # contiguous copies: device-to-device memcpy, no kernel
                flat[off : off + t.numel()].copy_(t.reshape(-1))
                off += t.numel()
            self._reduce(flat)
            off = 0
            for t in ts:
                t.reshape(-1).copy_(flat[off : off + t.numel()])
                off += t.numel()

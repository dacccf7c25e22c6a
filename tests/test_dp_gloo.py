"""Host-side data-parallel logic on CPU: world-size-2 gloo process groups.

* batch sharding covers every row exactly once;
* the bucketed gradient all-reduce sums / averages like the reference's AllReduce
  known-answer test (``tests/distributed/test_multi_process_collectives.py:83-103``:
  ranks holding [r+1, 2(r+1)] reduce to the sum);
* the exchange reproduces the single-process gradients: each rank evaluates the
  reference-traced MLP graph (oracle) on its shard of the batch, the shard gradients are
  all-reduced, and the result equals the full-batch gradients.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def test_shard_rows_cover_the_batch():
    from b200.dp import shard_rows

    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                s = shard_rows(n, r, world)
                rows.extend(range(n)[s])
            assert rows == list(range(n)), (n, world)
    with pytest.raises(ValueError):
        shard_rows(4, 2, 2)


def test_bucket_plan_packs_small_gradients():
    from b200.dp import GradAllReduce

    grads = [torch.zeros(10), torch.zeros(1 << 21), torch.zeros(3), torch.zeros(5, dtype=torch.float64), torch.zeros(7)]
    plan = GradAllReduce(pack_below=1 << 20).buckets(grads)
    assert sorted(i for b in plan for i in b) == list(range(len(grads)))
    assert [1] in plan  # 8 MB alone
    for b in plan:
        assert len({grads[i].dtype for i in b}) == 1


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "ml-switcheroo-compiler_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from b200.dp import GradAllReduce, shard_rows
    from conftest import load_golden
    from oracle import evaluator as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # known answer: [r+1, 2(r+1)] summed and averaged, plus packed small tensors
        a = torch.tensor([rank + 1.0, 2.0 * (rank + 1)])
        b = torch.full((3,), float(rank))
        GradAllReduce("sum", pack_below=1 << 20)([a, b])
        c = torch.tensor([rank + 1.0, 2.0 * (rank + 1)])
        GradAllReduce("mean")([c])
        # shard gradients of the reference-traced MLP graph (it divides by the global batch,
        # so the shard gradients sum to the full-batch gradients)
        ins, _ = load_golden("mlp_small")
        g = O.load_graph("mlp_small")
        s = shard_rows(ins["x"].shape[0], rank, world)
        mine = dict(ins)
        mine["x"], mine["labels"] = ins["x"][s], ins["labels"][s]
        res = O.evaluate_roles(g, mine)
        names = sorted(k for k in res if k.startswith("d_"))
        grads = [torch.from_numpy(np.ascontiguousarray(res[k], dtype=np.float32)) for k in names]
        GradAllReduce("sum", pack_below=1 << 16)(grads)
        q.put((rank, a.tolist(), b.tolist(), c.tolist(), {k: t.numpy() for k, t in zip(names, grads)}))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gradient_exchange():
    from conftest import load_golden
    from oracle import evaluator as O

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get() for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ins, _ = load_golden("mlp_small")
    full = O.evaluate_roles(O.load_graph("mlp_small"), ins)
    for rank, a, b, c, grads in results:
        assert a == [3.0, 6.0]
        assert b == [1.0, 1.0, 1.0]
        assert c == [1.5, 3.0]
        for k, v in grads.items():
            np.testing.assert_allclose(v, full[k], rtol=1e-5, atol=1e-6 * float(np.abs(full[k]).max()), err_msg=k)


def _bare_step(params, nstates=2):
    """An OptimizerStep over host tensors, built without its CUDA-only constructor: only
    the shape checks are exercised, no kernel runs."""
    from b200.dp import OptimizerStep

    st = OptimizerStep.__new__(OptimizerStep)
    st.op, st.kind, st.lr, st.nstates = "ApplyAdam", 0, 1e-3, nstates
    st.params = list(params)
    st.states = [tuple(torch.zeros_like(p) for _ in range(nstates)) for p in st.params]
    return st


def test_optimizer_step_rejects_mismatched_tensors():
    """A parameter, state or gradient whose element count differs from its partner's is
    rejected on the host before any exchange or kernel: the kernels index them all with the
    gradient's offsets and would write past the end of the smaller one."""
    from b200.dp import GradAllReduce

    step = _bare_step([torch.zeros(8), torch.zeros(3, 5)])
    step.check_matches(0, torch.zeros(8))
    with pytest.raises(ValueError):
        step.check_matches(1, torch.zeros(16))
    with pytest.raises(ValueError):
        GradAllReduce("sum")([torch.zeros(8), torch.zeros(16)], step)  # raises before any collective
    bad_state = _bare_step([torch.zeros(8)])
    bad_state.states[0] = (torch.zeros(8), torch.zeros(7))
    with pytest.raises(ValueError):
        bad_state.check_matches(0, torch.zeros(8))


class _FakePeer:
    """Stands in for PeerAllReduce: only its failure status is read by check()."""

    def __init__(self, failed: bool) -> None:
        self._failed = failed
        self.device = torch.device("cpu")

    def failed(self) -> bool:
        return self._failed


def _check_rank_main(rank: int, world: int, port: int, q) -> None:
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (here, root, os.path.join(root, "ml-switcheroo-compiler_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    from b200.dp import GradAllReduce

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        sync = GradAllReduce("sum")
        sync.peer = _FakePeer(failed=(rank == 1))  # only rank 1's wait gave up
        raised = False
        try:
            sync.check()
        except TimeoutError:
            raised = True
        # after the failure every rank exchanges through the collective library
        t = torch.tensor([float(rank + 1)])
        sync([t])
        q.put((rank, raised, sync.peer is None, sync._peer_failed, t.item()))
    finally:
        dist.destroy_process_group()


def test_peer_timeout_is_agreed_and_fatal_on_every_rank():
    """A timeout seen by one rank makes check() raise on every rank, and every rank drops
    the peer path, so no rank keeps exchanging with diverged call numbers."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_check_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get() for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, raised, dropped, failed, val in results:
        assert raised and dropped and failed, rank
        assert val == 3.0

"""The peer-memory all-reduce kernel (``b200_peer_allreduce_f32``).

On one GPU every case is a single kernel launch that waits on no other kernel:
* world 1: the values come back times ``scale``;
* an emulated world-2 exchange: the peer's words (value + call number) are written into
  this rank's receive area beforehand, so the kernel finds them and adds the two ranks'
  values in rank order (also with the fused optimizer epilogue);
* the bounded wait: words that never arrive make the kernel give up, report
  B200_ERR_TIMEOUT through the status word and leave the values unchanged.
With two or more GPUs, ``GradAllReduce`` over NCCL process groups (peer kernel for the
small fp32 bucket) is checked against NCCL's own all-reduce.
"""

import os
import queue as queue_mod
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


def _words(values: torch.Tensor, call: int) -> torch.Tensor:
    """The 64-bit words a rank pushes: call number in the high half, value bits in the low."""
    return (values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (call << 32)


def _area(world, cap):
    return torch.zeros(2 * world * cap, dtype=torch.int64, device="cuda")


def _run(data, bufs, cap, rank, world, epoch, status, spin, scale):
    from b200 import _lib as L
    from b200 import ops

    tab = _ptrs(bufs)  # alive until the kernel has run
    L.call("b200_peer_allreduce_f32", data.data_ptr(), data.numel(), tab.data_ptr(), cap, rank, world, epoch.data_ptr(),
           status.data_ptr(), spin, scale, ops.stream_ptr())
    torch.cuda.synchronize()


@pytest.mark.parametrize("n", [1, 8192, 100000])
def test_peer_allreduce_world1_and_emulated_pair(cuda, n):
    from b200 import _lib as L

    blocks = int(L.lib().b200_peer_allreduce_blocks(n))
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).cuda()
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # world 1
    d = x.clone()
    _run(d, [_area(1, n)], n, 0, 1, epoch, status, 1000, 0.5)
    assert int(status.item()) == 0
    assert torch.equal(d, x * 0.5)
    assert epoch[:blocks].tolist() == [1] * blocks
    # world 2, this rank 0, call 1 (half 1): rank 1's words already in this rank's area
    y = torch.randn(n, generator=g).cuda()
    a0, a1 = _area(2, n), _area(2, n)
    a0[(1 * 2 + 1) * n : (1 * 2 + 2) * n] = _words(y, 1)
    epoch.zero_()
    d = x.clone()
    _run(d, [a0, a1], n, 0, 2, epoch, status, 1 << 20, 1.0)
    assert int(status.item()) == 0
    assert torch.equal(d, x + y)  # rank order: rank 0's value first
    assert torch.equal(a1[(1 * 2 + 0) * n : (1 * 2 + 1) * n], _words(x, 1))  # this rank's words reached the peer


@pytest.mark.parametrize("op", ["ApplyAdam", "ApplyAdagrad", "ApplyFtrl", "ApplyRMSProp"])
def test_peer_allreduce_fused_optimizer_step_emulated_pair(cuda, op):
    """Exchange plus optimizer epilogue in one kernel: two parameter tensors laid end to
    end, the peer's words planted in this rank's area; the summed gradients and the updated
    parameters / states equal the oracle's step on the summed gradients bit for bit."""
    import ctypes as C

    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O

    rng = np.random.default_rng(9)
    sizes = [1000, 3333]
    n = sum(sizes)
    nst = 1 if op == "ApplyAdagrad" else 2
    host_p = [rng.standard_normal(k).astype(np.float32) for k in sizes]
    host_s = [[np.abs(rng.standard_normal(k)).astype(np.float32) * np.float32(0.1) for _ in range(nst)] for k in sizes]
    x = rng.standard_normal(n).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    params = [torch.from_numpy(p).cuda() for p in host_p]
    states = [[torch.from_numpy(v).cuda() for v in st] for st in host_s]
    data = torch.from_numpy(x).cuda()
    a0, a1 = _area(2, n), _area(2, n)
    a0[3 * n : 4 * n] = _words(torch.from_numpy(y).cuda(), 1)
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = C.c_void_p * 2
    offs = (C.c_int64 * 3)(0, sizes[0], n)
    s2 = P(*[st[1].data_ptr() for st in states]) if nst == 2 else None
    tab = _ptrs([a0, a1])  # alive until the kernel has run
    L.call("b200_peer_allreduce_apply_f32", data.data_ptr(), n, tab.data_ptr(), n, 0, 2, epoch.data_ptr(), status.data_ptr(),
           1 << 20, 1.0, ops._OPT_KIND[op], 2, offs, P(*[q.data_ptr() for q in params]),
           P(*[st[0].data_ptr() for st in states]), s2, 0.01, ops.stream_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    g = x + y
    np.testing.assert_array_equal(data.cpu().numpy(), g)
    lo = 0
    for k, size in enumerate(sizes):
        ref = O.execute_op(op, host_p[k], *host_s[k], g[lo : lo + size], lr=0.01)
        got = [params[k]] + list(states[k])
        for r, t in zip(ref, got):
            np.testing.assert_array_equal(t.cpu().numpy(), r)
        lo += size


@pytest.mark.parametrize("with_step", [False, True])
def test_peer_allreduce_tensors_in_place_emulated_pair(cuda, with_step):
    """The exchange over two tensors without packing (values read from and sums written
    back to the tensors themselves), optionally with the Adam epilogue; the peer's words
    planted in this rank's area as in the flat case."""
    import ctypes as C

    from b200 import _lib as L
    from b200 import ops
    from oracle import evaluator as O

    rng = np.random.default_rng(11)
    sizes = [1000, 3333]
    n = sum(sizes)
    xs = [rng.standard_normal(k).astype(np.float32) for k in sizes]
    y = rng.standard_normal(n).astype(np.float32)
    ts = [torch.from_numpy(x).cuda() for x in xs]
    a0, a1 = _area(2, n), _area(2, n)
    a0[3 * n : 4 * n] = _words(torch.from_numpy(y).cuda(), 1)
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = C.c_void_p * 2
    offs = (C.c_int64 * 3)(0, sizes[0], n)
    host_p = [rng.standard_normal(k).astype(np.float32) for k in sizes]
    params = [torch.from_numpy(q).cuda() for q in host_p]
    ms = [torch.zeros(k, device="cuda") for k in sizes]
    vs = [torch.zeros(k, device="cuda") for k in sizes]
    tab = _ptrs([a0, a1])  # alive until the kernel has run
    L.call("b200_peer_allreduce_tensors_f32", 2, offs, P(*[t.data_ptr() for t in ts]), tab.data_ptr(), n, 0, 2,
           epoch.data_ptr(), status.data_ptr(), 1 << 20, 0.5, ops._OPT_KIND["ApplyAdam"] if with_step else -1,
           P(*[q.data_ptr() for q in params]) if with_step else None, P(*[m.data_ptr() for m in ms]) if with_step else None,
           P(*[v.data_ptr() for v in vs]) if with_step else None, 0.01, ops.stream_ptr())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    lo = 0
    for k, size in enumerate(sizes):
        g = (xs[k] + y[lo : lo + size]) * np.float32(0.5)
        np.testing.assert_array_equal(ts[k].cpu().numpy(), g)
        if with_step:
            ref = O.execute_op("ApplyAdam", host_p[k], np.zeros(size, np.float32), np.zeros(size, np.float32), g, lr=0.01)
            for r, t in zip(ref, (params[k], ms[k], vs[k])):
                np.testing.assert_array_equal(t.cpu().numpy(), r)
        else:
            np.testing.assert_array_equal(params[k].cpu().numpy(), host_p[k])
        lo += size
    assert torch.equal(a1[2 * n : 3 * n], _words(torch.from_numpy(np.concatenate(xs)).cuda(), 1))


def test_peer_allreduce_wait_gives_up(cuda):
    n = 4096
    x = torch.arange(n, dtype=torch.float32, device="cuda")
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = x.clone()
    _run(d, [_area(2, n), _area(2, n)], n, 0, 2, epoch, status, 2000, 1.0)  # rank 1 never sends
    assert int(status.item()) == 4  # B200_ERR_TIMEOUT
    assert torch.equal(d, x)
    assert int(epoch[0].item()) == 0


def test_peer_allreduce_after_timeout_refuses_stale_words(cuda):
    """A timeout is fatal: after one, the peer's words of the call that timed out are
    planted under the call number this rank expects next (what a peer that did complete
    that call leaves behind). The next call must not add them: it returns at once with the
    values unchanged, the status still set and the call counter not advanced."""
    n = 4096
    x = torch.arange(n, dtype=torch.float32, device="cuda")
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a0, a1 = _area(2, n), _area(2, n)
    d = x.clone()
    _run(d, [a0, a1], n, 0, 2, epoch, status, 2000, 1.0)  # rank 1 never sends: times out
    assert int(status.item()) == 4 and torch.equal(d, x) and int(epoch[0].item()) == 0
    stale = torch.full((n,), 7.0, device="cuda")
    a0[(1 * 2 + 1) * n : (1 * 2 + 2) * n] = _words(stale, 1)  # peer's words of call 1, half 1
    a1.zero_()
    _run(d, [a0, a1], n, 0, 2, epoch, status, 1 << 20, 1.0)
    assert torch.equal(d, x), "a call after a timeout added a stale peer word"
    assert int(status.item()) == 4
    assert int(epoch[0].item()) == 0
    assert int(a1.abs().sum().item()) == 0, "a call after a timeout still sent words"
    # a collective reset (areas, counters and status cleared) re-opens the exchange
    status.zero_()
    a0.zero_()
    y = torch.randn(n, device="cuda")
    a0[(1 * 2 + 1) * n : (1 * 2 + 2) * n] = _words(y, 1)
    _run(d, [a0, a1], n, 0, 2, epoch, status, 1 << 20, 1.0)
    assert int(status.item()) == 0
    assert torch.equal(d, x + y)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "ml-switcheroo-compiler_b200"))
    sys.path.insert(0, os.path.dirname(here))
    import torch.distributed as dist

    from b200.dp import GradAllReduce

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(100 + rank)
        grads = [torch.randn(4096, generator=g).cuda(), torch.randn(4096, generator=g).cuda(),
                 torch.randn(3, 5, generator=g).cuda()]
        ref = [t.clone() for t in grads]
        sync = GradAllReduce("mean")
        ok = []
        for step in range(5):  # several calls: both halves of the slot buffer, growing flags
            mine = [t * (step + 1) for t in ref]
            sync(mine)
            nccl = [t * (step + 1) for t in ref]
            for t in nccl:
                dist.all_reduce(t, op=dist.ReduceOp.SUM)
                t.div_(world)
            ok.append(all(torch.allclose(a, b, rtol=1e-6, atol=1e-6) for a, b in zip(mine, nccl)))
        # the exchange with a fused Adam step: every rank ends with the same parameters,
        # equal to one step on the mean gradient
        from b200.dp import OptimizerStep
        from oracle import evaluator as O

        params = [torch.full((4096,), 0.5, device="cuda"), torch.linspace(-1, 1, 15, device="cuda").reshape(3, 5)]
        gs = [torch.randn(4096, generator=g).cuda(), torch.randn(3, 5, generator=g).cuda()]
        mean = [t.clone() for t in gs]
        for t in mean:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            t.div_(world)
        step = OptimizerStep("ApplyAdam", params, lr=0.01)
        p0 = [t.cpu().numpy() for t in params]
        sync(gs, step)
        sync.check()
        for pr, p_init, gm in zip(params, p0, mean):
            ref = O.execute_op("ApplyAdam", p_init, np.zeros_like(p_init), np.zeros_like(p_init), gm.cpu().numpy(), lr=0.01)
            ok.append(bool(np.allclose(pr.cpu().numpy(), ref[0], rtol=1e-6, atol=1e-7)))
        q.put((rank, ok, sync.peer is not None, [t.cpu() for t in mine] + [t.cpu() for t in params]))
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_grad_allreduce_peer_path_matches_nccl():
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(world):
            res.append(q.get(timeout=240))  # a rank that failed never reports: give up, do not wait forever
    except queue_mod.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join(timeout=10)
    assert [p.exitcode for p in procs] == [0] * world, [p.exitcode for p in procs]
    assert len(res) == world
    res.sort(key=lambda r: r[0])
    for rank, ok, used_peer, _ in res:
        assert used_peer and all(ok), (rank, ok, used_peer)
    for a, b in zip(res[0][3], res[1][3]):
        assert torch.equal(a, b)  # bit-identical on both ranks


def _overlap_rank_main(rank: int, world: int, port: int, q) -> None:
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "ml-switcheroo-compiler_b200"))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from b200 import graph as G
        from b200.dp import GradAllReduce, OverlappedStep
        from b200.executor import CompiledGraph
        from b200.workloads import make_inputs
        from gpu_helpers import set_policy

        g = G.load("transformer_small")
        set_policy("transformer")
        arrays = make_inputs(g.meta["workload"], g.meta["dims"], seed=10 + rank)  # each rank its own shard
        inputs = {nid: torch.from_numpy(np.ascontiguousarray(arrays[r])).cuda() for r, nid in g.roles.items()}
        grads = [g.output_names[k] for k in g.output_names if k.startswith("d_")]
        # small buckets: several segments and a release after each
        ov = OverlappedStep(g, inputs, grads, GradAllReduce("mean"), bucket_bytes=64 << 10)
        outs = []
        for _ in range(3):
            o = ov()
            outs.append({k: o[k].clone() for k in grads})
        torch.cuda.synchronize()
        cg = CompiledGraph(g)
        ref = cg(inputs)
        ref = {k: ref[k].clone() for k in grads}
        GradAllReduce("mean")([ref[k] for k in grads])
        torch.cuda.synchronize()
        ok = [all(torch.allclose(o[k], ref[k], rtol=1e-6, atol=1e-7) for k in grads) for o in outs]
        q.put((rank, ok, ov.describe(), [ref[k].cpu() for k in grads]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_overlapped_step_matches_exchange_after_the_step():
    """The data-parallel step with each gradient bucket all-reduced during the backward
    (segmented CUDA-graph replay + a communication stream) gives the same gradients as
    the whole step followed by the exchange, on every rank, over several replays."""
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_overlap_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(world):
            res.append(q.get(timeout=240))
    except queue_mod.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join(timeout=10)
    assert [p.exitcode for p in procs] == [0] * world, [p.exitcode for p in procs]
    assert len(res) == world
    res.sort(key=lambda r: r[0])
    for rank, ok, desc, _ in res:
        assert all(ok), (rank, ok, desc)
        assert desc["segments"] > 1, desc
    for a, b in zip(res[0][3], res[1][3]):
        assert torch.equal(a, b)  # identical gradients on both ranks

"""The peer-memory all-reduce kernel (``b200_peer_allreduce_f32``).

On one GPU every case is a single kernel launch that waits on no other kernel:
* world 1: the values come back times ``scale``;
* an emulated world-2 exchange: the peer's slot and its flag are written beforehand, so
  the kernel finds them and adds the two ranks' values in rank order;
* the bounded wait: a flag that nothing sets makes the kernel give up, report
  B200_ERR_TIMEOUT through the status word and leave the values unchanged.
With two or more GPUs, ``GradAllReduce`` over NCCL process groups (peer kernel for the
small fp32 bucket) is checked against NCCL's own all-reduce.
"""

import os
import queue as queue_mod
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


def _run(data, slots, pads, rank, world, epoch, status, spin, scale, blocks):
    from b200 import _lib as L
    from b200 import ops

    sd, pd = _ptrs(slots), _ptrs(pads)
    L.call("b200_peer_allreduce_f32", data.data_ptr(), data.numel(), sd.data_ptr(), pd.data_ptr(), rank, world,
           epoch.data_ptr(), status.data_ptr(), spin, scale, blocks, ops.stream_ptr())
    torch.cuda.synchronize()


@pytest.mark.parametrize("n,blocks", [(1, 1), (8192, 1), (100000, 4)])
def test_peer_allreduce_world1_and_emulated_pair(cuda, n, blocks):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, generator=g).cuda()
    # world 1
    buf = torch.zeros(2 * n, device="cuda")
    pad = torch.zeros(64, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = x.clone()
    _run(d, [buf], [pad], 0, 1, epoch, status, 1000, 0.5, blocks)
    assert int(status.item()) == 0
    assert torch.equal(d, x * 0.5)
    assert epoch[:blocks].tolist() == [1] * blocks
    # world 2, this rank 0; rank 1's values for call 1 already in its slot (half 1) and its
    # flags raised in rank 0's pad
    y = torch.randn(n, generator=g).cuda()
    buf0, buf1 = torch.zeros(2 * n, device="cuda"), torch.zeros(2 * n, device="cuda")
    buf1[n:] = y
    pad0 = torch.zeros(2 * blocks, dtype=torch.int32, device="cuda")
    pad1 = torch.zeros(2 * blocks, dtype=torch.int32, device="cuda")
    pad0[1::2] = 1  # slot b * world + 1: peer 1, call 1
    epoch.zero_()
    d = x.clone()
    _run(d, [buf0, buf1], [pad0, pad1], 0, 2, epoch, status, 1 << 20, 1.0, blocks)
    assert int(status.item()) == 0
    assert torch.equal(d, x + y)  # rank order: rank 0's value first
    assert torch.equal(buf0[n:], x)  # this rank's values landed in its slot
    assert pad1[0::2].tolist() == [1] * blocks  # and its flags in the peer's pad


def test_peer_allreduce_wait_gives_up(cuda):
    n = 4096
    x = torch.arange(n, dtype=torch.float32, device="cuda")
    bufs = [torch.zeros(2 * n, device="cuda") for _ in range(2)]
    pads = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = x.clone()
    _run(d, bufs, pads, 0, 2, epoch, status, 2000, 1.0, 1)  # nobody raises rank 1's flag
    assert int(status.item()) == 4  # B200_ERR_TIMEOUT
    assert torch.equal(d, x)
    assert int(epoch[0].item()) == 0


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
        sync.check()
        q.put((rank, ok, sync.peer is not None, [t.cpu() for t in mine]))
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

"""The sharded exact-MSE path through the real kernels and NCCL (one rank in a
child process: the same code the multi-GPU sweep runs per rank)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _child(port, q):
    import torch.distributed as dist

    import frame_analytics_b200 as fa
    from frame_analytics_b200.distributed import sharded_mse
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        g = torch.Generator(device="cuda").manual_seed(0)
        res = []
        for dt in (torch.uint8, torch.uint16):
            hi = 256 if dt == torch.uint8 else 65536
            x = torch.randint(0, hi, (5, 3, 70, 90), generator=g, device="cuda",
                              dtype=torch.int32).to(dt)
            y = torch.randint(0, hi, (5, 3, 70, 90), generator=g, device="cuda",
                              dtype=torch.int32).to(dt)
            per, total = sharded_mse(x, y, 5)
            res.append(torch.equal(per, fa.mse(x, y, reduction="none"))
                       and total == float(fa.mse(x, y)))
        q.put(res)
    finally:
        dist.destroy_process_group()


def test_sharded_exact_mse_one_rank_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(_port(), q))
    p.start()
    res = q.get(timeout=300)
    p.join(timeout=60)
    assert res == [True, True]


def _ranks(rank, world, port, q):
    import torch.distributed as dist

    import frame_analytics_b200 as fa
    from frame_analytics_b200.distributed import ShardedMetrics, shard_bounds
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        n = 7
        g = torch.Generator().manual_seed(3)
        x = torch.randint(0, 256, (n, 3, 200, 240), generator=g, dtype=torch.uint8)
        y = (x.to(torch.int16) + torch.randint(-9, 10, x.shape, generator=g,
                                                dtype=torch.int16)).clamp(0, 255).to(torch.uint8)
        lo, hi = shard_bounds(n, rank, world)
        xl, yl = x[lo:hi].to(dev), y[lo:hi].to(dev)
        names = ("ssim", "gmsd", "psnr")
        got = ShardedMetrics(names)(xl, yl, n)
        ref = fa.metrics(x.to(dev), y.to(dev), names, reduction="none")
        q.put((rank, {k: float((got[k] - ref[k].double()).abs().max()) for k in names}))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_metrics_two_ranks_nccl():
    """Seven images over two NCCL ranks (uneven shards): every rank gathers
    per-image SSIM / GMSD / PSNR equal to one GPU scoring the whole batch."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ranks, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, diffs in out:
        for k, v in diffs.items():
            assert v < 1e-7, (rank, k, v)

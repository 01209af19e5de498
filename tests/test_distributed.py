"""Batch sharding and the per-image gather, as gloo ranks on CPU (world 2-3),
plus the failure path: a rank that dies before the gather makes the others'
collective end with an error instead of hanging."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from frame_analytics_b200.distributed import (batch_mean, exact_mse_from_ssd, gather_per_image,
                                              gather_stacked, shard_bounds)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_bounds_cover_the_batch():
    for n in range(0, 20):
        for world in range(1, 6):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _worker(rank, world, port, n, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=8))
        lo, hi = shard_bounds(n, rank, world)
        local = torch.arange(lo, hi, dtype=torch.float64) * 1.5 + 0.25
        if mode == "die" and rank == 1:
            raise SystemExit(3)  # leaves before the gather, with nothing in flight
        full = gather_per_image(local, n)
        if mode == "stacked":
            res = gather_stacked([local, -local, local * local], ("a", "b", "c"), n)
            q.put((rank, "ok", [res[k].tolist() for k in ("a", "b", "c")], None))
            dist.barrier()
            dist.destroy_process_group()
            return
        if mode == "ssd":
            # integer sums near 2^53 / n: the exact path must not round them
            ssd = (torch.arange(lo, hi, dtype=torch.int64) * 1_000_003 + (1 << 40))
            per, total = exact_mse_from_ssd(ssd, n, 6220800)
            q.put((rank, "ok", per.tolist(), total))
            dist.barrier()
            dist.destroy_process_group()
            return
        q.put((rank, "ok", full.tolist(), float(batch_mean(full))))
        dist.barrier()
        dist.destroy_process_group()
    except SystemExit:
        q.put((rank, "died", None, None))
    except Exception as exc:  # the survivors must see an error, not hang
        q.put((rank, "error", type(exc).__name__, None))


def _run(world, n, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, n, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


@pytest.mark.parametrize("world,n", [(2, 5), (3, 7), (2, 2)])
def test_gather_matches_single_process(world, n):
    out = _run(world, n, "ok")
    want = [i * 1.5 + 0.25 for i in range(n)]
    for rank, status, full, mean in out:
        assert status == "ok", out
        assert full == want
        assert abs(mean - sum(want) / n) < 1e-12


def test_dead_rank_fails_the_gather_instead_of_hanging():
    out = _run(2, 6, "die")
    assert out[1][1] == "died"
    assert out[0][1] == "error", out


@pytest.mark.parametrize("world,n", [(2, 5), (3, 8)])
def test_exact_mse_gathers_integer_sums(world, n):
    """Sharded integer MSE: the gathered int64 sums give the per-image MSE and
    the batch total exactly as one GPU forms them ((sum ssd) / (samples n))."""
    out = _run(world, n, "ssd")
    ssd = [i * 1_000_003 + (1 << 40) for i in range(n)]
    for rank, status, per, total in out:
        assert status == "ok", out
        assert per == [v / 6220800 for v in ssd]
        assert total == float(sum(ssd)) / float(6220800 * n)


@pytest.mark.parametrize("world,n", [(2, 5), (3, 7)])
def test_stacked_gather_moves_several_metrics_in_one_collective(world, n):
    out = _run(world, n, "stacked")
    want = [i * 1.5 + 0.25 for i in range(n)]
    for rank, status, (a, b, c), _ in out:
        assert status == "ok", out
        assert a == want and b == [-v for v in want] and c == [v * v for v in want]

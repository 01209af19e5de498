"""Batch sharding of the metrics over the GPUs of one node.

Images are independent, so the metric path shards by batch with no data
exchange: rank r scores images [lo, hi) of the batch on its own GPU, and the
per-image results (a few bytes each) are all-gathered so every rank holds the
whole batch's values.  The reference has no multi-device code; this is the
layer BASELINE.json's multi-GPU sweep needs.

One process per GPU, `torch.distributed` initialised by the caller (NCCL on
GPUs; the gather logic is backend-agnostic and is tested with gloo on CPU).
"""

from __future__ import annotations

from typing import Callable, Dict, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def shard_bounds(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) of an n-image batch owned by `rank`; the first
    n % world ranks hold one image more.  Every rank can compute every
    rank's bounds, so no sizes are exchanged."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_per_image(local: torch.Tensor, n: int, group=None) -> torch.Tensor:
    """All-gather per-image values (1-D, this rank's shard) into the full
    (n,) batch, in batch order, on every rank.  Uneven shards are padded to
    the largest shard for the collective and trimmed after it."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(n, rank, world)
    if local.ndim != 1 or local.numel() != hi - lo:
        raise ValueError(f"rank {rank} holds images [{lo}, {hi}) but passed {tuple(local.shape)}")
    width = max(shard_bounds(n, r, world)[1] - shard_bounds(n, r, world)[0] for r in range(world))
    buf = torch.zeros(width, dtype=local.dtype, device=local.device)
    buf[: local.numel()] = local
    out = torch.empty(world * width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    parts = []
    for r in range(world):
        a, b = shard_bounds(n, r, world)
        parts.append(out[r * width: r * width + (b - a)])
    return torch.cat(parts)


def batch_mean(per_image: torch.Tensor) -> torch.Tensor:
    """Mean over the gathered batch, summed in batch order on every rank
    (deterministic; equal to the single-GPU mean to ~1e-15 relative)."""
    return per_image.sum() / per_image.numel()


def exact_mse_from_ssd(ssd_local: torch.Tensor, n: int, samples_per_image: int,
                       group=None) -> Tuple[torch.Tensor, float]:
    """Batch MSE of integer frames from each rank's exact per-image sums of
    squared differences (int64, as the uint8 / uint16 kernels return them).
    The sums are gathered, not the float MSEs, so the per-image values and
    the batch total equal the single-GPU results bit for bit: the total is
    (sum of all sums) / (samples * n) in float64, as the kernel forms it."""
    if ssd_local.dtype != torch.int64:
        raise TypeError("exact MSE needs the int64 per-image sums")
    ssd = gather_per_image(ssd_local, n, group)
    # true float64 divisions, as the kernel's finaliser does them (a device
    # tensor divided by a scalar may become a multiplication by its reciprocal)
    sums = [int(v) for v in ssd.tolist()]
    per_image = torch.tensor([v / float(samples_per_image) for v in sums], dtype=torch.float64,
                             device=ssd.device)
    total = float(sum(sums)) / float(samples_per_image * n)
    return per_image, total


def sharded_mse(x_local: torch.Tensor, y_local: torch.Tensor, n: int,
                group=None) -> Tuple[torch.Tensor, float]:
    """Exact batch MSE of sharded integer (uint8 / uint16) frames: each rank's
    kernel returns its per-image sums, which are gathered."""
    from . import backend
    from .functional import _as_nchw
    x4, y4 = _as_nchw(x_local), _as_nchw(y_local)
    if x4.dtype not in (torch.uint8, torch.uint16):
        raise TypeError("sharded_mse is the exact path for uint8 / uint16 frames")
    _, ssd = backend.pixel(x4, y4, op=backend.OP_MSE, per_image=True, want_isum=True)
    return exact_mse_from_ssd(ssd, n, x4[0].numel(), group)


class ShardedMetrics:
    """Score a batch sharded over ranks and return whole-batch per-image results.

    ``metrics`` is either a mapping name -> callable ``f(x, y) -> (n_local,)``
    (e.g. ``lambda x, y: fa.ssim(x, y, reduction='none')``), one collective
    per name, or a sequence of metric names for
    :func:`frame_analytics_b200.metrics`: then the names are scored together
    (SSIM with GMSD / MSE / PSNR from one read of the shard, one launch) and
    their per-image values travel in ONE all-gather.  Each rank passes its own
    shard; the result holds every image's value on every rank.
    """

    def __init__(self, metrics, group=None, **kw):
        self.group = group
        self.kw = kw
        if isinstance(metrics, dict):
            self.metrics, self.names = dict(metrics), None
        else:
            self.metrics, self.names = None, tuple(metrics)

    def __call__(self, x_local: torch.Tensor, y_local: torch.Tensor, n: int) -> Dict[str, torch.Tensor]:
        if self.metrics is not None:
            return {name: gather_per_image(fn(x_local, y_local).reshape(-1), n, self.group)
                    for name, fn in self.metrics.items()}
        from .functional import metrics as _metrics
        res = _metrics(x_local, y_local, self.names, reduction="none", **self.kw)
        return gather_stacked([res[k].reshape(-1).to(torch.float64) for k in self.names],
                              self.names, n, self.group)


def gather_stacked(values: Sequence[torch.Tensor], names: Sequence[str], n: int,
                   group=None) -> Dict[str, torch.Tensor]:
    """All-gather several per-image float64 vectors of this rank's shard with
    one collective: they are stacked as (k, n_local) and gathered image-major,
    so the (n_local, k) rows travel together."""
    stacked = torch.stack(list(values), dim=1).contiguous()  # (n_local, k)
    k = stacked.shape[1]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(n, rank, world)
    if stacked.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds images [{lo}, {hi}) but scored {stacked.shape[0]}")
    width = max(shard_bounds(n, r, world)[1] - shard_bounds(n, r, world)[0] for r in range(world))
    buf = torch.zeros((width, k), dtype=stacked.dtype, device=stacked.device)
    buf[: hi - lo] = stacked
    out = torch.empty((world * width, k), dtype=stacked.dtype, device=stacked.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    rows = [out[r * width: r * width + (shard_bounds(n, r, world)[1] - shard_bounds(n, r, world)[0])]
            for r in range(world)]
    full = torch.cat(rows)
    return {name: full[:, i].contiguous() for i, name in enumerate(names)}


def default_metrics(names: Sequence[str] = ("ssim", "gmsd"), **kw) -> Dict[str, Callable]:
    """Per-image SSIM / GMSD / GMS / PSNR / MSE callables for ShardedMetrics."""
    from . import functional as F

    table = {"ssim": F.ssim, "gmsd": F.gmsd, "gms": F.gms, "psnr": F.psnr, "mse": F.mse,
             "ms_ssim": F.ms_ssim}
    return {n: (lambda f: (lambda x, y: f(x, y, reduction="none", **kw)))(table[n]) for n in names}

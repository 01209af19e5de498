"""``nn.Module`` wrappers with the reference's constructors and ``.loss``
conventions (frame_analytics/modules.py:42-241): SSIM/MSSSIM loss is
``1 - metric``, GMSD loss is ``1 - GMS``, pixel losses are their own loss."""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
from torch import nn

from . import backend
from .functional import (MS_SSIM_WEIGHTS, charbonnier, gms, gmsd, huber, l1, ms_ssim,
                         mse, psnr, ssim)

__all__ = ["MSE", "PSNR", "SSIM", "MSSSIM", "GMSD", "L1", "Charbonnier", "Huber",
           "StreamingMetrics"]


class MSE(nn.Module):
    def __init__(self, reduction: str = "mean", dtype: Optional[torch.dtype] = None,
                 out_dtype: torch.dtype = torch.float64, luma=None, crop_border: int = 0):
        super().__init__()
        self.reduction, self.dtype_, self.out_dtype = reduction, dtype, out_dtype
        self.luma, self.crop_border = luma, crop_border

    def forward(self, x, y):
        return mse(x, y, reduction=self.reduction, dtype=self.dtype_,
                   out_dtype=self.out_dtype, luma=self.luma, crop_border=self.crop_border)


class PSNR(nn.Module):
    """``PSNR(luma="matlab", crop_border=scale)`` is the super-resolution Y-PSNR."""

    def __init__(self, data_range: Optional[float] = None, reduction: str = "mean",
                 dtype: Optional[torch.dtype] = None, out_dtype: torch.dtype = torch.float64,
                 eps: float = 0.0, luma=None, crop_border: int = 0):
        super().__init__()
        self.data_range, self.reduction, self.dtype_ = data_range, reduction, dtype
        self.out_dtype, self.eps, self.luma, self.crop_border = out_dtype, eps, luma, crop_border

    def forward(self, x, y):
        return psnr(x, y, data_range=self.data_range, reduction=self.reduction,
                    dtype=self.dtype_, out_dtype=self.out_dtype, eps=self.eps,
                    luma=self.luma, crop_border=self.crop_border)


class SSIM(nn.Module):
    """SSIM; differentiable through the fused backward kernel."""

    def __init__(self, data_range: Optional[float] = None, win_size: int = 11,
                 sigma: float = 1.5, K: Sequence[float] = (0.01, 0.03),
                 reduction: str = "mean", return_map: bool = False,
                 dtype: Optional[torch.dtype] = None, downsample: bool = False,
                 luma=None, crop_border: int = 0):
        super().__init__()
        self.data_range, self.win_size, self.sigma, self.K = data_range, win_size, sigma, tuple(K)
        self.reduction, self.return_map, self.dtype_ = reduction, return_map, dtype
        self.downsample, self.luma, self.crop_border = downsample, luma, crop_border

    def forward(self, x, y):
        return ssim(x, y, data_range=self.data_range, win_size=self.win_size,
                    sigma=self.sigma, K=self.K, reduction=self.reduction,
                    return_map=self.return_map, dtype=self.dtype_,
                    downsample=self.downsample, luma=self.luma, crop_border=self.crop_border)

    def loss(self, x, y):
        """``1 - SSIM``, for use as a training objective."""
        return 1.0 - self.forward(x, y)


class MSSSIM(nn.Module):
    """Multi-scale SSIM; ``.loss()`` is ``1 - MS-SSIM``."""

    def __init__(self, data_range: Optional[float] = None, win_size: int = 11,
                 sigma: float = 1.5, K: Sequence[float] = (0.01, 0.03),
                 weights: Optional[Sequence[float]] = None, reduction: str = "mean",
                 dtype: Optional[torch.dtype] = None, luma=None, crop_border: int = 0):
        super().__init__()
        self.data_range, self.win_size, self.sigma, self.K = data_range, win_size, sigma, tuple(K)
        self.weights = tuple(weights) if weights is not None else MS_SSIM_WEIGHTS
        self.reduction, self.dtype_, self.luma, self.crop_border = reduction, dtype, luma, crop_border

    def forward(self, x, y):
        return ms_ssim(x, y, data_range=self.data_range, win_size=self.win_size,
                       sigma=self.sigma, K=self.K, weights=self.weights,
                       reduction=self.reduction, dtype=self.dtype_, luma=self.luma,
                       crop_border=self.crop_border)

    def loss(self, x, y):
        return 1.0 - self.forward(x, y)


class GMSD(nn.Module):
    """``forward`` is the deviation; ``.loss()`` is ``1 - mean(GMS)``."""

    def __init__(self, data_range: Optional[float] = None, T: Optional[float] = None,
                 eps: Optional[float] = None, downsample: bool = True,
                 reduction: str = "mean", dtype: Optional[torch.dtype] = None,
                 luma=None, crop_border: int = 0):
        super().__init__()
        self.data_range, self.T, self.eps, self.downsample = data_range, T, eps, downsample
        self.reduction, self.dtype_, self.luma, self.crop_border = reduction, dtype, luma, crop_border

    def _kwargs(self):
        return dict(data_range=self.data_range, T=self.T, eps=self.eps,
                    downsample=self.downsample, reduction=self.reduction,
                    dtype=self.dtype_, luma=self.luma, crop_border=self.crop_border)

    def forward(self, x, y):
        return gmsd(x, y, **self._kwargs())

    def loss(self, x, y):
        return 1.0 - gms(x, y, **self._kwargs())


class _PixelLoss(nn.Module):
    _fn = None

    def __init__(self, reduction: str = "mean", dtype: Optional[torch.dtype] = None,
                 out_dtype: torch.dtype = torch.float64, luma=None, crop_border: int = 0):
        super().__init__()
        self.reduction, self.dtype_, self.out_dtype = reduction, dtype, out_dtype
        self.luma, self.crop_border = luma, crop_border
        self.extra = {}

    def forward(self, x, y):
        return type(self)._fn(x, y, reduction=self.reduction, dtype=self.dtype_,
                              out_dtype=self.out_dtype, luma=self.luma,
                              crop_border=self.crop_border, **self.extra)

    def loss(self, x, y):
        return self.forward(x, y)


class L1(_PixelLoss):
    """Mean absolute error."""
    _fn = staticmethod(l1)


class Charbonnier(_PixelLoss):
    """Charbonnier penalty; ``eps`` is the width of the quadratic region."""
    _fn = staticmethod(charbonnier)

    def __init__(self, eps: float = 1e-3, **kwargs):
        super().__init__(**kwargs)
        self.extra = {"eps": float(eps)}


class Huber(_PixelLoss):
    """Huber loss, matching ``torch.nn.HuberLoss``."""
    _fn = staticmethod(huber)

    def __init__(self, delta: float = 1.0, **kwargs):
        super().__init__(**kwargs)
        self.extra = {"delta": float(delta)}


class _Slot:
    """One pair of device frames with its own staging, events and graph."""

    __slots__ = ("ref", "dist", "host", "uploaded", "scored", "graph", "out")

    def __init__(self, shape, dtype, device, pinned: bool):
        self.ref = torch.zeros(shape, dtype=dtype, device=device)
        self.dist = torch.zeros(shape, dtype=dtype, device=device)
        self.host = None
        if pinned:
            try:
                self.host = (torch.empty(shape, dtype=dtype, pin_memory=True),
                             torch.empty(shape, dtype=dtype, pin_memory=True))
            except RuntimeError:  # no pinned memory available: pageable copies
                self.host = None
        self.uploaded = torch.cuda.Event()
        self.scored = torch.cuda.Event()
        self.graph = None
        self.out = None


class StreamingMetrics:
    """Score a stream of frame pairs of one fixed shape (the reference's
    streaming scorer, modules.py:308-451).

    Two frame slots alternate.  Pair k is uploaded on a copy stream into slot
    k % 2 while pair k-1 may still be scored on the scoring stream, so with
    ``update(..., as_float=False)`` uploads overlap scoring.  Each slot has
    its own CUDA graph (one replay per pair when capture succeeds, eager calls
    otherwise), and the instance owns its kernel scratch
    (``backend.private_workspaces``): several instances may replay at the
    same time on different streams.

    ``metrics`` defaults to ``("mse", "psnr", "ssim")``, which
    :func:`frame_analytics_b200.metrics` computes in a single launch and one
    read of the pair.  The reference's ``lpips`` is outside this package and
    raises ``NotImplementedError``."""

    _KNOWN = ("mse", "psnr", "ssim", "ms_ssim", "gmsd", "gms", "l1", "charbonnier", "huber",
              "ssimulacra2")
    _ELSEWHERE = ("lpips",)

    def __init__(self, shape, device="cuda", dtype=torch.uint8,
                 data_range: Optional[float] = None, metrics=("mse", "psnr", "ssim"),
                 use_cuda_graph: bool = True, pinned_staging: bool = True):
        from .functional import _infer_data_range
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise TypeError("StreamingMetrics runs on a CUDA device")
        self.dtype = dtype
        self.shape = tuple(shape)
        self.metrics = tuple(metrics)
        elsewhere = [m for m in self.metrics if m in self._ELSEWHERE]
        if elsewhere:
            raise NotImplementedError(f"{elsewhere} are not part of frame_analytics_b200")
        unknown = [m for m in self.metrics if m not in self._KNOWN]
        if unknown:
            raise ValueError(f"unknown metric(s) {unknown}; expected any of {list(self._KNOWN)}")
        self._scratch: dict = {}
        self._copy = torch.cuda.Stream(device=self.device)
        self._work = torch.cuda.Stream(device=self.device)
        with torch.cuda.device(self.device):
            self._slots = [_Slot(self.shape, dtype, self.device, pinned_staging) for _ in range(2)]
        self._L = (float(data_range) if data_range is not None
                   else _infer_data_range(self._slots[0].ref))
        self._turn = 0
        self.capture_error: Optional[str] = None  # why graph capture was given up, if it was
        if use_cuda_graph and not all(self._record(s) for s in self._slots):
            for s in self._slots:  # all or nothing: graph replay is an optimisation
                s.graph = s.out = None

    # -- scoring ---------------------------------------------------------- #

    def _score(self, slot: _Slot) -> dict:
        from .functional import metrics as _metrics
        with backend.private_workspaces(self._scratch):
            return _metrics(slot.ref, slot.dist, self.metrics, data_range=self._L)

    def _record(self, slot: _Slot) -> bool:
        """Capture the slot's scoring into a graph on the scoring stream.  The
        eager passes first set the kernels' one-time attributes and allocate
        (zeroed) scratch outside the capture."""
        try:
            self._work.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self._work):
                self._score(slot)
                self._score(slot)
            self._work.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self._work):
                out = self._score(slot)
            slot.graph, slot.out = g, out
            return True
        except Exception as exc:
            slot.graph = slot.out = None
            self.capture_error = f"{type(exc).__name__}: {exc}"
            return False

    # -- staging ---------------------------------------------------------- #

    def _as_frame(self, src) -> torch.Tensor:
        t = src if torch.is_tensor(src) else torch.from_numpy(src)
        if tuple(t.shape) != self.shape:
            if t.numel() != math.prod(self.shape):
                raise ValueError(f"frame of shape {tuple(t.shape)} does not fit {self.shape}")
            t = t.reshape(self.shape)
        return t

    def _upload(self, dst: torch.Tensor, src, pinned: Optional[torch.Tensor]) -> None:
        """Enqueue src -> dst on the copy stream (the caller holds it current)."""
        t = self._as_frame(src)
        if t.is_cuda:
            dst.copy_(t, non_blocking=True)
            t.record_stream(self._copy)  # keep the source alive until the copy ran
        elif pinned is not None:
            pinned.copy_(t)  # host memcpy; the slot's previous upload has finished
            dst.copy_(pinned, non_blocking=True)
        else:
            dst.copy_(t)

    def update(self, ref, dist, *, as_float: bool = True):
        """Score one frame pair; returns a dict metric -> value (Python floats,
        or 0-d / per-image device tensors with ``as_float=False``)."""
        slot = self._slots[self._turn]
        self._turn ^= 1
        slot.scored.synchronize()  # this slot's previous pair is done with its buffers
        caller = torch.cuda.current_stream(self.device)
        self._copy.wait_stream(caller)  # device frames written on the caller's stream
        with torch.cuda.stream(self._copy):
            self._upload(slot.ref, ref, slot.host[0] if slot.host else None)
            self._upload(slot.dist, dist, slot.host[1] if slot.host else None)
            slot.uploaded.record(self._copy)
        self._work.wait_event(slot.uploaded)
        with torch.cuda.stream(self._work):
            if slot.graph is not None:
                slot.graph.replay()
                res = slot.out
            else:
                res = self._score(slot)
            if not as_float:
                res = {k: v.clone() for k, v in res.items()}
            slot.scored.record(self._work)
        if as_float:
            slot.scored.synchronize()
            return {k: float(v) for k, v in res.items()}
        caller.wait_stream(self._work)
        for v in res.values():
            v.record_stream(caller)
        return res

    @property
    def graph_captured(self) -> bool:
        return all(s.graph is not None for s in self._slots)

"""``nn.Module`` wrappers with the reference's constructors and ``.loss``
conventions (frame_analytics/modules.py:42-241): SSIM/MSSSIM loss is
``1 - metric``, GMSD loss is ``1 - GMS``, pixel losses are their own loss."""

from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import nn

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


class StreamingMetrics:
    """Score a stream of frame pairs of one fixed shape (modules.py:308-451 of
    the reference): the metrics are computed into static device buffers, by
    one CUDA-graph replay per pair when capture succeeds.

    ``metrics`` defaults to ``("mse", "psnr", "ssim")``, which
    :func:`frame_analytics_b200.metrics` computes in a single launch and one
    read of the pair.  Host frames are staged through pinned buffers.  The
    reference's ``lpips`` and ``ssimulacra2`` are outside this package and
    raise ``NotImplementedError``."""

    _KNOWN = ("mse", "psnr", "ssim", "ms_ssim", "gmsd", "gms", "l1", "charbonnier", "huber")
    _ELSEWHERE = ("lpips", "ssimulacra2")

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
        other = [m for m in self.metrics if m in self._ELSEWHERE]
        if other:
            raise NotImplementedError(f"{other} are not part of frame_analytics_b200")
        unknown = [m for m in self.metrics if m not in self._KNOWN]
        if unknown:
            raise ValueError(f"unknown metric(s) {unknown}; expected any of {list(self._KNOWN)}")
        self.ref = torch.zeros(self.shape, dtype=dtype, device=self.device)
        self.dist = torch.zeros(self.shape, dtype=dtype, device=self.device)
        self._L = float(data_range) if data_range is not None else _infer_data_range(self.ref)
        self._host = None
        if pinned_staging:
            self._host = (torch.empty(self.shape, dtype=dtype, pin_memory=True),
                          torch.empty(self.shape, dtype=dtype, pin_memory=True))
        self._graph = None
        self._static_out = None
        if use_cuda_graph:
            self._try_capture()

    def _compute(self):
        from .functional import metrics as _metrics
        return _metrics(self.ref, self.dist, self.metrics, data_range=self._L)

    def _try_capture(self):
        try:
            side = torch.cuda.Stream(device=self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                for _ in range(3):  # kernels' one-time attributes, workspaces
                    self._compute()
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._static_out = self._compute()
            self._graph = g
        except Exception:  # capture is an optimisation: fall back to eager calls
            self._graph = None
            self._static_out = None

    def _stage(self, buf: torch.Tensor, src, slot: int) -> None:
        if not torch.is_tensor(src):
            src = torch.from_numpy(src)
        if tuple(src.shape) != self.shape:
            src = src.reshape(self.shape)
        if src.is_cuda:
            buf.copy_(src, non_blocking=True)
        elif self._host is not None:
            self._host[slot].copy_(src)
            buf.copy_(self._host[slot], non_blocking=True)
        else:
            buf.copy_(src)

    def update(self, ref, dist, *, as_float: bool = True):
        """Score one frame pair; returns a dict metric -> value."""
        self._stage(self.ref, ref, 0)
        self._stage(self.dist, dist, 1)
        if self._graph is not None:
            self._graph.replay()
            out = self._static_out
        else:
            out = self._compute()
        if as_float:
            return {k: float(v) for k, v in out.items()}
        return {k: v.clone() for k, v in out.items()}

    @property
    def graph_captured(self) -> bool:
        return self._graph is not None

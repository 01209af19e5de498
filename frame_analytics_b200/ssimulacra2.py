"""SSIMULACRA 2 (Sneyers 2022/2023), the reference's ``fa.ssimulacra2``
(frame_analytics/ssimulacra2.py), computed by the sm_100a kernels of
``csrc/ssimulacra2.cu``.

Higher is better; 100 is a pixel-identical pair.  Inputs are sRGB-encoded RGB
(``(3, H, W)`` or ``(N, 3, H, W)``, a 1-channel image is replicated to three,
at least 8 x 8); the metric is not symmetric: the first argument is the
original.  ``dtype=torch.float64`` computes colour, blur and maps in double
(float32 by default, as upstream and the reference do); the sums and the
final weighting are double either way.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import nn

from . import backend
from .functional import _prep

__all__ = ["ssimulacra2", "SSIMULACRA2", "SSIMULACRA2_WEIGHTS"]

# Msssim::Score weights (libjxl tools/ssimulacra2.cc): for each channel, for
# each scale, for each norm (mean, 4-norm): SSIM', ringing, blurring.  A
# published constant of the metric.
SSIMULACRA2_WEIGHTS = (
    0.0, 0.0007376606707406586, 0.0, 0.0, 0.0007793481682867309, 0.0,
    0.0, 0.0004371155730107379, 0.0, 1.1041726426657346, 0.00066284834129271, 0.00015231632783718752,
    0.0, 0.0016406437456599754, 0.0, 1.8422455520539298, 11.441172603757666, 0.0,
    0.0007989109436015163, 0.000176816438078653, 0.0, 1.8787594979546387, 10.94906990605142, 0.0,
    0.0007289346991508072, 0.9677937080626833, 0.0, 0.00014003424285435884, 0.9981766977854967, 0.00031949755934435053,
    0.0004550992113792063, 0.0, 0.0, 0.0013648766163243398, 0.0, 0.0,
    0.0, 0.0, 0.0, 7.466890328078848, 0.0, 17.445833984131262,
    0.0006235601634041466, 0.0, 0.0, 6.683678146179332, 0.00037724407979611296, 1.027889937768264,
    225.20515300849274, 0.0, 0.0, 19.213238186143016, 0.0011401524586618361, 0.001237755635509985,
    176.39317598450694, 0.0, 0.0, 24.43300999870476, 0.28520802612117757, 0.0004485436923833408,
    0.0, 0.0, 0.0, 34.77906344483772, 44.835625328877896, 0.0,
    0.0, 0.0, 0.0, 0.0, 0.0, 0.0,
    0.0, 0.0008680556573291698, 0.0, 0.0, 0.0, 0.0,
    0.0, 0.0005313191874358747, 0.0, 0.00016533814161379112, 0.0, 0.0,
    0.0, 0.0, 0.0, 0.0004179171803251336, 0.0017290828234722833, 0.0,
    0.0020827005846636437, 0.0, 0.0, 8.826982764996862, 23.19243343998926, 0.0,
    95.1080498811086, 0.9863978034400682, 0.9834382792465353, 0.0012286405048278493, 171.2667255897307, 0.9807858872435379,
    0.0, 0.0, 0.0, 0.0005130064588990679, 0.0, 0.00010854057858411537,)
assert len(SSIMULACRA2_WEIGHTS) == 108
_W = (ctypes.c_double * 108)(*SSIMULACRA2_WEIGHTS)


def ssimulacra2(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
                reduction: str = "mean", dtype: Optional[torch.dtype] = None,
                crop_border: int = 0) -> torch.Tensor:
    """SSIMULACRA 2 score per image (``reduction='none'``, float64 ``(N,)``)
    or its batch mean (the reference's signature, ssimulacra2.py:465-500)."""
    if reduction not in ("mean", "none"):
        raise ValueError(f"reduction must be 'mean' or 'none', got {reduction!r}")
    x4, y4, L, _ = _prep(x, y, None, crop_border, data_range)
    backend.require_cuda(x4)
    if dtype is not None and dtype not in (torch.float32, torch.float64):
        raise ValueError(f"SSIMULACRA 2 computes in float32 or float64, not {dtype}")
    f64 = dtype == torch.float64 or (dtype is None and x4.dtype == torch.float64)
    c = x4.shape[1]
    if c == 1:  # a gray plane replicated to RGB: a zero channel stride, no copy
        x4, y4 = x4.expand(-1, 3, -1, -1), y4.expand(-1, 3, -1, -1)
    elif c != 3:
        raise ValueError(f"SSIMULACRA 2 needs 1- or 3-channel RGB, got {c} channels")
    if min(x4.shape[-2:]) < 8:
        raise ValueError(f"SSIMULACRA 2 needs at least 8x8, got {tuple(x4.shape[-2:])}")
    return backend.ssimulacra2(x4.detach(), y4.detach(), data_range=L, f64=f64,
                               weights=_W, per_image=(reduction == "none"))


class SSIMULACRA2(nn.Module):
    """Module form of :func:`ssimulacra2` (higher is better)."""

    def __init__(self, data_range: Optional[float] = None, reduction: str = "mean",
                 dtype: Optional[torch.dtype] = None, crop_border: int = 0):
        super().__init__()
        self.data_range, self.reduction = data_range, reduction
        self.dtype_, self.crop_border = dtype, crop_border

    def forward(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        return ssimulacra2(x, y, data_range=self.data_range, reduction=self.reduction,
                           dtype=self.dtype_, crop_border=self.crop_border)

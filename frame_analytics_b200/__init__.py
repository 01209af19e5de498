"""frame_analytics_b200 -- full-reference image metrics on B200 (sm_100a).

A drop-in for the metric path of frame_analytics: ``psnr``, ``mse``, ``l1``,
``charbonnier``, ``huber``, ``ssim`` (forward and fused backward),
``ms_ssim``, ``gmsd`` / ``gms``, ``ssimulacra2``, with the same arguments and results,
computed by hand-written CUDA kernels behind a C ABI (``include/fa_b200.h``).

>>> import torch, frame_analytics_b200 as fa
>>> a = torch.randint(0, 256, (8, 3, 1080, 1920), dtype=torch.uint8, device="cuda")
>>> b = (a.float() + 4 * torch.randn(a.shape, device="cuda")).clamp(0, 255).byte()
>>> fa.psnr(a, b), fa.ssim(a, b)
"""

from .functional import (  # noqa: F401
    LUMA_COEFFS,
    MS_SSIM_WEIGHTS,
    charbonnier,
    gaussian_window_1d,
    gms,
    gmsd,
    huber,
    l1,
    ms_ssim,
    mse,
    psnr,
    rgb_to_luma,
    set_compile_enabled,
    metrics,
    set_fused_loss_grad,
    ssim,
)
from . import planes  # noqa: F401
from .ssimulacra2 import SSIMULACRA2, ssimulacra2  # noqa: F401
from .modules import (GMSD, L1, MSE, MSSSIM, PSNR, SSIM, Charbonnier, Huber,  # noqa: F401
                      StreamingMetrics)

__version__ = "0.1.0"

__all__ = [
    "mse", "psnr", "ssim", "ms_ssim", "gmsd", "gms", "l1", "charbonnier", "huber",
    "rgb_to_luma", "gaussian_window_1d", "set_compile_enabled",
    "set_fused_loss_grad", "metrics", "StreamingMetrics",
    "MSE", "PSNR", "SSIM", "MSSSIM", "GMSD", "L1", "Charbonnier", "Huber",
    "ssimulacra2", "SSIMULACRA2", "backend_status",
]


def backend_status() -> dict:
    """Where the kernels come from (frame_analytics/__init__.py:91-95)."""
    from . import backend

    return backend.status()

"""Public metric functions: the drop-in surface of frame_analytics.functional.

Same names, arguments, defaults, shapes and error behaviour as the reference
(frame_analytics/functional.py), computed by the sm_100a kernels of
libfa_b200.so.  Luma projection and border cropping are folded into the kernel
loads; there is no portable/torch path, so a call the kernels cannot serve
raises instead of falling back.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import backend

__all__ = [
    "mse", "psnr", "ssim", "ms_ssim", "gmsd", "gms", "l1", "charbonnier",
    "huber", "rgb_to_luma", "gaussian_window_1d", "set_compile_enabled",
    "set_fused_loss_grad", "metrics",
    "MS_SSIM_WEIGHTS", "LUMA_COEFFS",
]

# Wang et al. 2003, table 1 (functional.py:697 in the reference).
MS_SSIM_WEIGHTS = (0.0448, 0.2856, 0.3001, 0.2363, 0.1333)

# (r, g, b, offset as a fraction of the data range) -- functional.py:193-197.
LUMA_COEFFS = {
    "bt601": (0.299, 0.587, 0.114, 0.0),
    "bt709": (0.2126, 0.7152, 0.0722, 0.0),
    "matlab": (65.481 / 255.0, 128.553 / 255.0, 24.966 / 255.0, 16.0 / 255.0),
}


def set_compile_enabled(flag: bool) -> None:
    """Accepted for drop-in compatibility (functional.py:55-59); the kernels
    here are compiled ahead of time, so there is nothing to switch."""


# --------------------------------------------------------------------------- #
# input handling (functional.py:141-271)
# --------------------------------------------------------------------------- #

# Peak value of integer sample types; every floating type is taken as [0, 1].
_INT_PEAK = {torch.uint8: 255.0, torch.int16: 65535.0, torch.int32: 65535.0}
if getattr(torch, "uint16", None) is not None:
    _INT_PEAK[torch.uint16] = 65535.0


def _infer_data_range(t: torch.Tensor) -> float:
    return _INT_PEAK.get(t.dtype, 1.0)


def _as_nchw(t: torch.Tensor) -> torch.Tensor:
    """(H,W) / (C,H,W) / (N,C,H,W) as a 4-D view with leading unit axes."""
    if not 2 <= t.ndim <= 4:
        raise ValueError(f"images must have 2, 3 or 4 dimensions (H,W / C,H,W / "
                         f"N,C,H,W); this one has shape {tuple(t.shape)}")
    return t.view((1,) * (4 - t.ndim) + tuple(t.shape)) if t.ndim < 4 else t


def _check_pair(x: torch.Tensor, y: torch.Tensor):
    for what, u, v in (("shape", tuple(x.shape), tuple(y.shape)),
                       ("device", x.device, y.device)):
        if u != v:
            raise ValueError(f"the two images differ in {what}: {u} and {v}")
    return _as_nchw(x), _as_nchw(y)


def _resolve_luma(luma) -> Optional[str]:
    """None/False -> no projection, True -> bt601, a name -> that convention."""
    if isinstance(luma, bool) or luma is None:
        return "bt601" if luma else None
    if not isinstance(luma, str):
        raise TypeError(f"luma is None, a bool or a convention name, "
                        f"not {type(luma).__name__}")
    if luma in LUMA_COEFFS:
        return luma
    raise ValueError(f"luma convention {luma!r} is not one of {sorted(LUMA_COEFFS)}")


def _crop_border(t: torch.Tensor, b: int) -> torch.Tensor:
    """Drop `b` pixels on every side, as a view (the kernels take strides)."""
    if b < 0:
        raise ValueError(f"crop_border cannot be negative ({b})")
    if b == 0:
        return t
    h, w = t.shape[-2:]
    if min(h, w) <= 2 * b:
        raise ValueError(f"crop_border={b} leaves nothing of a {h}x{w} image")
    return t.narrow(-2, b, h - 2 * b).narrow(-1, b, w - 2 * b)


def _prep(x, y, luma, crop_border, data_range):
    """Validate a pair and return (x4, y4, L, luma mode): 4-D views with the
    border already cropped; L is `data_range` or the dtype's peak."""
    x4, y4 = _check_pair(x, y)
    mode = _resolve_luma(luma)
    if mode is not None and x4.shape[1] != 3:
        raise ValueError(f"a luma projection needs RGB input (3 channels), "
                         f"not {x4.shape[1]}")
    L = _infer_data_range(x4) if data_range is None else float(data_range)
    return _crop_border(x4, crop_border), _crop_border(y4, crop_border), L, mode


def _luma_k(mode: Optional[str], L: float):
    """Luma coefficients in the metric's units: (cr, cg, cb, offset * L)."""
    if mode is None:
        return None
    cr, cg, cb, off = LUMA_COEFFS[mode]
    return (cr, cg, cb, off * L)


def _check_reduction(reduction: str) -> None:
    if reduction not in ("mean", "none"):
        raise ValueError(f"reduction must be 'mean' or 'none', got {reduction!r}")


def _check_hint(backend_hint: str) -> None:
    if backend_hint not in ("auto", "native", "torch"):
        raise ValueError(f"backend_hint must be 'auto', 'native' or 'torch', got {backend_hint!r}")
    if backend_hint == "torch":
        raise NotImplementedError(
            "frame_analytics_b200 has no portable torch path; every metric runs on the "
            "sm_100a kernels (backend_hint='auto' or 'native')")


def _grad_wanted(*ts: torch.Tensor) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in ts)


def rgb_to_luma(t: torch.Tensor, mode: str = "bt601", *,
                data_range: Optional[float] = None,
                dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``(N,3,H,W)`` RGB -> ``(N,1,H,W)`` luma (functional.py:213-237).

    The metric functions never call this: their kernels apply the same
    projection while loading.  It is kept for callers that want the plane."""
    t4 = _as_nchw(t)
    if t4.shape[1] != 3:
        raise ValueError(f"luma needs a 3-channel image, got {t4.shape[1]} channels")
    m = _resolve_luma(mode)
    if m is None:
        raise ValueError("rgb_to_luma needs a luma convention, not None/False")
    cr, cg, cb, off = LUMA_COEFFS[m]
    L = float(data_range) if data_range is not None else _infer_data_range(t4)
    wdt = dtype if dtype is not None else (torch.float64 if t4.dtype == torch.float64
                                           else torch.float32)
    v = t4.to(wdt)
    out = cr * v[:, 0:1] + cg * v[:, 1:2] + cb * v[:, 2:3]
    if off:
        out = out + off * L
    return out


# --------------------------------------------------------------------------- #
# pixel reductions with autograd
# --------------------------------------------------------------------------- #

class _PixelLoss(torch.autograd.Function):
    """Differentiable pixel reduction: forward by the fused kernel, backward by
    the elementwise derivative of the penalty (nothing is saved but x, y)."""

    @staticmethod
    def forward(ctx, x, y, op, param, per_image, luma):
        out = backend.pixel(x, y, op=op, param=param, per_image=per_image, luma=luma)
        ctx.save_for_backward(x, y)
        ctx.op, ctx.param, ctx.per_image, ctx.luma = op, param, per_image, luma
        return out

    @staticmethod
    def backward(ctx, g):
        _reject_double_backward()
        x, y = ctx.saved_tensors
        dx, dy = backend.pixel_backward(x, y, g, op=ctx.op, param=ctx.param,
                                        per_image=ctx.per_image, luma=ctx.luma,
                                        need_dx=ctx.needs_input_grad[0],
                                        need_dy=ctx.needs_input_grad[1])
        return dx, dy, None, None, None, None


class _PixelLossGrad(torch.autograd.Function):
    """A pixel loss computed together with its gradient (one read of x and y;
    contiguous float32, no luma).  The kernel returns the gradient for an
    upstream gradient of 1, the one ``loss = fa.mse(...)`` sends; backward
    rescales that buffer in place (a factor of exactly 1 costs nothing).  A
    second backward through the same graph recomputes from the saved inputs."""

    @staticmethod
    def forward(ctx, x, y, op, param, per_image):
        out, dx, dy = backend.pixel_loss_grad(x, y, op=op, param=param, per_image=per_image,
                                              need_dx=x.requires_grad, need_dy=y.requires_grad)
        ctx.save_for_backward(x, y)
        ctx.grads = (dx, dy)
        ctx.op, ctx.param, ctx.per_image = op, param, per_image
        return out

    @staticmethod
    def backward(ctx, g):
        _reject_double_backward()
        nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if ctx.grads is not None:
            dx, dy = ctx.grads
            ctx.grads = None  # handed to autograd below

            def scaled(u):
                return backend.grad_scale(u, g, per_image=ctx.per_image, inplace=True)

            return (scaled(dx) if (nx and dx is not None) else None,
                    scaled(dy) if (ny and dy is not None) else None, None, None, None)
        x, y = ctx.saved_tensors
        dx, dy = backend.pixel_backward(x, y, g, op=ctx.op, param=ctx.param,
                                        per_image=ctx.per_image, need_dx=nx, need_dy=ny)
        return dx, dy, None, None, None


def _pixel(x4, y4, op, param, per_image, luma_k, psnr_bias=backend.PSNR_NONE):
    backend.require_cuda(x4)
    if _grad_wanted(x4, y4):
        if (_fused_loss_grad and psnr_bias == backend.PSNR_NONE and luma_k is None
                and x4.dtype == torch.float32 and y4.dtype == torch.float32
                and x4.is_contiguous() and y4.is_contiguous()):
            return _PixelLossGrad.apply(x4, y4, op, param, per_image)
        if psnr_bias != backend.PSNR_NONE:
            m = _PixelLoss.apply(x4, y4, op, param, per_image, luma_k)
            return psnr_bias - 10.0 * torch.log10(m)
        return _PixelLoss.apply(x4, y4, op, param, per_image, luma_k)
    return backend.pixel(x4.detach(), y4.detach(), op=op, param=param,
                         per_image=per_image, psnr_bias=psnr_bias, luma=luma_k)


def mse(x: torch.Tensor, y: torch.Tensor, *, reduction: str = "mean",
        dtype: Optional[torch.dtype] = None, out_dtype: torch.dtype = torch.float64,
        luma=None, crop_border: int = 0) -> torch.Tensor:
    """Mean squared error (functional.py:289-343).  uint8 input is summed in
    64-bit integers on the device, so the result is exact."""
    x4, y4, L, mode = _prep(x, y, luma, crop_border, None)
    _check_reduction(reduction)
    out = _pixel(x4, y4, backend.OP_MSE, 0.0, reduction == "none", _luma_k(mode, L))
    return out.to(out_dtype)


def psnr(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
         reduction: str = "mean", dtype: Optional[torch.dtype] = None,
         out_dtype: torch.dtype = torch.float64, eps: float = 0.0, luma=None,
         crop_border: int = 0) -> torch.Tensor:
    """PSNR in dB (functional.py:345-387); +inf for identical inputs unless
    ``eps`` clamps the MSE.  The dB conversion happens inside the kernel."""
    _check_reduction(reduction)
    x4, y4, L, mode = _prep(x, y, luma, crop_border, data_range)
    bias = math.log10(L * L) * 10.0
    if not eps:
        return _pixel(x4, y4, backend.OP_MSE, 0.0, reduction == "none",
                      _luma_k(mode, L), psnr_bias=bias).to(out_dtype)
    m = _pixel(x4, y4, backend.OP_MSE, 0.0, reduction == "none", _luma_k(mode, L))
    m = m.clamp_min(eps)
    return (bias - 10.0 * torch.log10(m)).to(out_dtype)


def _pixel_loss(op, x, y, param, reduction, out_dtype, luma, crop_border, backend_hint):
    _check_reduction(reduction)
    _check_hint(backend_hint)
    x4, y4, L, mode = _prep(x, y, luma, crop_border, None)
    return _pixel(x4, y4, op, param, reduction == "none", _luma_k(mode, L)).to(out_dtype)


def l1(x: torch.Tensor, y: torch.Tensor, *, reduction: str = "mean",
       dtype: Optional[torch.dtype] = None, out_dtype: torch.dtype = torch.float64,
       luma=None, crop_border: int = 0, backend_hint: str = "auto") -> torch.Tensor:
    """Mean absolute error (functional.py:1157-1170)."""
    return _pixel_loss(backend.OP_L1, x, y, 0.0, reduction, out_dtype, luma,
                       crop_border, backend_hint)


def charbonnier(x: torch.Tensor, y: torch.Tensor, *, eps: float = 1e-3,
                reduction: str = "mean", dtype: Optional[torch.dtype] = None,
                out_dtype: torch.dtype = torch.float64, luma=None, crop_border: int = 0,
                backend_hint: str = "auto") -> torch.Tensor:
    """``mean sqrt((x-y)^2 + eps^2)`` (functional.py:1173-1191)."""
    return _pixel_loss(backend.OP_CHARB, x, y, float(eps) ** 2, reduction, out_dtype,
                       luma, crop_border, backend_hint)


def huber(x: torch.Tensor, y: torch.Tensor, *, delta: float = 1.0,
          reduction: str = "mean", dtype: Optional[torch.dtype] = None,
          out_dtype: torch.dtype = torch.float64, luma=None, crop_border: int = 0,
          backend_hint: str = "auto") -> torch.Tensor:
    """Huber loss matching ``torch.nn.HuberLoss`` (functional.py:1194-1210)."""
    if delta <= 0:
        raise ValueError(f"delta must be > 0, got {delta}")
    return _pixel_loss(backend.OP_HUBER, x, y, float(delta), reduction, out_dtype,
                       luma, crop_border, backend_hint)


# --------------------------------------------------------------------------- #
# SSIM
# --------------------------------------------------------------------------- #

_window_cache: dict = {}


def gaussian_window_1d(win_size: int = 11, sigma: float = 1.5, *, device=None,
                       dtype=torch.float32) -> torch.Tensor:
    """The separable SSIM window (functional.py:397-420 of the reference): a
    1-D Gaussian normalised to sum 1; the 2-D window is its outer product.
    One tensor per (size, sigma, device, dtype) is kept."""
    key = (win_size, float(sigma), str(device), dtype)
    if key not in _window_cache:
        _window_cache[key] = torch.tensor(backend.gaussian_taps(int(win_size), float(sigma)),
                                          dtype=torch.float64).to(device=device, dtype=dtype)
    return _window_cache[key]


def _reject_double_backward() -> None:
    """Refuse ``create_graph=True`` through a fused kernel (functional.py:496-518)."""
    if torch.is_grad_enabled():
        raise RuntimeError(
            "frame_analytics_b200's fused backward kernels are not twice "
            "differentiable, so create_graph=True (gradient penalties, "
            "Hessian-vector products, torch.func.hessian) cannot use them.")


def _kernel_window(win_size: int, sigma: float, device) -> "backend.Taps":
    if win_size not in backend.KERNEL_WINDOWS:
        raise ValueError(f"win_size must be one of {backend.KERNEL_WINDOWS}, got {win_size}")
    return backend.host_taps(win_size, sigma)


class _FusedSSIM(torch.autograd.Function):
    """Differentiable SSIM (functional.py:521-572).  Forward: the fused
    kernel.  Backward: one fused kernel that recomputes the moments; only x,
    y and the window are saved.

    ``mode``: "mean" (batch mean scalar), "none" (per image) or "map"."""

    @staticmethod
    def forward(ctx, x, y, win, shift, C1, C2, mode):
        res = backend.ssim_forward(x, y, win, shift=shift, C1=C1, C2=C2,
                                   want_map=(mode == "map"),
                                   want_per_image=(mode == "none"),
                                   want_total=(mode == "mean"))
        ctx.save_for_backward(x, y)
        ctx.win = win
        ctx.consts = (shift, C1, C2)
        ctx.mode = mode
        if mode == "map":
            return res["map"]
        return res["per_image"] if mode == "none" else res["total"]

    @staticmethod
    def backward(ctx, g):
        _reject_double_backward()
        x, y = ctx.saved_tensors
        win = ctx.win
        shift, C1, C2 = ctx.consts
        nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (nx or ny):
            return (None,) * 7
        kw = dict(shift=shift, C1=C1, C2=C2, need_dx=nx, need_dy=ny)
        if ctx.mode == "map":
            dx, dy = backend.ssim_backward(x, y, win, dmap=g, **kw)
        elif ctx.mode == "mean":
            # the scalar upstream gradient stays on the device: no host sync
            dx, dy = backend.ssim_backward(x, y, win, gscalar=g, **kw)
        else:
            n, c = x.shape[0], x.shape[1]
            gdt = torch.float64 if x.dtype == torch.float64 else torch.float32
            gs = (g.to(gdt) / c).repeat_interleave(c)
            dx, dy = backend.ssim_backward(x, y, win, gs=gs, gcs=torch.zeros_like(gs), **kw)
        return (dx.to(x.dtype) if nx else None, dy.to(y.dtype) if ny else None,
                None, None, None, None, None)


class _SSIMLossGrad(torch.autograd.Function):
    """Differentiable scalar / per-image SSIM computed together with its
    gradient (one launch, no separate forward).  The kernel returns the
    gradient of the batch-mean SSIM for an upstream gradient of -1, the one a
    loss ``1 - ssim`` sends; backward rescales that buffer in place by the
    real upstream gradient (by ``-g`` for the batch mean, by ``-g[n] * N``
    per image for ``reduction='none'``), which for ``1 - ssim`` is a factor
    of exactly 1 and costs nothing.  The buffer becomes the input's gradient,
    so a second backward through the same graph (``retain_graph``) recomputes
    from the saved inputs.  The gradient is computed even if backward is
    never called: :func:`set_fused_loss_grad` turns this off for callers that
    evaluate with gradients enabled but rarely backpropagate."""

    @staticmethod
    def forward(ctx, x, y, win, shift, C1, C2, mode, nx, ny):
        total, per_image, dx, dy = backend.ssim_loss_grad(
            x, y, win, shift=shift, C1=C1, C2=C2, need_dx=nx, need_dy=ny,
            want_per_image=(mode == "none"), upstream=-1.0)
        ctx.save_for_backward(x, y)
        ctx.grads = (dx, dy)
        ctx.win = win
        ctx.consts = (shift, C1, C2)
        ctx.mode, ctx.n = mode, x.shape[0]
        return per_image if mode == "none" else total

    @staticmethod
    def backward(ctx, g):
        _reject_double_backward()
        nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        per_image = ctx.mode == "none"
        if ctx.grads is not None:
            dx, dy = ctx.grads
            ctx.grads = None  # handed to autograd below
            mult = -float(ctx.n) if per_image else -1.0

            def scaled(u):
                return backend.grad_scale(u, g, per_image=per_image, mult=mult, inplace=True)

            return (scaled(dx) if (nx and dx is not None) else None,
                    scaled(dy) if (ny and dy is not None) else None,
                    None, None, None, None, None, None, None)
        # a second backward through the same graph: recompute
        x, y = ctx.saved_tensors
        shift, C1, C2 = ctx.consts
        kw = dict(shift=shift, C1=C1, C2=C2, need_dx=nx, need_dy=ny)
        if per_image:
            c = x.shape[1]
            gs = (g.to(torch.float32) / c).repeat_interleave(c)
            dx, dy = backend.ssim_backward(x, y, ctx.win, gs=gs, gcs=torch.zeros_like(gs), **kw)
        else:
            dx, dy = backend.ssim_backward(x, y, ctx.win, gscalar=g, **kw)
        return (dx if nx else None, dy if ny else None, None, None, None, None, None, None, None)


_fused_loss_grad = True


def set_fused_loss_grad(enabled: bool) -> None:
    """Compute the SSIM gradient, and that of a float32 pixel loss, in the
    same pass as the value whenever an input requires grad (default on).  Off: the forward computes the value
    only and the backward recomputes the moments."""
    global _fused_loss_grad
    _fused_loss_grad = bool(enabled)


class _BoxDownFn(torch.autograd.Function):
    """MATLAB ssim.m's automatic downsample (functional.py:575-586): f x f box
    mean with replicated borders, every f-th sample; forward and adjoint are
    one kernel each."""

    @staticmethod
    def forward(ctx, x, f):
        ctx.shape, ctx.dtype, ctx.f = tuple(x.shape), x.dtype, f
        return backend.box_downsample(x, f)

    @staticmethod
    def backward(ctx, g):
        return backend.box_downsample_backward(g, ctx.shape, ctx.f).to(ctx.dtype), None


def _matlab_downsample(x: torch.Tensor, f: int, luma=None) -> torch.Tensor:
    """The automatic downsample MATLAB's ssim.m applies to large images, to
    float32; ``luma`` projects RGB inside the same kernel (no gradient)."""
    if f <= 1:
        return x
    if luma is not None or not (torch.is_grad_enabled() and x.requires_grad):
        return backend.box_downsample(x.detach(), f, luma=luma)
    return _BoxDownFn.apply(x, f)


def ssim(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
         win_size: int = 11, sigma: float = 1.5, K: Sequence[float] = (0.01, 0.03),
         reduction: str = "mean", return_map: bool = False,
         dtype: Optional[torch.dtype] = None, downsample: bool = False,
         backend_hint: str = "auto", luma=None, crop_border: int = 0) -> torch.Tensor:
    """Structural similarity (functional.py:589-689): 11x11 Gaussian, sigma
    1.5, K = (0.01, 0.03), valid support.  ``reduction`` 'mean' -> scalar,
    'none' -> (N,); ``return_map`` -> (N, C, H-10, W-10) float32."""
    _check_reduction(reduction)
    _check_hint(backend_hint)
    x4, y4, L, mode = _prep(x, y, luma, crop_border, data_range)
    backend.require_cuda(x4)
    K1, K2 = float(K[0]), float(K[1])
    C1, C2 = (K1 * L) ** 2, (K2 * L) ** 2
    shift = 0.5 * L
    lk = _luma_k(mode, L)
    grad = _grad_wanted(x4, y4)

    if downsample:
        f = max(1, int(round(min(x4.shape[-2], x4.shape[-1]) / 256.0)))
        if lk is not None and (grad or f == 1):
            x4, y4 = rgb_to_luma(x4, mode, data_range=L), rgb_to_luma(y4, mode, data_range=L)
            lk = None
        if f > 1:
            # luma (when still pending) is projected inside the downsample kernel
            x4 = _matlab_downsample(x4, f, luma=lk)
            y4 = _matlab_downsample(y4, f, luma=lk)
            lk = None

    if x4.shape[-2] < win_size or x4.shape[-1] < win_size:
        raise ValueError(f"image {tuple(x4.shape[-2:])} smaller than window {win_size}x{win_size}")
    win = _kernel_window(win_size, sigma, x4.device)

    if grad:
        # the fused backward reads float32 planes (float64 frames: float64
        # planes and the float64 kernels): luma/crop/cast are applied with
        # differentiable torch ops first
        if lk is not None:
            x4, y4 = rgb_to_luma(x4, mode, data_range=L), rgb_to_luma(y4, mode, data_range=L)
        cdt = torch.float64 if x4.dtype == torch.float64 else torch.float32
        xf = x4 if x4.dtype == cdt else x4.to(cdt)
        yf = y4 if y4.dtype == cdt else y4.to(cdt)
        m = "map" if return_map else reduction
        if _fused_loss_grad and m != "map" and cdt == torch.float32:
            return _SSIMLossGrad.apply(xf.contiguous(), yf.contiguous(), win, shift, C1, C2, m,
                                       xf.requires_grad, yf.requires_grad)
        return _FusedSSIM.apply(xf.contiguous(), yf.contiguous(), win, shift, C1, C2, m)

    x4, y4 = x4.detach(), y4.detach()
    res = backend.ssim_forward(x4, y4, win, shift=shift, C1=C1, C2=C2, luma=lk,
                               want_map=return_map,
                               want_per_image=(not return_map and reduction == "none"),
                               want_total=(not return_map and reduction == "mean"))
    if return_map:
        out = res["map"]
        if x4.dtype == torch.float64 or dtype == torch.float64:
            out = out.to(torch.float64)
        return out
    return res["per_image"] if reduction == "none" else res["total"]


# --------------------------------------------------------------------------- #
# several metrics of one frame pair
# --------------------------------------------------------------------------- #

METRIC_NAMES = ("mse", "psnr", "ssim", "ms_ssim", "gmsd", "gms", "l1", "charbonnier", "huber",
                "ssimulacra2")


def metrics(x: torch.Tensor, y: torch.Tensor, names: Sequence[str] = ("mse", "psnr", "ssim"),
            *, data_range: Optional[float] = None, reduction: str = "mean",
            win_size: int = 11, sigma: float = 1.5,
            K: Sequence[float] = (0.01, 0.03), fuse_gmsd: bool = False) -> dict:
    """Several metrics of one batch of frame pairs, as a dict name -> tensor.

    SSIM together with MSE and/or PSNR comes from a single kernel that sums the
    squared differences while it stages the frames for SSIM: one read of the
    pair instead of two, one launch instead of two.  GMSD / GMS join the same
    pass (a 2x2-pooled Prewitt on the staged rows) for uint8 / float32 frames
    with the default 11-tap window when ``fuse_gmsd=True``.  That reads each
    frame once, but on B200 it measures slower than the SSIM and GMSD kernels
    run back to back (1.48 vs 1.37 ms for 8 uint8 4K frames: the SSIM kernel
    is bound by instruction issue, so the GMSD work it takes on costs more
    than the second read of the frames saves), so it is off by default.  The values equal those of
    :func:`ssim`, :func:`mse` and :func:`psnr` (uint8 MSE exact); the other
    names are computed by their own functions.  This is the computation behind
    the reference's StreamingMetrics (modules.py:373-402), with the same
    defaults."""
    _check_reduction(reduction)
    names = tuple(names)
    bad = [n for n in names if n not in METRIC_NAMES]
    if bad:
        raise ValueError(f"unknown metric(s) {bad}; expected any of {list(METRIC_NAMES)}")
    x4, y4, L, _ = _prep(x, y, None, 0, data_range)
    backend.require_cuda(x4)
    out = {}
    no_grad = not _grad_wanted(x4, y4)
    f32_ssim = x4.dtype != torch.float64  # float64 SSIM has kernels of its own
    want_gm = [n for n in ("gms", "gmsd") if n in names]
    want_sq = "mse" in names or "psnr" in names
    if fuse_gmsd and f32_ssim and "ssim" in names and want_gm and no_grad and win_size == 11 and \
            backend.ssim_gmsd_fusable(x4, y4, win_size):
        K1, K2 = float(K[0]), float(K[1])
        res = backend.ssim_gmsd(x4.detach(), y4.detach(), _kernel_window(win_size, sigma, x4.device),
                                shift=0.5 * L, C1=(K1 * L) ** 2, C2=(K2 * L) ** 2,
                                T=170.0 * (L / 255.0) ** 2, eps=(1e-6 * L) ** 2,
                                psnr_bias=math.log10(L * L) * 10.0,
                                per_image=(reduction == "none"), want_mse=want_sq)
        for n in ("mse", "psnr", "ssim"):
            if n in names and n in res:
                out[n] = res[n]
        for n in want_gm:
            out[n] = res[n] if reduction == "none" else res[n].mean()
    fused = f32_ssim and "ssim" in names and "ssim" not in out and want_sq and no_grad and \
        min(x4.shape[-2:]) >= win_size
    if fused:
        K1, K2 = float(K[0]), float(K[1])
        res = backend.ssim_mse(x4.detach(), y4.detach(), _kernel_window(win_size, sigma, x4.device),
                               shift=0.5 * L, C1=(K1 * L) ** 2, C2=(K2 * L) ** 2,
                               psnr_bias=math.log10(L * L) * 10.0,
                               per_image=(reduction == "none"))
        for n in ("mse", "psnr", "ssim"):
            if n in names:
                out[n] = res[n]
    kw_range = {"data_range": L}
    table = {
        "mse": lambda: mse(x4, y4, reduction=reduction),
        "psnr": lambda: psnr(x4, y4, reduction=reduction, **kw_range),
        "ssim": lambda: ssim(x4, y4, reduction=reduction, win_size=win_size, sigma=sigma, K=K,
                             **kw_range),
        "ms_ssim": lambda: ms_ssim(x4, y4, reduction=reduction, win_size=win_size, sigma=sigma,
                                   K=K, **kw_range),
        "gmsd": lambda: gmsd(x4, y4, reduction=reduction, **kw_range),
        "gms": lambda: gms(x4, y4, reduction=reduction, **kw_range),
        "l1": lambda: l1(x4, y4, reduction=reduction),
        "charbonnier": lambda: charbonnier(x4, y4, reduction=reduction),
        "huber": lambda: huber(x4, y4, reduction=reduction),
        "ssimulacra2": lambda: _ssimulacra2()(x4, y4, reduction=reduction, **kw_range),
    }
    for n in names:
        if n not in out:
            out[n] = table[n]()
    return out


def _ssimulacra2():
    from .ssimulacra2 import ssimulacra2
    return ssimulacra2


# --------------------------------------------------------------------------- #
# MS-SSIM
# --------------------------------------------------------------------------- #

class _FusedSSIMCS(torch.autograd.Function):
    """Differentiable per-plane ``(ssim, cs)`` means (functional.py:749-783)."""

    @staticmethod
    def forward(ctx, x, y, win, shift, C1, C2):
        res = backend.ssim_forward(x, y, win, shift=shift, C1=C1, C2=C2, want_cs=True)
        ctx.save_for_backward(x, y)
        ctx.win = win
        ctx.consts = (shift, C1, C2)
        return res["plane_s"], res["plane_cs"]

    @staticmethod
    def backward(ctx, g_s, g_cs):
        _reject_double_backward()
        x, y = ctx.saved_tensors
        win = ctx.win
        shift, C1, C2 = ctx.consts
        nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (nx or ny):
            return (None,) * 6
        if g_s is None:
            g_s = torch.zeros(x.shape[0] * x.shape[1], dtype=x.dtype, device=x.device)
        if g_cs is None:
            g_cs = torch.zeros_like(g_s)
        dx, dy = backend.ssim_backward(x, y, win, shift=shift, C1=C1, C2=C2,
                                       gs=g_s, gcs=g_cs, need_dx=nx, need_dy=ny)
        return (dx if nx else None, dy if ny else None, None, None, None, None)


class _Pool2Fn(torch.autograd.Function):
    """2x2 mean pool between MS-SSIM scales (functional.py:885), forward and
    adjoint both one kernel launch."""

    @staticmethod
    def forward(ctx, x):
        ctx.shape, ctx.dtype = tuple(x.shape), x.dtype
        return backend.pool2(x)

    @staticmethod
    def backward(ctx, g):
        return backend.pool2_backward(g, ctx.shape).to(ctx.dtype)


def _ms_weights(w, device) -> torch.Tensor:
    """Per-scale exponents as a (scales, 1, 1) float64 tensor on `device`."""
    key = (tuple(float(v) for v in w), str(device))
    if key not in _ms_weight_cache:
        _ms_weight_cache[key] = torch.as_tensor(key[0], dtype=torch.float64,
                                                device=device).reshape(len(key[0]), 1, 1)
    return _ms_weight_cache[key]


_ms_weight_cache: dict = {}


_ms_stream_cache: dict = {}


def _ms_streams(device, k):
    key = (device.index, k)
    st = _ms_stream_cache.get(key)
    if st is None:
        st = [torch.cuda.Stream(device=device) for _ in range(k)]
        _ms_stream_cache[key] = st
    return st


def _ms_terms_concurrent(x, y, lk, scales, win, shift, C1, C2):
    """Per-plane MS-SSIM factors (cs per scale, S at the coarsest), no
    gradient.  Scale 0 runs on the caller's stream and is enqueued first, so
    its blocks take the SMs first; the pyramid is pooled on a side stream
    (forked before scale 0, so it does not wait for it) and each coarser
    scale's SSIM runs on a stream of its own as soon as its level exists.
    The small grids of the coarse scales then fill the SMs that scale 0's
    blocks free, instead of delaying scale 0's last blocks.  Every side stream
    forks from and joins back into the caller's stream (each has its own
    workspace)."""
    main = torch.cuda.current_stream(x.device)
    streams = _ms_streams(x.device, scales)
    pyr_st, scale_st = streams[0], streams[1:]
    out = [None] * scales

    def one(i, cx, cy, luma, last):
        res = backend.ssim_forward(cx, cy, win, shift=shift, C1=C1, C2=C2, luma=luma,
                                   want_cs=True)
        return res["plane_s"] if last else res["plane_cs"]

    pyr_st.wait_stream(main)
    out[0] = one(0, x, y, lk, scales == 1)
    with torch.cuda.stream(pyr_st):
        cx, cy = x, y
        for i in range(1, scales):
            pl = lk if i == 1 else None
            cx, cy = backend.pool2(cx, luma=pl), backend.pool2(cy, luma=pl)
            st = scale_st[i - 1]
            st.wait_stream(pyr_st)
            with torch.cuda.stream(st):
                cx.record_stream(st)
                cy.record_stream(st)
                t = one(i, cx, cy, None, i == scales - 1)
                t.record_stream(main)
                out[i] = t
    for st in streams:
        main.wait_stream(st)
    return out


def ms_ssim(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
            win_size: int = 11, sigma: float = 1.5, K: Sequence[float] = (0.01, 0.03),
            weights: Optional[Sequence[float]] = None, reduction: str = "mean",
            dtype: Optional[torch.dtype] = None, backend_hint: str = "auto", luma=None,
            crop_border: int = 0) -> torch.Tensor:
    """Multi-scale SSIM (functional.py:811-901): per channel
    prod_j max(cs_j, 0)^w_j (the coarsest scale contributes full SSIM),
    channels averaged after the product, 2x2 mean pooling between scales."""
    _check_reduction(reduction)
    _check_hint(backend_hint)
    w = tuple(float(v) for v in (weights if weights is not None else MS_SSIM_WEIGHTS))
    if not w:
        raise ValueError("weights must not be empty")
    x4, y4, L, mode = _prep(x, y, luma, crop_border, data_range)
    backend.require_cuda(x4)
    K1, K2 = float(K[0]), float(K[1])
    C1, C2 = (K1 * L) ** 2, (K2 * L) ** 2
    shift = 0.5 * L
    need = (win_size - 1) * (1 << (len(w) - 1)) + (1 << (len(w) - 1))
    if min(x4.shape[-2], x4.shape[-1]) < need:
        raise ValueError(
            f"image {tuple(x4.shape[-2:])} is too small for {len(w)} scales with a "
            f"{win_size}x{win_size} window; needs at least {need} px on a side")
    win = _kernel_window(win_size, sigma, x4.device)
    lk = _luma_k(mode, L)
    grad = _grad_wanted(x4, y4)
    f64 = x4.dtype == torch.float64
    if lk is not None and (grad or f64):
        # (float64 pooling reads luma planes)
        x4, y4 = rgb_to_luma(x4, mode, data_range=L), rgb_to_luma(y4, mode, data_range=L)
        lk = None
    n = x4.shape[0]
    if not grad:
        terms = _ms_terms_concurrent(x4.detach(), y4.detach(), lk, len(w), win, shift, C1, C2)
        stacked = torch.stack([t.view(n, -1) for t in terms]).clamp_min(0.0)
        per_plane = stacked.pow(_ms_weights(w, x4.device)).prod(dim=0)
        per_image = per_plane.mean(dim=1)
        return per_image if reduction == "none" else per_image.mean()
    cx, cy = x4, y4
    terms = []
    for i in range(len(w)):
        # Scale 0 reads the inputs as given (luma projected inside the SSIM
        # kernel); the first pool projects too, so no full-resolution float
        # or luma copy is ever written.
        scale_lk = lk if i == 0 else None
        if i:
            if grad:
                cx, cy = _Pool2Fn.apply(cx), _Pool2Fn.apply(cy)
            else:
                pl = lk if i == 1 else None
                cx, cy = backend.pool2(cx, luma=pl), backend.pool2(cy, luma=pl)
        if grad:
            cdt = torch.float64 if f64 else torch.float32
            xf = cx.to(cdt).contiguous()
            yf = cy.to(cdt).contiguous()
            s, cs = _FusedSSIMCS.apply(xf, yf, win, shift, C1, C2)
        else:
            res = backend.ssim_forward(cx.detach(), cy.detach(), win, shift=shift, C1=C1,
                                       C2=C2, luma=scale_lk, want_cs=True)
            s, cs = res["plane_s"], res["plane_cs"]
        terms.append((s if i == len(w) - 1 else cs).view(n, -1))
    stacked = torch.stack(terms).clamp_min(0.0)
    per_plane = stacked.pow(_ms_weights(w, x4.device)).prod(dim=0)
    per_image = per_plane.mean(dim=1)
    return per_image if reduction == "none" else per_image.mean()


# --------------------------------------------------------------------------- #
# GMSD / GMS
# --------------------------------------------------------------------------- #

class _GmsdFn(torch.autograd.Function):
    """Differentiable per-image (GMS mean, GMSD) -- the GMSD.loss path.
    Forward: the fused kernel; backward: one fused kernel (transposed Prewitt
    and pool) fed with the forward's statistics."""

    @staticmethod
    def forward(ctx, x, y, T, eps, downsample):
        mean, std = backend.gmsd(x, y, T=T, eps=eps, downsample=downsample)
        ctx.save_for_backward(x, y, mean, std)
        ctx.consts = (T, eps, downsample)
        return mean, std

    @staticmethod
    def backward(ctx, g_mean, g_std):
        _reject_double_backward()
        x, y, mean, std = ctx.saved_tensors
        T, eps, down = ctx.consts
        nx, ny = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (nx or ny):
            return (None,) * 5
        dx, dy = backend.gmsd_backward(x, y, T=T, eps=eps, downsample=down, mean=mean,
                                       std=std, g_mean=g_mean, g_std=g_std,
                                       need_dx=nx, need_dy=ny)
        return dx, dy, None, None, None


def _gmsd_common(x, y, data_range, T, eps, downsample, luma, crop_border, reduction,
                 return_map, backend_hint):
    _check_reduction(reduction)
    _check_hint(backend_hint)
    x4, y4, L, mode = _prep(x, y, luma, crop_border, data_range)
    backend.require_cuda(x4)
    Tv = float(T) if T is not None else 170.0 * (L / 255.0) ** 2
    ev = float(eps) if eps is not None else (1e-6 * L) ** 2
    lk = _luma_k(mode, L)
    if return_map:
        q = backend.gms_map(x4, y4, T=Tv, eps=ev, downsample=downsample, luma=lk)
        return q, None
    hd = x4.shape[-2] // 2 if downsample else x4.shape[-2]
    wd = x4.shape[-1] // 2 if downsample else x4.shape[-1]
    if hd < 3 or wd < 3:
        raise ValueError(f"image {hd}x{wd} is smaller than the 3x3 Prewitt window")
    if _grad_wanted(x4, y4):
        # the fused backward reads float32 planes: luma/crop/cast with
        # differentiable torch ops first
        if lk is not None:
            x4, y4 = rgb_to_luma(x4, mode, data_range=L), rgb_to_luma(y4, mode, data_range=L)
        cdt = torch.float64 if x4.dtype == torch.float64 else torch.float32
        xf = x4.to(cdt).contiguous()
        yf = y4.to(cdt).contiguous()
        return None, _GmsdFn.apply(xf, yf, Tv, ev, bool(downsample))
    return None, backend.gmsd(x4.detach(), y4.detach(), T=Tv, eps=ev,
                              downsample=downsample, luma=lk)


def gms(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
        T: Optional[float] = None, eps: Optional[float] = None, downsample: bool = True,
        reduction: str = "mean", return_map: bool = False,
        dtype: Optional[torch.dtype] = None, luma=None, crop_border: int = 0,
        backend_hint: str = "auto") -> torch.Tensor:
    """Mean gradient-magnitude similarity (functional.py:1016-1038)."""
    q, stats = _gmsd_common(x, y, data_range, T, eps, downsample, luma, crop_border,
                            reduction, return_map, backend_hint)
    if q is not None:
        return q
    return stats[0] if reduction == "none" else stats[0].mean()


def gmsd(x: torch.Tensor, y: torch.Tensor, *, data_range: Optional[float] = None,
         T: Optional[float] = None, eps: Optional[float] = None, downsample: bool = True,
         reduction: str = "mean", return_map: bool = False,
         dtype: Optional[torch.dtype] = None, luma=None, crop_border: int = 0,
         backend_hint: str = "auto") -> torch.Tensor:
    """Gradient magnitude similarity deviation (functional.py:1041-1082):
    population std of the GMS map, pooled over every channel of an image."""
    q, stats = _gmsd_common(x, y, data_range, T, eps, downsample, luma, crop_border,
                            reduction, return_map, backend_hint)
    if q is not None:
        return q
    return stats[1] if reduction == "none" else stats[1].mean()

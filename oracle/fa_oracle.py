"""CPU oracle for the metric path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

A float64 numpy restatement of the reference's algorithms, written from the
reference's own oracle (frame_analytics/reference.py) and its batch/channel
conventions (frame_analytics/functional.py).  Only tests/, bench.py's
CPU-baseline leg and __graft_entry__.smoke() may import this module, and only
as the checker; the package never does.

Pinned against the reference: tests/golden/ holds vectors produced by running
the reference's own reference.py and its CPU library (fa_cpu.cpp) on seeded
inputs (script: tests/golden/make_golden.py), and tests/test_oracle.py checks
this module against every one of them.
"""

from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

MS_SSIM_WEIGHTS = (0.0448, 0.2856, 0.3001, 0.2363, 0.1333)  # reference.py:70
LUMA_COEFFS = {                                              # reference.py:81-85
    "bt601": (0.299, 0.587, 0.114, 0.0),
    "bt709": (0.2126, 0.7152, 0.0722, 0.0),
    "matlab": (65.481 / 255.0, 128.553 / 255.0, 24.966 / 255.0, 16.0 / 255.0),
}
_PREWITT_X = np.array([[1.0, 0.0, -1.0]] * 3) / 3.0          # reference.py:284-285
_PREWITT_Y = _PREWITT_X.T.copy()


# --------------------------------------------------------------------------- #
# windows and filters
# --------------------------------------------------------------------------- #

def gaussian_window_1d(win_size: int = 11, sigma: float = 1.5) -> np.ndarray:
    """Sum-normalised 1-D Gaussian (functional.py:397-420).  Its outer product
    is reference.gaussian_window_2d (reference.py:88-99): for the supported
    sizes no tap falls below eps*max, so MATLAB's zeroing never triggers."""
    r = (win_size - 1) / 2.0
    c = np.arange(win_size, dtype=np.float64) - r
    g = np.exp(-(c * c) / (2.0 * sigma * sigma))
    return g / g.sum()


def sep_valid(img: np.ndarray, w: np.ndarray) -> np.ndarray:
    """'valid' correlation with the separable window w (x) w over the last two
    axes (reference._valid_correlate2d, reference.py:103-115, for a rank-1
    kernel).  Vectorised over leading axes."""
    k = w.size
    h, wd = img.shape[-2], img.shape[-1]
    oh, ow = h - k + 1, wd - k + 1
    if oh <= 0 or ow <= 0:
        raise ValueError(f"image {img.shape[-2:]} smaller than window {k}")
    t = np.zeros(img.shape[:-1] + (ow,), dtype=np.float64)
    for j in range(k):
        t += w[j] * img[..., :, j:j + ow]
    out = np.zeros(img.shape[:-2] + (oh, ow), dtype=np.float64)
    for i in range(k):
        out += w[i] * t[..., i:i + oh, :]
    return out


def sep_full_transpose(m: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Adjoint of sep_valid: scatter an (oh, ow) map back onto (oh+k-1, ow+k-1)."""
    k = w.size
    oh, ow = m.shape[-2], m.shape[-1]
    t = np.zeros(m.shape[:-2] + (oh + k - 1, ow), dtype=np.float64)
    for i in range(k):
        t[..., i:i + oh, :] += w[i] * m
    out = np.zeros(m.shape[:-2] + (oh + k - 1, ow + k - 1), dtype=np.float64)
    for j in range(k):
        out[..., :, j:j + ow] += w[j] * t
    return out


def valid_correlate2d(img: np.ndarray, kern: np.ndarray) -> np.ndarray:
    """reference._valid_correlate2d (reference.py:103-115), leading axes vectorised."""
    kh, kw = kern.shape
    oh, ow = img.shape[-2] - kh + 1, img.shape[-1] - kw + 1
    out = np.zeros(img.shape[:-2] + (oh, ow), dtype=np.float64)
    for i in range(kh):
        for j in range(kw):
            if kern[i, j] != 0.0:
                out += kern[i, j] * img[..., i:i + oh, j:j + ow]
    return out


def avg_pool2(x: np.ndarray) -> np.ndarray:
    """2x2 non-overlapping mean, odd trailing row/column dropped (reference.py:231-241)."""
    h, w = x.shape[-2] // 2 * 2, x.shape[-1] // 2 * 2
    v = x[..., :h, :w]
    return v.reshape(*v.shape[:-2], h // 2, 2, w // 2, 2).mean(axis=(-3, -1))


# --------------------------------------------------------------------------- #
# input conventions (functional.py:141-271)
# --------------------------------------------------------------------------- #

def matlab_downsample(x: np.ndarray, f: int) -> np.ndarray:
    """MATLAB ssim.m's automatic downsample as the reference writes it
    (functional.py:575-586): replicate-pad f//2, f x f box mean (valid), then
    every f-th row and column.  x: (..., H, W) float64."""
    if f <= 1:
        return x
    pad = f // 2
    xp = np.pad(x, [(0, 0)] * (x.ndim - 2) + [(pad, pad), (pad, pad)], mode="edge")
    h, w = xp.shape[-2] - f + 1, xp.shape[-1] - f + 1
    acc = np.zeros(x.shape[:-2] + (h, w))
    for a in range(f):
        for b in range(f):
            acc += xp[..., a:a + h, b:b + w]
    return (acc / (f * f))[..., ::f, ::f]


def as_nchw(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a)
    if a.ndim == 2:
        return a[None, None]
    if a.ndim == 3:
        return a[None]
    if a.ndim == 4:
        return a
    raise ValueError(f"expected 2/3/4-D, got {a.shape}")


def rgb_to_luma(img: np.ndarray, mode: str, data_range: float) -> np.ndarray:
    """(N,3,H,W) -> (N,1,H,W) float64 (reference.rgb_to_luma_reference, reference.py:212-223)."""
    cr, cg, cb, off = LUMA_COEFFS[mode]
    v = np.asarray(img, dtype=np.float64)
    return (cr * v[:, 0:1] + cg * v[:, 1:2] + cb * v[:, 2:3] + off * float(data_range))


def prep(x, y, luma=None, crop_border=0, data_range=255.0):
    """NCHW float64 planes after crop and luma, as functional._prep/_apply_luma."""
    x4 = as_nchw(x).astype(np.float64)
    y4 = as_nchw(y).astype(np.float64)
    if crop_border:
        b = crop_border
        x4 = x4[..., b:-b, b:-b]
        y4 = y4[..., b:-b, b:-b]
    if luma:
        mode = "bt601" if luma is True else luma
        x4 = rgb_to_luma(x4, mode, data_range)
        y4 = rgb_to_luma(y4, mode, data_range)
    return x4, y4


# --------------------------------------------------------------------------- #
# pixel reductions (reference.py:118-204, functional.py:289-387)
# --------------------------------------------------------------------------- #

def ssd_uint8(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """Exact per-image sum of squared uint8 differences, int64."""
    x4, y4 = as_nchw(x), as_nchw(y)
    d = x4.astype(np.int64) - y4.astype(np.int64)
    return (d * d).reshape(d.shape[0], -1).sum(axis=1)


def pixel(x, y, op: str, param: float = 0.0, reduction: str = "mean",
          luma=None, crop_border=0, data_range=255.0):
    """mse / l1 / charbonnier (param = eps) / huber (param = delta), float64."""
    x4, y4 = prep(x, y, luma, crop_border, data_range)
    d = x4 - y4
    if op == "mse":
        t = d * d
    elif op == "l1":
        t = np.abs(d)
    elif op == "charbonnier":
        t = np.sqrt(d * d + float(param) ** 2)
    elif op == "huber":
        a = np.abs(d)
        t = np.where(a <= param, 0.5 * a * a, param * (a - 0.5 * param))
    else:
        raise ValueError(op)
    per = t.reshape(t.shape[0], -1).mean(axis=1)
    return per if reduction == "none" else float(t.mean())


def psnr(x, y, data_range=255.0, reduction="mean", luma=None, crop_border=0):
    m = pixel(x, y, "mse", reduction=reduction, luma=luma, crop_border=crop_border,
              data_range=data_range)
    with np.errstate(divide="ignore"):
        return 10.0 * np.log10(data_range * data_range / np.asarray(m)) if reduction == "none" \
            else (float("inf") if m == 0 else float(10.0 * np.log10(data_range ** 2 / m)))


# --------------------------------------------------------------------------- #
# SSIM (reference.py:118-175; batch conventions functional.py:589-689)
# --------------------------------------------------------------------------- #

def ssim_maps(x, y, data_range=255.0, win_size=11, sigma=1.5, K1=0.01, K2=0.03):
    """(ssim_map, cs_map) over the last two axes, float64 (reference._ssim_maps)."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    w = gaussian_window_1d(win_size, sigma)
    C1, C2 = (K1 * data_range) ** 2, (K2 * data_range) ** 2
    mx, my = sep_valid(x, w), sep_valid(y, w)
    sxx = sep_valid(x * x, w) - mx * mx
    syy = sep_valid(y * y, w) - my * my
    sxy = sep_valid(x * y, w) - mx * my
    cs = (2 * sxy + C2) / (sxx + syy + C2)
    lum = (2 * mx * my + C1) / (mx * mx + my * my + C1)
    return lum * cs, cs


def ssim(x, y, data_range=255.0, win_size=11, sigma=1.5, K=(0.01, 0.03),
         reduction="mean", return_map=False, luma=None, crop_border=0):
    x4, y4 = prep(x, y, luma, crop_border, data_range)
    s, _ = ssim_maps(x4, y4, data_range, win_size, sigma, K[0], K[1])
    if return_map:
        return s
    per = s.reshape(s.shape[0], -1).mean(axis=1)
    return per if reduction == "none" else float(s.mean())


def ssim_grad(x, y, data_range=1.0, win_size=11, sigma=1.5, K=(0.01, 0.03),
              upstream=None):
    """d(sum_o upstream(o) * S(o)) / dx and / dy for NCHW float64 inputs.

    ``upstream`` defaults to the batch-mean weight 1 / (N*C*Hout*Wout).
    Restates the reference's backward (fa_cuda.cu:551-607 coefficient maps and
    the transposed blur of 655-784) in float64 without the shift."""
    x = np.asarray(x, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    w = gaussian_window_1d(win_size, sigma)
    C1, C2 = (K[0] * data_range) ** 2, (K[1] * data_range) ** 2
    mx, my = sep_valid(x, w), sep_valid(y, w)
    sxx = sep_valid(x * x, w) - mx * mx
    syy = sep_valid(y * y, w) - my * my
    sxy = sep_valid(x * y, w) - mx * my
    A1, A2 = 2 * mx * my + C1, 2 * sxy + C2
    B1, B2 = mx * mx + my * my + C1, sxx + syy + C2
    S = A1 * A2 / (B1 * B2)
    g = np.full(S.shape, 1.0 / S.size) if upstream is None else np.broadcast_to(upstream, S.shape)
    b = g * (-S / B2)                       # dS/dsxx (= dS/dsyy)
    c = g * (2 * A1 / (B1 * B2))            # dS/dsxy
    dmx = g * (2 * A2 / (B1 * B2)) * (my - mx * A1 / B1)
    dmy = g * (2 * A2 / (B1 * B2)) * (mx - my * A1 / B1)
    tx = dmx - 2 * b * mx - c * my
    ty = dmy - 2 * b * my - c * mx
    Pb, Pc = sep_full_transpose(b, w), sep_full_transpose(c, w)
    dx = 2 * x * Pb + y * Pc + sep_full_transpose(tx, w)
    dy = 2 * y * Pb + x * Pc + sep_full_transpose(ty, w)
    return dx, dy


# --------------------------------------------------------------------------- #
# MS-SSIM (reference.py:244-276; channel convention functional.py:876-901)
# --------------------------------------------------------------------------- #

def ms_ssim(x, y, data_range=255.0, win_size=11, sigma=1.5, K=(0.01, 0.03),
            weights: Sequence[float] = MS_SSIM_WEIGHTS, reduction="mean",
            luma=None, crop_border=0):
    """Per plane prod_j max(v_j, 0)^w_j (v = cs, full SSIM at the coarsest
    scale); channels averaged after the product, then images."""
    cx, cy = prep(x, y, luma, crop_border, data_range)
    per_plane = np.ones(cx.shape[:2])
    for i, wi in enumerate(weights):
        if i:
            cx, cy = avg_pool2(cx), avg_pool2(cy)
        s, cs = ssim_maps(cx, cy, data_range, win_size, sigma, K[0], K[1])
        v = (s if i == len(weights) - 1 else cs).mean(axis=(-2, -1))
        per_plane = per_plane * np.maximum(v, 0.0) ** wi
    per_image = per_plane.mean(axis=1)
    return per_image if reduction == "none" else float(per_image.mean())


# --------------------------------------------------------------------------- #
# GMSD (reference.py:288-335; channel pooling fa_cpu.cpp:964-978)
# --------------------------------------------------------------------------- #

def gms_map(x, y, data_range=255.0, T=None, downsample=True, eps=None,
            luma=None, crop_border=0):
    cx, cy = prep(x, y, luma, crop_border, data_range)
    if T is None:
        T = 170.0 * (float(data_range) / 255.0) ** 2
    if eps is None:
        eps = (1e-6 * float(data_range)) ** 2
    if downsample:
        cx, cy = avg_pool2(cx), avg_pool2(cy)
    g1 = np.sqrt(valid_correlate2d(cx, _PREWITT_X) ** 2 + valid_correlate2d(cx, _PREWITT_Y) ** 2 + eps)
    g2 = np.sqrt(valid_correlate2d(cy, _PREWITT_X) ** 2 + valid_correlate2d(cy, _PREWITT_Y) ** 2 + eps)
    return (2 * g1 * g2 + T) / (g1 * g1 + g2 * g2 + T)


def gmsd(x, y, data_range=255.0, T=None, downsample=True, eps=None,
         luma=None, crop_border=0):
    """(gms mean, gmsd) per image: population mean/std over all C' maps."""
    q = gms_map(x, y, data_range, T, downsample, eps, luma, crop_border)
    f = q.reshape(q.shape[0], -1)
    return f.mean(axis=1), f.std(axis=1)

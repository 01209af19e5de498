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


# --------------------------------------------------------------------------- #
# SSIMULACRA 2 (reference.py:540-700, the float64 transcription of libjxl's
# tools/ssimulacra2.cc; frame_analytics/ssimulacra2.py for the conventions)
# --------------------------------------------------------------------------- #

# Msssim::Score weights: channel-major, then scale, then norm (1, 4), then the
# three maps (SSIM', ringing, blurring).  A published constant of the metric.
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
    0.0, 0.0, 0.0, 0.0005130064588990679, 0.0, 0.00010854057858411537,
)
_S2_OPSIN = np.array([[0.30, 1.0 - 0.078 - 0.30, 0.078],
                      [0.23, 1.0 - 0.078 - 0.23, 0.078],
                      [0.24342268924547819, 0.20476744424496821,
                       1.0 - 0.24342268924547819 - 0.20476744424496821]])
_S2_BIAS = 0.0037930732552754493
_S2_C2 = 0.0009


def recursive_gaussian_taps(sigma: float = 1.5) -> np.ndarray:
    """The FIR equivalent of the truncated-cosine recursive Gaussian of
    Charalampidis (2016), the blur libjxl's SSIMULACRA 2 uses: three cosines
    cos(w_k t), w_k = (2k+1) pi / (2N), N = round(3.2795 sigma + 0.2546),
    weighted by the beta that solves the paper's normalisation, first-moment
    and Gaussian-fit conditions (eqs. 37-56); 2N + 1 taps, the outer two 0."""
    n = int(round(3.2795 * sigma + 0.2546))
    w = np.array([1.0, 3.0, 5.0]) * np.pi / (2.0 * n)
    p = np.array([1.0, -1.0, 1.0]) / np.tan(0.5 * w)
    r = np.array([1.0, -1.0, 1.0]) * p * p / np.sin(w)
    rho = np.exp(-0.5 * sigma * sigma * w * w) / n
    d13 = p[0] * r[1] - r[0] * p[1]
    z15 = (p[1] * r[2] - r[1] * p[2]) / d13
    z35 = (p[2] * r[0] - r[2] * p[0]) / d13
    beta = np.linalg.solve(np.array([p, r, [z15, z35, 1.0]]),
                           np.array([1.0, n * n - sigma * sigma,
                                     z15 * rho[0] + z35 * rho[1] + rho[2]]))
    t = np.arange(-n, n + 1, dtype=np.float64)
    return (beta[:, None] * np.cos(w[:, None] * t[None, :])).sum(axis=0)


def _s2_blur(img: np.ndarray, taps: np.ndarray) -> np.ndarray:
    """Separable same-size blur of (..., H, W) planes, zero outside."""
    k = len(taps) // 2
    out = np.zeros_like(img)
    pad = np.pad(img, [(0, 0)] * (img.ndim - 1) + [(k, k)])
    for j, w in enumerate(taps):
        out += w * pad[..., j:j + img.shape[-1]]
    pad = np.pad(out, [(0, 0)] * (img.ndim - 2) + [(k, k), (0, 0)])
    out2 = np.zeros_like(img)
    for j, w in enumerate(taps):
        out2 += w * pad[..., j:j + img.shape[-2], :]
    return out2


def _s2_linear(v: np.ndarray) -> np.ndarray:
    return np.where(v <= 0.04045, v / 12.92, ((v + 0.055) / 1.055) ** 2.4)


def _s2_xyb(lin: np.ndarray) -> np.ndarray:
    """(3, H, W) linear sRGB -> positive XYB."""
    m = np.einsum("ji,ihw->jhw", _S2_OPSIN, lin) + _S2_BIAS
    m = np.cbrt(np.maximum(m, 0.0)) - np.cbrt(_S2_BIAS)
    x, y = 0.5 * (m[0] - m[1]), 0.5 * (m[0] + m[1])
    return np.stack([14.0 * x + 0.42, y + 0.01, (m[2] - y) + 0.55])


def _s2_down(img: np.ndarray) -> np.ndarray:
    """2x2 box mean, an odd last row / column averaged with itself."""
    c, h, w = img.shape
    p = np.pad(img, [(0, 0), (0, h % 2), (0, w % 2)], mode="edge")
    return 0.25 * (p[:, 0::2, 0::2] + p[:, 1::2, 0::2] + p[:, 0::2, 1::2] + p[:, 1::2, 1::2])


def ssimulacra2(x: np.ndarray, y: np.ndarray, data_range: float = 255.0) -> float:
    """SSIMULACRA 2 of one (3, H, W) sRGB pair (original x, distorted y)."""
    taps = recursive_gaussian_taps(1.5)
    l1 = _s2_linear(np.asarray(x, np.float64) / data_range)
    l2 = _s2_linear(np.asarray(y, np.float64) / data_range)
    norms = []
    prev = l1.shape[1:]
    for scale in range(6):
        if min(prev) < 8:
            break
        if scale:
            l1, l2 = _s2_down(l1), _s2_down(l2)
        a, b = _s2_xyb(l1), _s2_xyb(l2)
        mu1, mu2 = _s2_blur(a, taps), _s2_blur(b, taps)
        s11, s22, s12 = _s2_blur(a * a, taps), _s2_blur(b * b, taps), _s2_blur(a * b, taps)
        num_m = 1.0 - (mu1 - mu2) ** 2
        num_s = 2.0 * (s12 - mu1 * mu2) + _S2_C2
        den_s = (s11 - mu1 * mu1) + (s22 - mu2 * mu2) + _S2_C2
        d = np.maximum(1.0 - num_m * num_s / den_s, 0.0)
        e = (1.0 + np.abs(b - mu2)) / (1.0 + np.abs(a - mu1)) - 1.0
        maps = (d, np.maximum(e, 0.0), np.maximum(-e, 0.0))
        norms.append([(m.mean(axis=(1, 2)), np.sqrt(np.sqrt((m ** 4).mean(axis=(1, 2)))))
                      for m in maps])
        prev = l1.shape[1:]
    total, i = 0.0, 0
    for c in range(3):
        for sc in norms:
            for nrm in range(2):
                for mp in range(3):
                    total += SSIMULACRA2_WEIGHTS[i] * abs(sc[mp][nrm][c])
                    i += 1
    s = total * 0.9562382616834844
    s = 2.326765642916932 * s - 0.020884521182843837 * s * s + 6.248496625763138e-05 * s ** 3
    return 100.0 if s <= 0.0 else 100.0 - 10.0 * s ** 0.6276336467831387

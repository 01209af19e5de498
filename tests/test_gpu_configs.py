"""Parity at the benchmarked configurations, at their full size, and the
reference's own gradient bars for MS-SSIM and GMS.

* config 2 (fp32 8x3x1080x1920 SSIM loss, forward + backward, gradient with
  respect to the prediction) runs exactly as ``bench.py`` times it,
  ``1 - fa.ssim(a, b)``; two of its images are checked against the float64
  oracle: per-image value at 5e-6, gradient at 1e-4 relative.
* config 3 (uint8 MS-SSIM): one full 3x1080x1920 pair against the oracle.
* config 4 (uint8 SSIM + GMSD, ``reduction='none'``): one 3x2160x3840 pair.
* MS-SSIM gradient: within 2e-4 of float64 torch autograd and 1e-3 of central
  differences of the float64 oracle (the bars of the reference's
  tests/test_training_metrics.py:134-175).
* GMS / GMSD gradient: within 1e-4 of float64 torch autograd.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import fa_oracle as O
from conftest import baseline_pair

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu
SHAPE2 = (8, 3, 1080, 1920)


def _cfg2_host():
    """Config 2's generator, the one bench.py uses: a ~ U[0,1],
    b = clamp(a + N(0, 0.05^2), 0, 1), fp32, seed 0."""
    g = torch.Generator().manual_seed(0)
    a = torch.rand(SHAPE2, generator=g)
    b = (a + 0.05 * torch.randn(SHAPE2, generator=g)).clamp_(0, 1)
    return a, b


def _rel(got, want):
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def test_config2_full_size_loss_and_gradient():
    a, b = _cfg2_host()
    x = a.cuda()
    y = b.cuda().requires_grad_(True)
    loss = 1 - fa.ssim(x, y, data_range=1.0)
    loss.backward()
    per = fa.ssim(x, y.detach(), data_range=1.0, reduction="none").cpu().numpy()
    assert abs((1 - float(loss)) - float(per.mean())) < 1e-7
    pick = [0, 7]
    an, bn = a[pick].double().numpy(), b[pick].double().numpy()
    np.testing.assert_allclose(per[pick], O.ssim(an, bn, data_range=1.0, reduction="none"),
                               rtol=0, atol=5e-6)
    # d(1 - mean over 8 images)/db of image i = -(1/8) d(mean of image i)/db
    g = y.grad[pick].double().cpu().numpy()
    for j in range(2):
        _, dy = O.ssim_grad(an[j:j + 1], bn[j:j + 1], data_range=1.0)
        assert _rel(-8.0 * g[j:j + 1], dy) < 1e-4


def test_config3_full_size_ms_ssim():
    a, b = baseline_pair((1, 3, 1080, 1920), 8.0, seed=0)
    x, y = torch.as_tensor(a, device="cuda"), torch.as_tensor(b, device="cuda")
    got = float(fa.ms_ssim(x, y, data_range=255.0))
    assert abs(got - O.ms_ssim(a, b, data_range=255.0)) < 5e-6


def test_config4_full_size_ssim_and_gmsd():
    a, b = baseline_pair((1, 3, 2160, 3840), 8.0, seed=4)
    x, y = torch.as_tensor(a, device="cuda"), torch.as_tensor(b, device="cuda")
    s = fa.ssim(x, y, reduction="none").cpu().numpy()
    np.testing.assert_allclose(s, O.ssim(a, b, reduction="none"), rtol=0, atol=5e-6)
    m, d = O.gmsd(a, b, eps=(1e-6 * 255.0) ** 2)
    np.testing.assert_allclose(fa.gmsd(x, y, reduction="none").cpu().numpy(), d, rtol=0, atol=5e-6)
    np.testing.assert_allclose(fa.gms(x, y, reduction="none").cpu().numpy(), m, rtol=0, atol=5e-6)


# ---------------------------------------------------------------------------- #
# MS-SSIM gradient
# ---------------------------------------------------------------------------- #

def _torch_ms_ssim(x, y, data_range=1.0, weights=O.MS_SSIM_WEIGHTS):
    """float64 torch autograd MS-SSIM: Gaussian 11/1.5, 2x2 average pooling
    between scales (odd trailing row / column dropped), per-plane product of
    clamped cs (SSIM at the last scale), mean over channels then images."""
    w = torch.tensor(O.gaussian_window_1d(11, 1.5), dtype=x.dtype, device=x.device)
    C1, C2 = (0.01 * data_range) ** 2, (0.03 * data_range) ** 2
    n, c = x.shape[:2]

    def blur(t):
        h, wd = t.shape[-2:]
        t = t.reshape(n * c, 1, h, wd)
        t = F.conv2d(F.conv2d(t, w.view(1, 1, 11, 1)), w.view(1, 1, 1, 11))
        return t.reshape(n, c, h - 10, wd - 10)

    prod = torch.ones(n, c, dtype=x.dtype, device=x.device)
    for i, wi in enumerate(weights):
        if i:
            x, y = F.avg_pool2d(x, 2), F.avg_pool2d(y, 2)
        mx, my = blur(x), blur(y)
        sxx, syy, sxy = blur(x * x) - mx * mx, blur(y * y) - my * my, blur(x * y) - mx * my
        cs = (2 * sxy + C2) / (sxx + syy + C2)
        v = (((2 * mx * my + C1) / (mx * mx + my * my + C1)) * cs if i == len(weights) - 1
             else cs).mean(dim=(-2, -1))
        prod = prod * torch.clamp(v, min=0.0) ** wi
    return prod.mean(1).mean()


@pytest.mark.parametrize("shape", [(1, 1, 192, 192), (2, 3, 180, 200)])
@pytest.mark.parametrize("wrt", ["x", "y", "xy"])
def test_ms_ssim_gradient_matches_float64_autograd(shape, wrt):
    g = torch.Generator().manual_seed(0)
    x0 = torch.rand(shape, generator=g)
    y0 = (x0 + 0.05 * torch.randn(shape, generator=g)).clamp(0, 1)
    x = x0.cuda().requires_grad_("x" in wrt)
    y = y0.cuda().requires_grad_("y" in wrt)
    (1.0 - fa.ms_ssim(x, y, data_range=1.0)).backward()
    xr = x0.double().cuda().requires_grad_("x" in wrt)
    yr = y0.double().cuda().requires_grad_("y" in wrt)
    (1.0 - _torch_ms_ssim(xr, yr)).backward()
    for got, want in ((x.grad, xr.grad), (y.grad, yr.grad)):
        assert (got is None) == (want is None)
        if got is not None:
            rel = float((got.double() - want).abs().max() / want.abs().max())
            assert rel < 2e-4, rel


def test_ms_ssim_gradient_vs_central_differences():
    """Independent of autograd: central differences of the float64 oracle at
    three pixels, 1e-3 relative."""
    rng = np.random.default_rng(2)
    a = rng.random((1, 1, 180, 180))
    b = np.clip(a + 0.05 * rng.standard_normal(a.shape), 0, 1)
    x = torch.as_tensor(a, dtype=torch.float32, device="cuda").requires_grad_(True)
    fa.ms_ssim(x, torch.as_tensor(b, dtype=torch.float32, device="cuda"), data_range=1.0).backward()
    gr = x.grad[0, 0].double().cpu().numpy()
    h = 1e-4
    for (i, j) in [(40, 60), (90, 90), (120, 33)]:
        p, m = a.copy(), a.copy()
        p[0, 0, i, j] += h
        m[0, 0, i, j] -= h
        fd = (O.ms_ssim(p, b, data_range=1.0) - O.ms_ssim(m, b, data_range=1.0)) / (2 * h)
        assert abs(fd - gr[i, j]) / max(abs(fd), 1e-12) < 1e-3


# ---------------------------------------------------------------------------- #
# GMS / GMSD gradient
# ---------------------------------------------------------------------------- #

def _torch_gms_stats(x, y, T, eps, down):
    if down:
        x, y = F.avg_pool2d(x, 2), F.avg_pool2d(y, 2)
    k = torch.tensor([[1.0, 0.0, -1.0]] * 3, dtype=x.dtype, device=x.device) / 3.0
    kk = torch.stack([k, k.t()]).unsqueeze(1)
    n, c, h, w = x.shape
    gx = F.conv2d(x.reshape(n * c, 1, h, w), kk)
    gy = F.conv2d(y.reshape(n * c, 1, h, w), kk)
    g1 = torch.sqrt((gx * gx).sum(1) + eps)
    g2 = torch.sqrt((gy * gy).sum(1) + eps)
    q = ((2 * g1 * g2 + T) / (g1 * g1 + g2 * g2 + T)).reshape(n, -1)
    return q.mean(1), q.std(1, correction=0)


@pytest.mark.parametrize("down", [True, False])
@pytest.mark.parametrize("shape", [(2, 3, 41, 53), (1, 1, 70, 97), (1, 3, 128, 160)])
def test_gms_gmsd_gradient_matches_float64_autograd(down, shape):
    g = torch.Generator().manual_seed(1)
    a = torch.rand(shape, generator=g, dtype=torch.float64)
    b = (a + 0.1 * torch.randn(shape, generator=g, dtype=torch.float64)).clamp(0, 1)
    # the float64 reference sees exactly the float32 values the kernel sees
    a, b = a.float().double().cuda(), b.float().double().cuda()
    T = 170.0 / 255 ** 2
    w1 = torch.randn(shape[0], generator=g, dtype=torch.float64).cuda()
    w2 = torch.randn(shape[0], generator=g, dtype=torch.float64).cuda()
    x, y = a.float().requires_grad_(), b.float().requires_grad_()
    m = fa.gms(x, y, data_range=1.0, downsample=down, reduction="none")
    s = fa.gmsd(x, y, data_range=1.0, downsample=down, reduction="none")
    gx, gy = torch.autograd.grad((m * w1).sum() + (s * w2).sum(), (x, y))
    xr, yr = a.clone().requires_grad_(), b.clone().requires_grad_()
    mr, sr = _torch_gms_stats(xr, yr, T, (1e-6) ** 2, down)
    rx, ry = torch.autograd.grad((mr * w1).sum() + (sr * w2).sum(), (xr, yr))
    for got, want in ((gx, rx), (gy, ry)):
        err = float((got.double() - want).abs().max() / want.abs().max())
        assert err < 1e-4, err

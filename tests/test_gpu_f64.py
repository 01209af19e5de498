"""float64 frames are computed in float64 (the reference's float64 torch path,
functional.py:589-689 / 697-901 / 974-1082, has no float32 step): values,
maps and gradients against the float64 oracle and float64 torch autograd at
float64 tolerances, including a pair that differs only below float32
resolution."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O
from test_gpu_configs import _torch_gms_stats, _torch_ms_ssim

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu


def _pair(shape, seed, noise=0.05):
    rng = np.random.default_rng(seed)
    a = rng.random(shape)
    return a, np.clip(a + noise * rng.standard_normal(shape), 0, 1)


def D(a):
    return torch.as_tensor(a, dtype=torch.float64, device="cuda")


@pytest.mark.parametrize("shape", [(2, 3, 40, 52), (1, 1, 11, 11), (1, 2, 77, 123)])
def test_ssim_value_map_and_reduction(shape):
    a, b = _pair(shape, sum(shape))
    x, y = D(a), D(b)
    assert abs(float(fa.ssim(x, y, data_range=1.0)) - O.ssim(a, b, data_range=1.0)) < 1e-12
    np.testing.assert_allclose(fa.ssim(x, y, data_range=1.0, reduction="none").cpu().numpy(),
                               O.ssim(a, b, data_range=1.0, reduction="none"), rtol=0, atol=1e-12)
    m = fa.ssim(x, y, data_range=1.0, return_map=True)
    assert m.dtype == torch.float64
    np.testing.assert_allclose(m.cpu().numpy(), O.ssim(a, b, data_range=1.0, return_map=True),
                               rtol=0, atol=1e-12)


def test_differences_below_float32_resolution_survive():
    """b = a + N(0, (2e-8)^2): below float32 resolution, so rounding the pair
    to float32 first would change the answer; float64 keeps it."""
    a, _ = _pair((1, 1, 64, 64), 7)
    rng = np.random.default_rng(8)
    b = a + 2e-8 * rng.standard_normal(a.shape)
    want = O.ssim(a, b, data_range=1.0)
    got = float(fa.ssim(D(a), D(b), data_range=1.0))
    f32 = O.ssim(a.astype(np.float32), b.astype(np.float32), data_range=1.0)
    assert want < 1.0 and abs(got - want) < 1e-15 < abs(f32 - want)
    wm, ws = O.gmsd(a, b, data_range=1.0, eps=1e-12)
    gs = fa.gmsd(D(a), D(b), data_range=1.0, reduction="none").cpu().numpy()
    np.testing.assert_allclose(gs, ws, rtol=1e-6, atol=1e-15)
    assert gs[0] > 0


def test_luma_and_crop():
    a, b = _pair((2, 3, 60, 70), 3)
    got = fa.ssim(D(a), D(b), data_range=1.0, luma="bt709", crop_border=4, reduction="none")
    want = O.ssim(a, b, data_range=1.0, luma="bt709", crop_border=4, reduction="none")
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=0, atol=1e-12)


@pytest.mark.parametrize("red", ["mean", "none", "map"])
def test_ssim_gradient(red):
    a, b = _pair((2, 2, 37, 45), 5)
    x, y = D(a).requires_grad_(), D(b).requires_grad_()
    if red == "map":
        m = fa.ssim(x, y, data_range=1.0, return_map=True)
        w = torch.randn(m.shape, generator=torch.Generator().manual_seed(0),
                        dtype=torch.float64).cuda()
        (m * w).sum().backward()
        up = w.cpu().numpy()
    elif red == "none":
        v = fa.ssim(x, y, data_range=1.0, reduction="none")
        wn = torch.tensor([0.7, -1.3], dtype=torch.float64, device="cuda")
        (v * wn).sum().backward()
        up = np.broadcast_to((wn.cpu().numpy() / (2 * 27 * 35))[:, None, None, None],
                             (2, 2, 27, 35))
    else:
        (1 - fa.ssim(x, y, data_range=1.0)).backward()
        up = -np.full((2, 2, 27, 35), 1.0 / (2 * 2 * 27 * 35))
    dx, dy = O.ssim_grad(a, b, data_range=1.0, upstream=up)
    for got, want in ((x.grad, dx), (y.grad, dy)):
        assert got.dtype == torch.float64
        rel = float(np.abs(got.cpu().numpy() - want).max() / np.abs(want).max())
        assert rel < 1e-10, rel


def test_ms_ssim_value_and_gradient():
    a, b = _pair((1, 2, 180, 192), 9)
    x, y = D(a), D(b)
    assert abs(float(fa.ms_ssim(x, y, data_range=1.0)) - O.ms_ssim(a, b, data_range=1.0)) < 1e-12
    xr = x.clone().requires_grad_()
    (1 - fa.ms_ssim(xr, y, data_range=1.0)).backward()
    xt = x.clone().requires_grad_()
    (1 - _torch_ms_ssim(xt, y)).backward()
    rel = float((xr.grad - xt.grad).abs().max() / xt.grad.abs().max())
    assert rel < 1e-9, rel


@pytest.mark.parametrize("down", [True, False])
def test_gmsd_value_and_gradient(down):
    a, b = _pair((2, 3, 41, 53), 11, noise=0.1)
    x, y = D(a), D(b)
    T, eps = 170.0 / 255 ** 2, 1e-12
    m, s = O.gmsd(a, b, data_range=1.0, downsample=down, eps=eps)
    np.testing.assert_allclose(fa.gmsd(x, y, data_range=1.0, downsample=down,
                                       reduction="none").cpu().numpy(), s, rtol=0, atol=1e-12)
    np.testing.assert_allclose(fa.gms(x, y, data_range=1.0, downsample=down,
                                      reduction="none").cpu().numpy(), m, rtol=0, atol=1e-12)
    q = fa.gms(x, y, data_range=1.0, downsample=down, return_map=True)
    assert q.dtype == torch.float64
    np.testing.assert_allclose(q.cpu().numpy(), O.gms_map(a, b, 1.0, downsample=down, eps=eps),
                               rtol=0, atol=1e-12)
    w1 = torch.randn(2, dtype=torch.float64, device="cuda")
    w2 = torch.randn(2, dtype=torch.float64, device="cuda")
    xg, yg = x.clone().requires_grad_(), y.clone().requires_grad_()
    mm = fa.gms(xg, yg, data_range=1.0, downsample=down, reduction="none")
    ss = fa.gmsd(xg, yg, data_range=1.0, downsample=down, reduction="none")
    gx, gy = torch.autograd.grad((mm * w1).sum() + (ss * w2).sum(), (xg, yg))
    xr, yr = x.clone().requires_grad_(), y.clone().requires_grad_()
    mr, sr = _torch_gms_stats(xr, yr, T, eps, down)
    rx, ry = torch.autograd.grad((mr * w1).sum() + (sr * w2).sum(), (xr, yr))
    for got, want in ((gx, rx), (gy, ry)):
        rel = float((got - want).abs().max() / want.abs().max())
        assert rel < 1e-9, rel

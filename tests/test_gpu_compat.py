"""The reference-compatible fa_cuda_* entry points, called the way the
reference's backend.py calls them (frame_analytics/backend.py:294-666)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import baseline_pair

from frame_analytics_b200 import _cabi

pytestmark = pytest.mark.gpu


def T(a, dt=torch.uint8):
    return torch.as_tensor(np.asarray(a), dtype=dt, device="cuda")


def _st():
    return torch.cuda.current_stream().cuda_stream


def _win(k=11):
    c = torch.arange(k, dtype=torch.float64) - (k - 1) / 2
    g = torch.exp(-(c * c) / 4.5)
    return (g / g.sum()).float().cuda()


def test_pixel_reduce_compat():
    lib = _cabi.load()
    a, b = baseline_pair((3, 2, 31, 47), 7.0, seed=1)
    x, y = T(a), T(b)
    n, per = 3, 2 * 31 * 47
    bpi = ctypes.c_int(0)
    assert lib.fa_cuda_pixel_workspace(n, per, 0, ctypes.byref(bpi)) == 0
    part = torch.empty((n, bpi.value), dtype=torch.float64, device="cuda")
    out = torch.empty(n, dtype=torch.float64, device="cuda")
    tot = torch.empty((), dtype=torch.float64, device="cuda")
    rc = lib.fa_cuda_pixel_reduce(x.data_ptr(), y.data_ptr(), 0, n, per, 0, 0.0, -1e300,
                                  part.data_ptr(), bpi.value, out.data_ptr(), tot.data_ptr(),
                                  None, None, 0, _st())
    assert rc == 0
    np.testing.assert_array_equal(out.cpu().numpy(), O.pixel(a, b, "mse", reduction="none"))
    assert float(tot) == O.pixel(a, b, "mse")


def test_ssim_and_cs_compat():
    lib = _cabi.load()
    a, b = baseline_pair((2, 3, 60, 70), 9.0, seed=2)
    x, y = T(a), T(b)
    w = _win()
    bpp = ctypes.c_int(0)
    assert lib.fa_cuda_ssim_workspace(60, 70, 11, ctypes.byref(bpp)) == 0
    part = torch.empty((6, bpp.value), dtype=torch.float64, device="cuda")
    per = torch.empty(2, dtype=torch.float64, device="cuda")
    tot = torch.empty((), dtype=torch.float64, device="cuda")
    rc = lib.fa_cuda_ssim(x.data_ptr(), y.data_ptr(), 0, 2, 3, 60, 70, w.data_ptr(), 11,
                          127.5, (0.01 * 255) ** 2, (0.03 * 255) ** 2, None, part.data_ptr(),
                          bpp.value, per.data_ptr(), tot.data_ptr(), 0, _st())
    assert rc == 0
    np.testing.assert_allclose(per.cpu().numpy(), O.ssim(a, b, reduction="none"), atol=5e-6)
    part2 = torch.empty_like(part)
    s = torch.empty(6, dtype=torch.float64, device="cuda")
    cs = torch.empty(6, dtype=torch.float64, device="cuda")
    rc = lib.fa_cuda_ssim_cs(x.data_ptr(), y.data_ptr(), 0, 2, 3, 60, 70, w.data_ptr(), 11,
                             127.5, (0.01 * 255) ** 2, (0.03 * 255) ** 2, part.data_ptr(),
                             part2.data_ptr(), bpp.value, s.data_ptr(), cs.data_ptr(), 0, _st())
    assert rc == 0
    sm, csm = O.ssim_maps(a.astype(np.float64), b.astype(np.float64))
    np.testing.assert_allclose(s.cpu().numpy(), sm.mean(axis=(-2, -1)).ravel(), atol=5e-6)
    np.testing.assert_allclose(cs.cpu().numpy(), csm.mean(axis=(-2, -1)).ravel(), atol=5e-6)


def test_ssim_backward_compat_without_aux():
    lib = _cabi.load()
    rng = np.random.default_rng(0)
    a = rng.random((1, 2, 30, 40)).astype(np.float32)
    b = np.clip(a + 0.05 * rng.standard_normal(a.shape), 0, 1).astype(np.float32)
    x, y = T(a, torch.float32), T(b, torch.float32)
    g = torch.ones(1, dtype=torch.float32, device="cuda")
    dx, dy = torch.empty_like(x), torch.empty_like(y)
    rc = lib.fa_cuda_ssim_backward(x.data_ptr(), y.data_ptr(), None, g.data_ptr(),
                                   _win().data_ptr(), 11, 1, 2, 30, 40, 0.5, 1e-4, 9e-4,
                                   None, dx.data_ptr(), dy.data_ptr(), 0, _st())
    assert rc == 0
    ox, oy = O.ssim_grad(a.astype(np.float64), b.astype(np.float64), data_range=1.0)
    assert np.abs(dx.double().cpu().numpy() - ox).max() < 1e-4 * np.abs(ox).max()
    assert np.abs(dy.double().cpu().numpy() - oy).max() < 1e-4 * np.abs(oy).max()


def test_gmsd_compat():
    lib = _cabi.load()
    a, b = baseline_pair((2, 3, 64, 80), 8.0, seed=5)
    x, y = T(a), T(b)
    bpp = ctypes.c_int(0)
    assert lib.fa_cuda_gmsd_workspace(64, 80, 1, ctypes.byref(bpp)) == 0
    ps = torch.empty((6, bpp.value), dtype=torch.float64, device="cuda")
    ps2 = torch.empty_like(ps)
    m = torch.empty(2, dtype=torch.float64, device="cuda")
    s = torch.empty(2, dtype=torch.float64, device="cuda")
    rc = lib.fa_cuda_gmsd(x.data_ptr(), y.data_ptr(), 0, 2, 3, 64, 80, 170.0,
                          (1e-6 * 255) ** 2, 1, ps.data_ptr(), ps2.data_ptr(), bpp.value,
                          m.data_ptr(), s.data_ptr(), 0, _st())
    assert rc == 0
    om, osd = O.gmsd(a, b, eps=(1e-6 * 255) ** 2)
    np.testing.assert_allclose(m.cpu().numpy(), om, atol=1e-6)
    np.testing.assert_allclose(s.cpu().numpy(), osd, atol=5e-6)

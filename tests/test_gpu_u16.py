"""uint16 input (10-16-bit video) read natively: exact integer MSE / L1, and
SSIM, MS-SSIM, GMSD and the fused SSIM+MSE pass against the float64 oracle
with data_range 65535 (the reference widens uint16 to float32 first,
functional.py:141-175)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu
L = 65535.0


def _pair(shape, sigma=2000.0, seed=0):
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:shape[-2], 0:shape[-1]].astype(np.float64)
    base = 30000 + 20000 * np.sin(xx / 13.0) * np.cos(yy / 17.0)
    a = np.clip(base + 3000 * rng.standard_normal(shape), 0, L).round().astype(np.uint16)
    b = np.clip(a + sigma * rng.standard_normal(shape), 0, L).round().astype(np.uint16)
    return a, b


def T(a):
    return torch.from_numpy(a.astype(np.int32)).to(torch.uint16).cuda()


@pytest.mark.parametrize("shape", [(2, 3, 64, 96), (1, 1, 37, 53), (3, 2, 120, 200)])
def test_mse_l1_exact(shape):
    a, b = _pair(shape)
    x, y = T(a), T(b)
    d = a.astype(np.int64) - b.astype(np.int64)
    per = x[0].numel()
    assert fa.mse(x, y, reduction="none").tolist() == [float(v) / per for v in
                                                        (d * d).reshape(shape[0], -1).sum(1)]
    assert fa.l1(x, y, reduction="none").tolist() == [float(v) / per for v in
                                                       np.abs(d).reshape(shape[0], -1).sum(1)]
    np.testing.assert_allclose(fa.psnr(x, y, reduction="none").cpu().numpy(),
                               O.psnr(a, b, data_range=L, reduction="none"), rtol=0, atol=1e-9)


@pytest.mark.parametrize("shape", [(2, 3, 64, 96), (1, 2, 45, 61), (1, 3, 140, 300)])
def test_ssim_gmsd(shape):
    a, b = _pair(shape, seed=1)
    x, y = T(a), T(b)
    np.testing.assert_allclose(fa.ssim(x, y, reduction="none").cpu().numpy(),
                               O.ssim(a, b, data_range=L, reduction="none"), rtol=0, atol=5e-6)
    _, osd = O.gmsd(a, b, data_range=L, eps=(1e-6 * L) ** 2)
    np.testing.assert_allclose(fa.gmsd(x, y, reduction="none").cpu().numpy(), osd,
                               rtol=0, atol=5e-6)


def test_ms_ssim_and_luma():
    a, b = _pair((2, 3, 200, 240), seed=2)
    x, y = T(a), T(b)
    np.testing.assert_allclose(fa.ms_ssim(x, y, reduction="none").cpu().numpy(),
                               O.ms_ssim(a, b, data_range=L, reduction="none"), rtol=0, atol=5e-6)
    np.testing.assert_allclose(fa.ssim(x, y, luma="bt709", reduction="none").cpu().numpy(),
                               O.ssim(a, b, data_range=L, luma="bt709", reduction="none"),
                               rtol=0, atol=5e-6)


def test_fused_metrics_exact_ssd():
    a, b = _pair((2, 3, 300, 500), seed=3)
    x, y = T(a), T(b)
    got = fa.metrics(x, y, ("mse", "psnr", "ssim"), reduction="none")
    assert torch.equal(got["mse"], fa.mse(x, y, reduction="none"))
    assert torch.equal(got["psnr"], fa.psnr(x, y, reduction="none"))
    assert torch.equal(got["ssim"], fa.ssim(x, y, reduction="none"))

"""PlaneScorer on the GPU: per-plane and luma metrics of packed planar frames
(uint8 4:2:0 and 10-bit uint16 4:2:0 read as they are) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O

from frame_analytics_b200 import planes

pytestmark = pytest.mark.gpu


def _frames(w, h, bits, seed):
    rng = np.random.default_rng(seed)
    n = h * w + 2 * (-(-h // 2)) * (-(-w // 2))
    hi = (1 << bits) - 1
    a = rng.integers(0, hi + 1, n)
    b = np.clip(a + np.round(rng.normal(0, 2 ** (bits - 6), n)), 0, hi)
    dt = np.uint8 if bits == 8 else np.uint16
    return a.astype(dt), b.astype(dt)


@pytest.mark.parametrize("bits", [8, 10])
def test_yuv420_scores_match_the_oracle(bits):
    w, h = 200, 190
    a, b = _frames(w, h, bits, seed=bits)
    ra = planes.frame_planes(torch.from_numpy(a).cuda(), w, h)
    rb = planes.frame_planes(torch.from_numpy(b).cuda(), w, h)
    sc = planes.PlaneScorer(["psnr", "mse", "ssim", "gmsd"], family="yuv", bits=bits)
    got = sc.scores(ra, rb)
    L = float((1 << bits) - 1)
    na = planes.frame_planes(torch.from_numpy(a.astype(np.int64)), w, h)
    nb = planes.frame_planes(torch.from_numpy(b.astype(np.int64)), w, h)
    for i, sfx in enumerate(("_y", "_cb", "_cr")):
        x, y = na[i].numpy().astype(np.float64), nb[i].numpy().astype(np.float64)
        mse = float(((x - y) ** 2).mean())
        assert got["mse" + sfx] == mse  # exact integer sums
        assert abs(got["psnr" + sfx] - 10 * np.log10(L * L / mse)) < 1e-9
    x, y = na[0].numpy(), nb[0].numpy()
    assert abs(got["float_ssim"] - O.ssim(x, y, data_range=L)) < 5e-6
    _, sd = O.gmsd(x, y, data_range=L, eps=(1e-6 * L) ** 2)
    assert abs(got["gmsd"] - float(sd[0])) < 5e-6


def test_rgb_planes_score_ssimulacra2_and_ssim():
    """Planar RGB frames: the image features see all three channels."""
    w, h = 96, 64
    rng = np.random.default_rng(3)
    a = rng.integers(0, 256, 3 * h * w).astype(np.uint8)
    b = np.clip(a.astype(np.int16) + rng.integers(-6, 7, a.shape), 0, 255).astype(np.uint8)
    ra = planes.frame_planes(torch.from_numpy(a).cuda(), w, h, "rgbp")
    rb = planes.frame_planes(torch.from_numpy(b).cuda(), w, h, "rgbp")
    got = planes.PlaneScorer(["ssim", "ssimulacra2", "psnr"], family="rgb").scores(ra, rb)
    x = a.reshape(1, 3, h, w)
    y = b.reshape(1, 3, h, w)
    assert abs(got["float_ssim"] - O.ssim(x, y)) < 5e-6
    assert abs(got["ssimulacra2"] - O.ssimulacra2(x[0], y[0], 255.0)) < 5e-3
    assert set(got) == {"float_ssim", "ssimulacra2", "psnr_r", "psnr_g", "psnr_b"}


def test_yuv422_and_444_views_score_each_plane():
    for layout, (cw, ch) in (("yuv422p", (2, 1)), ("yuv444p", (1, 1))):
        w, h = 64, 48
        n = h * w + 2 * (h // ch) * (w // cw)
        rng = np.random.default_rng(cw)
        a = rng.integers(0, 256, n).astype(np.uint8)
        b = np.clip(a.astype(np.int16) + rng.integers(-5, 6, n), 0, 255).astype(np.uint8)
        ra = planes.frame_planes(torch.from_numpy(a).cuda(), w, h, layout)
        rb = planes.frame_planes(torch.from_numpy(b).cuda(), w, h, layout)
        got = planes.PlaneScorer(["mse"], family="yuv").scores(ra, rb)
        na = planes.frame_planes(torch.from_numpy(a.astype(np.int64)), w, h, layout)
        nb = planes.frame_planes(torch.from_numpy(b.astype(np.int64)), w, h, layout)
        for i, sfx in enumerate(("_y", "_cb", "_cr")):
            d = (na[i] - nb[i]).double()
            assert got["mse" + sfx] == float((d * d).mean())

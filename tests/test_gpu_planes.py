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

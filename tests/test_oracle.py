"""The CPU oracle against the reference's own outputs (tests/golden/golden.npz).

Pins oracle/fa_oracle.py before any GPU result is compared with it."""

from __future__ import annotations

import numpy as np
import pytest

import fa_oracle as O
from conftest import REPO

GOLDEN_DIR = REPO / "tests" / "golden"

V = ["v0", "v1", "v2", "v3"]
M = ["m0", "m1", "m2"]
EPS_G = (1e-6 * 255.0) ** 2


@pytest.mark.parametrize("k", V)
def test_ssim_scalar_and_map(golden, k):
    a, b = golden[f"{k}_a"], golden[f"{k}_b"]
    assert abs(O.ssim(a, b) - golden[f"{k}_ssim"]) < 1e-12
    if f"{k}_map" in golden:
        m = O.ssim(a, b, return_map=True)[0, 0]
        assert np.abs(m - golden[f"{k}_map"]).max() < 1e-12
    for ksz in (3, 5, 7, 9):
        assert abs(O.ssim(a, b, win_size=ksz) - golden[f"{k}_ssim_k{ksz}"]) < 1e-12
    # the reference CPU library agrees with its float64 oracle
    assert abs(golden[f"{k}_cpu_ssim"] - golden[f"{k}_ssim"]) < 5e-6


@pytest.mark.parametrize("k", V)
def test_pixel_reductions(golden, k):
    a, b = golden[f"{k}_a"], golden[f"{k}_b"]
    assert O.pixel(a, b, "mse") == pytest.approx(float(golden[f"{k}_mse"]), rel=1e-14, abs=1e-14)
    assert O.psnr(a, b) == pytest.approx(float(golden[f"{k}_psnr"]), rel=1e-13)
    assert O.pixel(a, b, "l1") == pytest.approx(float(golden[f"{k}_l1"]), rel=1e-14, abs=1e-14)
    assert O.pixel(a, b, "charbonnier", 1e-3) == pytest.approx(float(golden[f"{k}_charb"]), rel=1e-13)
    assert O.pixel(a, b, "charbonnier", 2.0) == pytest.approx(float(golden[f"{k}_charb2"]), rel=1e-13)
    assert O.pixel(a, b, "huber", 1.0) == pytest.approx(float(golden[f"{k}_huber"]), rel=1e-13, abs=1e-15)
    assert O.pixel(a, b, "huber", 3.0) == pytest.approx(float(golden[f"{k}_huber3"]), rel=1e-13, abs=1e-15)
    ssd = int(O.ssd_uint8(a, b)[0])
    assert ssd / a.size == float(golden[f"{k}_mse"])


@pytest.mark.parametrize("k", V)
def test_gmsd_single_plane(golden, k):
    a, b = golden[f"{k}_a"], golden[f"{k}_b"]
    _, s = O.gmsd(a, b, eps=EPS_G)
    assert abs(s[0] - golden[f"{k}_gmsd"]) < 1e-12
    _, s = O.gmsd(a, b, eps=EPS_G, downsample=False)
    assert abs(s[0] - golden[f"{k}_gmsd_nodown"]) < 1e-12


@pytest.mark.parametrize("k", M)
def test_ms_ssim_gmsd_losses(golden, k):
    a, b = golden[f"{k}_a"], golden[f"{k}_b"]
    assert abs(O.ms_ssim(a, b) - golden[f"{k}_ms_ssim"]) < 1e-12
    assert abs(O.gmsd(a, b, eps=EPS_G)[1][0] - golden[f"{k}_gmsd"]) < 1e-12
    assert O.pixel(a, b, "l1") == pytest.approx(float(golden[f"{k}_l1"]), rel=1e-14)
    assert O.pixel(a, b, "charbonnier", 1e-3) == pytest.approx(float(golden[f"{k}_charb"]), rel=1e-13)
    assert O.pixel(a, b, "huber", 1.0) == pytest.approx(float(golden[f"{k}_huber"]), rel=1e-13)


@pytest.mark.parametrize("mode", ["bt601", "bt709", "matlab"])
@pytest.mark.parametrize("cb", [0, 4])
def test_luma_crop(golden, mode, cb):
    a, b = golden["luma_a"][None], golden["luma_b"][None]
    assert abs(O.ssim(a, b, luma=mode, crop_border=cb) - golden[f"luma_{mode}_{cb}_ssim"]) < 1e-12
    assert O.psnr(a, b, luma=mode, crop_border=cb) == pytest.approx(
        float(golden[f"luma_{mode}_{cb}_psnr"]), rel=1e-12)


@pytest.mark.parametrize("down", [1, 0])
def test_multichannel_gmsd_pooling(golden, down):
    """Channels pooled jointly per image, as the reference CPU library does."""
    m, s = O.gmsd(golden["gm3_a"], golden["gm3_b"], downsample=bool(down), eps=EPS_G)
    np.testing.assert_allclose(m, golden[f"gm3_cpu_mean_d{down}"], atol=2e-7)
    np.testing.assert_allclose(s, golden[f"gm3_cpu_std_d{down}"], atol=2e-7)


def test_config0_and_config1_generators(golden):
    from conftest import baseline_pair

    a, b = baseline_pair((1, 3, 512, 512), 8.0, seed=0)
    assert int(a.astype(np.int64).sum()) == int(golden["cfg0_a_sum"])
    assert abs(O.ssim(a, b) - float(golden["cfg0_ssim"])) < 1e-12
    assert abs(float(golden["cfg0_cpu_ssim"]) - float(golden["cfg0_ssim"])) < 5e-6


def test_ssim_grad_matches_finite_differences():
    """The oracle's analytic SSIM gradient against central differences."""
    rng = np.random.default_rng(7)
    x = rng.random((1, 2, 17, 19))
    y = np.clip(x + 0.05 * rng.standard_normal(x.shape), 0, 1)
    dx, dy = O.ssim_grad(x, y, data_range=1.0)
    h = 1e-6
    for (c, i, j) in [(0, 3, 4), (1, 8, 9), (0, 16, 18), (1, 0, 0), (0, 10, 2)]:
        for arr, g in ((x, dx), (y, dy)):
            p = arr.copy(); p[0, c, i, j] += h
            m = arr.copy(); m[0, c, i, j] -= h
            if arr is x:
                fd = (O.ssim(p, y, data_range=1.0) - O.ssim(m, y, data_range=1.0)) / (2 * h)
            else:
                fd = (O.ssim(x, p, data_range=1.0) - O.ssim(x, m, data_range=1.0)) / (2 * h)
            assert abs(g[0, c, i, j] - fd) <= 1e-6 * max(1.0, abs(fd)) + 1e-9


@pytest.mark.parametrize("f", [2, 3, 4])
def test_matlab_downsample_pinned(golden, f):
    """The oracle's MATLAB-mode downsample equals the reference's own
    (functional.py:575-586, run by make_golden.py)."""
    x = golden["mdown_x"].astype(np.float64)
    # the reference computes in float32: relative agreement to a few float32 ulp
    np.testing.assert_allclose(O.matlab_downsample(x, f), golden[f"mdown_f{f}"], rtol=1e-6, atol=0)


S2 = ["s0", "s1", "s2", "s3", "r0", "g0"]


@pytest.mark.parametrize("k", S2)
def test_ssimulacra2_oracle_matches_the_reference(k):
    """tests/golden/ssimulacra2.npz holds scores of the reference's float64
    transcription of libjxl (recursive Gaussian run as a recursion); the
    oracle convolves the FIR taps instead and must agree to float64 noise."""
    d = np.load(GOLDEN_DIR / "ssimulacra2.npz")
    a, b = d[f"{k}_a"], d[f"{k}_b"]
    if a.shape[0] == 1:
        a, b = np.repeat(a, 3, axis=0), np.repeat(b, 3, axis=0)
    assert abs(O.ssimulacra2(a, b, 255.0) - float(d[f"{k}_ref64"])) < 1e-8
    assert abs(float(d[f"{k}_torch64"]) - float(d[f"{k}_ref64"])) < 1e-8


def test_ssimulacra2_taps_sum_to_one():
    t = O.recursive_gaussian_taps(1.5)
    assert len(t) == 11 and abs(t.sum() - 1.0) < 1e-12 and abs(t[0]) < 1e-15

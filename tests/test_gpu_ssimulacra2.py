"""SSIMULACRA 2 on the GPU against the reference: the float64 transcription of
libjxl (reference.py) and the reference's own torch path, on the pairs of
tests/golden/ssimulacra2.npz.  Bars: float32 pipeline within 5e-3 of the
float64 reference (the reference's own bar, 3e-2 on gray input), float64
pipeline within 1e-8 (tests/test_ssimulacra2.py of the reference)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import REPO

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu
G = np.load(REPO / "tests" / "golden" / "ssimulacra2.npz")
CASES = ["s0", "s1", "s2", "s3", "r0", "g0"]


def _t(k, which, dt=torch.uint8):
    return torch.as_tensor(G[f"{k}_{which}"], dtype=dt, device="cuda")


@pytest.mark.parametrize("k", CASES)
def test_matches_reference(k):
    x, y = _t(k, "a"), _t(k, "b")
    want = float(G[f"{k}_ref64"])
    tol = 3e-2 if k == "g0" else 5e-3
    assert abs(float(fa.ssimulacra2(x, y, data_range=255.0)) - want) < tol
    assert abs(float(fa.ssimulacra2(x, y, data_range=255.0, dtype=torch.float64)) - want) < 1e-8
    # and close to the reference's own float32 torch result
    assert abs(float(fa.ssimulacra2(x, y, data_range=255.0)) - float(G[f"{k}_torch32"])) < tol


def test_identical_is_100_and_order_matters():
    x, y = _t("s0", "a"), _t("s0", "b")
    assert float(fa.ssimulacra2(x, x, data_range=255.0)) == 100.0
    assert float(fa.ssimulacra2(x, y, data_range=255.0)) != float(fa.ssimulacra2(y, x, data_range=255.0))


def test_batch_reduction_dtypes_and_crop():
    a = np.stack([G["s0_a"], G["r0_a"][:, :64, :72]])
    b = np.stack([G["s0_b"], G["r0_b"][:, :64, :72]])
    x = torch.as_tensor(a, device="cuda")
    y = torch.as_tensor(b, device="cuda")
    per = fa.ssimulacra2(x, y, data_range=255.0, reduction="none")
    assert per.shape == (2,)
    assert abs(float(fa.ssimulacra2(x, y, data_range=255.0)) - float(per.mean())) < 1e-12
    for i in range(2):
        assert abs(float(fa.ssimulacra2(x[i], y[i], data_range=255.0)) - float(per[i])) < 1e-9
        assert abs(float(per[i]) - O.ssimulacra2(a[i], b[i], 255.0)) < 5e-3
    f32 = fa.ssimulacra2(x.float() / 255.0, y.float() / 255.0, reduction="none")
    assert float((f32 - per).abs().max()) < 2e-3
    got = float(fa.ssimulacra2(x, y, data_range=255.0, crop_border=4))
    want = float(fa.ssimulacra2(x[..., 4:-4, 4:-4].contiguous(), y[..., 4:-4, 4:-4].contiguous(),
                                data_range=255.0))
    assert abs(got - want) < 1e-9
    assert float(fa.SSIMULACRA2(data_range=255.0)(x, y)) == float(fa.ssimulacra2(x, y, data_range=255.0))
    with pytest.raises(ValueError):
        fa.ssimulacra2(x[..., :7, :], y[..., :7, :], data_range=255.0)
    with pytest.raises(ValueError):
        fa.ssimulacra2(x[:, :2], y[:, :2], data_range=255.0)


def test_monotone_in_distortion():
    a = G["s0_a"].astype(np.float64)
    rng = np.random.default_rng(5)
    mild = np.clip(a + 3 * rng.standard_normal(a.shape), 0, 255).round()
    harsh = np.clip(a + 30 * rng.standard_normal(a.shape), 0, 255).round()
    x = torch.as_tensor(a, dtype=torch.uint8, device="cuda")
    s = [float(fa.ssimulacra2(x, torch.as_tensor(v, dtype=torch.uint8, device="cuda"),
                              data_range=255.0)) for v in (mild, harsh)]
    assert s[0] > s[1]


def test_uint16_strided_and_gray_inputs():
    """16-bit input (data_range 65535), a strided crop view, and a 1-channel
    frame (replicated through a zero channel stride) all match the oracle."""
    a, b = G["s0_a"].astype(np.float64), G["s0_b"].astype(np.float64)
    x16 = torch.as_tensor((a * 257).astype(np.uint16), device="cuda")
    y16 = torch.as_tensor((b * 257).astype(np.uint16), device="cuda")
    want = float(G["s0_ref64"])
    assert abs(float(fa.ssimulacra2(x16, y16, data_range=65535.0)) - want) < 5e-3
    big = torch.zeros((3, 80, 96), dtype=torch.uint8, device="cuda")
    big2 = big.clone()
    big[:, 5:69, 7:79] = _t("s0", "a")
    big2[:, 5:69, 7:79] = _t("s0", "b")
    view_x, view_y = big[:, 5:69, 7:79], big2[:, 5:69, 7:79]
    assert not view_x.is_contiguous()
    assert abs(float(fa.ssimulacra2(view_x, view_y, data_range=255.0, dtype=torch.float64))
               - want) < 1e-8
    g_ref = float(G["g0_ref64"])
    assert abs(float(fa.ssimulacra2(_t("g0", "a"), _t("g0", "b"), data_range=255.0,
                                    dtype=torch.float64)) - g_ref) < 1e-8

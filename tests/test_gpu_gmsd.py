"""GMSD / GMS on the GPU against the reference's goldens and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import baseline_pair

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu
EPS_G = (1e-6 * 255.0) ** 2


def T(a, dt=torch.uint8):
    return torch.as_tensor(np.asarray(a), dtype=dt, device="cuda")


@pytest.mark.parametrize("k", ["v0", "v1", "v2", "v3", "m0", "m1", "m2"])
@pytest.mark.parametrize("dt", [torch.uint8, torch.float32])
def test_gmsd_matches_golden(golden, k, dt):
    a, b = T(golden[f"{k}_a"], dt), T(golden[f"{k}_b"], dt)
    assert abs(float(fa.gmsd(a, b, data_range=255.0)) - float(golden[f"{k}_gmsd"])) < 5e-6
    if f"{k}_gmsd_nodown" in golden:
        got = float(fa.gmsd(a, b, data_range=255.0, downsample=False))
        assert abs(got - float(golden[f"{k}_gmsd_nodown"])) < 5e-6


@pytest.mark.parametrize("down", [1, 0])
def test_multichannel_pooling(golden, down):
    a, b = T(golden["gm3_a"]), T(golden["gm3_b"])
    m = fa.gms(a, b, downsample=bool(down), reduction="none").cpu().numpy()
    s = fa.gmsd(a, b, downsample=bool(down), reduction="none").cpu().numpy()
    np.testing.assert_allclose(m, golden[f"gm3_cpu_mean_d{down}"], atol=1e-6)
    np.testing.assert_allclose(s, golden[f"gm3_cpu_std_d{down}"], atol=1e-6)


@pytest.mark.parametrize("shape", [(1, 1, 6, 6), (1, 1, 7, 1031), (2, 3, 1031, 9),
                                   (1, 2, 517, 1029), (3, 1, 64, 1024)])
@pytest.mark.parametrize("down", [True, False])
def test_shapes_vs_oracle(shape, down):
    a, b = baseline_pair(shape, 13.0, seed=shape[-1])
    m, s = O.gmsd(a, b, downsample=down, eps=EPS_G)
    np.testing.assert_allclose(fa.gms(T(a), T(b), downsample=down, reduction="none").cpu().numpy(), m, atol=1e-6)
    np.testing.assert_allclose(fa.gmsd(T(a), T(b), downsample=down, reduction="none").cpu().numpy(), s, atol=5e-6)


@pytest.mark.parametrize("h", [64, 66, 68, 70, 300])
def test_register_kernel_row_remainders(h):
    """uint8 pooled frames with W % 8 == 0 take the register-streaming kernel;
    these heights give every remainder of its four-row loop (and several
    chunks at 300), two planes wide enough for a partial last strip."""
    a, b = baseline_pair((2, 1, h, 1000), 11.0, seed=h)
    m, s = O.gmsd(a, b, downsample=True, eps=EPS_G)
    np.testing.assert_allclose(fa.gms(T(a), T(b), reduction="none").cpu().numpy(), m, atol=1e-6)
    np.testing.assert_allclose(fa.gmsd(T(a), T(b), reduction="none").cpu().numpy(), s, atol=5e-6)


def test_map_and_identity():
    a, b = baseline_pair((2, 3, 50, 61), 8.0, seed=3)
    q = fa.gms(T(a), T(b), return_map=True)
    assert tuple(q.shape) == (2, 3, 23, 28)
    np.testing.assert_allclose(q.double().cpu().numpy(), O.gms_map(a, b), atol=1e-6)
    x = T(a)
    assert float(fa.gmsd(x, x)) < 1e-6
    assert abs(float(fa.gms(x, x)) - 1.0) < 1e-7


def test_luma_and_crop():
    a, b = baseline_pair((2, 3, 90, 70), 10.0, seed=6)
    m, s = O.gmsd(a, b, luma="bt709", crop_border=3, eps=EPS_G)
    np.testing.assert_allclose(fa.gmsd(T(a), T(b), luma="bt709", crop_border=3,
                                       reduction="none").cpu().numpy(), s, atol=5e-6)


def _torch_gms_stats(x, y, T, eps, down):
    """float64 torch restatement of reference.gmsd_reference for gradients."""
    import torch.nn.functional as F

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
@pytest.mark.parametrize("shape", [(2, 3, 41, 53), (1, 1, 70, 97)])
def test_gms_gmsd_gradients(down, shape):
    torch.manual_seed(1)
    a = torch.rand(shape, device="cuda", dtype=torch.float64)
    b = (a + 0.1 * torch.randn_like(a)).clamp(0, 1)
    # the float64 reference differentiates at exactly the float32 inputs
    a, b = a.float().double(), b.float().double()
    T, eps = 170.0 / 255 ** 2, 1e-12
    x = a.float().requires_grad_()
    y = b.float().requires_grad_()
    w1 = torch.randn(shape[0], device="cuda", dtype=torch.float64)
    w2 = torch.randn(shape[0], device="cuda", dtype=torch.float64)
    m = fa.gms(x, y, data_range=1.0, downsample=down, reduction="none")
    s = fa.gmsd(x, y, data_range=1.0, downsample=down, reduction="none")
    gx, gy = torch.autograd.grad((m * w1).sum() + (s * w2).sum(), (x, y))
    xr, yr = a.clone().requires_grad_(), b.clone().requires_grad_()
    mr, sr = _torch_gms_stats(xr, yr, T, (1e-6) ** 2, down)
    rx, ry = torch.autograd.grad((mr * w1).sum() + (sr * w2).sum(), (xr, yr))
    for got, want in ((gx, rx), (gy, ry)):
        err = float((got.double() - want).abs().max() / want.abs().max())
        assert err < 1e-4, err


def test_gmsd_module_loss_backward():
    torch.manual_seed(2)
    a = torch.rand(2, 3, 64, 80, device="cuda")
    p = (a + 0.05 * torch.randn_like(a)).clamp(0, 1).requires_grad_()
    loss = fa.GMSD(data_range=1.0).loss(p, a)
    loss.backward()
    assert p.grad is not None and torch.isfinite(p.grad).all() and float(p.grad.abs().max()) > 0
    assert abs(float(loss.detach()) - (1 - float(fa.gms(p.detach(), a, data_range=1.0)))) < 1e-12

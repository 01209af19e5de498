"""Pixel reductions on the GPU against the oracle and the reference's goldens."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import baseline_pair

import frame_analytics_b200 as fa
from frame_analytics_b200 import backend

pytestmark = pytest.mark.gpu
V = ["v0", "v1", "v2", "v3"]


def T(a, dt=torch.uint8):
    return torch.as_tensor(np.asarray(a), dtype=dt, device="cuda")


@pytest.mark.parametrize("k", V)
def test_uint8_matches_golden(golden, k):
    a, b = T(golden[f"{k}_a"]), T(golden[f"{k}_b"])
    assert float(fa.mse(a, b)) == float(golden[f"{k}_mse"])            # exact
    want_p = float(golden[f"{k}_psnr"])
    got_p = float(fa.psnr(a, b))
    assert (math.isinf(want_p) and math.isinf(got_p)) or abs(got_p - want_p) < 1e-6
    assert abs(float(fa.l1(a, b)) - float(golden[f"{k}_l1"])) < 1e-12    # exact sum
    assert abs(float(fa.charbonnier(a, b)) - float(golden[f"{k}_charb"])) < 1e-6
    assert abs(float(fa.charbonnier(a, b, eps=2.0)) - float(golden[f"{k}_charb2"])) < 1e-6
    assert abs(float(fa.huber(a, b)) - float(golden[f"{k}_huber"])) < 1e-6
    assert abs(float(fa.huber(a, b, delta=3.0)) - float(golden[f"{k}_huber3"])) < 1e-6


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_float_dtypes(golden, dt):
    a, b = golden["v1_a"], golden["v1_b"]
    x, y = T(a, dt), T(b, dt)
    assert abs(float(fa.mse(x, y)) - float(golden["v1_mse"])) < 1e-9 * float(golden["v1_mse"]) + 1e-9
    assert abs(float(fa.psnr(x, y, data_range=255.0)) - float(golden["v1_psnr"])) < 1e-6
    assert abs(float(fa.l1(x, y)) - float(golden["v1_l1"])) < 1e-6
    assert abs(float(fa.charbonnier(x, y)) - float(golden["v1_charb"])) < 1e-6
    assert abs(float(fa.huber(x, y)) - float(golden["v1_huber"])) < 1e-6


def test_config1_exact_ssd_full_size(golden):
    """uint8 8x3x1080x1920: per-image integer SSD bit-exact, PSNR to 1e-9."""
    a, b = baseline_pair((8, 3, 1080, 1920), 5.0, seed=0)
    x, y = T(a), T(b)
    out, isum = backend.pixel(x, y, op=backend.OP_MSE, per_image=True, want_isum=True)
    np.testing.assert_array_equal(isum.cpu().numpy(), golden["cfg1_ssd"])
    n = 3 * 1080 * 1920
    np.testing.assert_array_equal(out.cpu().numpy(), golden["cfg1_ssd"] / n)
    tot = float(golden["cfg1_ssd"].sum()) / (8 * n)
    assert float(fa.mse(x, y)) == tot
    assert abs(float(fa.psnr(x, y)) - 10 * math.log10(255.0 ** 2 / tot)) < 1e-9


@pytest.mark.parametrize("offset", [0, 1, 2, 3, 5, 13])
@pytest.mark.parametrize("fn", [fa.mse, fa.l1, fa.huber, fa.charbonnier])
def test_unaligned_uint8_views(fn, offset):
    n = 64 * 33
    g = torch.Generator(device="cuda").manual_seed(offset)
    a = torch.randint(0, 256, (n + 16,), dtype=torch.uint8, device="cuda", generator=g)
    b = torch.randint(0, 256, (n + 16,), dtype=torch.uint8, device="cuda", generator=g)
    x = a[offset:offset + n].view(1, 1, 33, 64)
    y = b[offset:offset + n].view(1, 1, 33, 64)
    got = float(fn(x, y))
    name = {fa.mse: "mse", fa.l1: "l1", fa.huber: "huber", fa.charbonnier: "charbonnier"}[fn]
    param = {"mse": 0.0, "l1": 0.0, "huber": 1.0, "charbonnier": 1e-3}[name]
    want = O.pixel(x.cpu().numpy(), y.cpu().numpy(), name, param)
    assert abs(got - want) < 1e-6 * max(1.0, abs(want))


def test_mismatched_alignment_of_a_and_b():
    a = torch.randint(0, 256, (4100,), dtype=torch.uint8, device="cuda")
    b = torch.randint(0, 256, (4100,), dtype=torch.uint8, device="cuda")
    x, y = a[1:4097].view(1, 1, 64, 64), b[3:4099].view(1, 1, 64, 64)
    assert float(fa.mse(x, y)) == O.pixel(x.cpu().numpy(), y.cpu().numpy(), "mse")


@pytest.mark.parametrize("fn,kw,want", [("mse", {}, 1e-12), ("huber", {}, 5e-13),
                                         ("l1", {}, 1e-6), ("charbonnier", {"eps": 0.0}, 1e-6)])
def test_float64_input_is_not_narrowed(fn, kw, want):
    x = torch.full((1, 1, 64, 64), 100.0, dtype=torch.float64, device="cuda")
    y = x + 1e-6
    got = float(getattr(fa, fn)(x, y, **kw))
    assert abs(got - want) <= 1e-3 * want


def test_reduction_none_and_batch_mean():
    a, b = baseline_pair((5, 3, 37, 53), 9.0, seed=4)
    x, y = T(a), T(b)
    per = fa.mse(x, y, reduction="none").cpu().numpy()
    np.testing.assert_array_equal(per, O.pixel(a, b, "mse", reduction="none"))
    assert float(fa.mse(x, y)) == O.pixel(a, b, "mse")
    p = fa.psnr(x, y, reduction="none").cpu().numpy()
    np.testing.assert_allclose(p, O.psnr(a, b, reduction="none"), atol=1e-9)
    for name, fn, param in [("l1", fa.l1, 0.0), ("huber", fa.huber, 1.0)]:
        np.testing.assert_allclose(fn(x, y, reduction="none").cpu().numpy(),
                                   O.pixel(a, b, name, param, reduction="none"), atol=1e-9)


def test_identities():
    a, _ = baseline_pair((2, 3, 40, 50), 5.0, seed=1)
    x = T(a)
    assert float(fa.mse(x, x)) == 0.0
    assert math.isinf(float(fa.psnr(x, x)))
    assert float(fa.l1(x, x)) == 0.0 and float(fa.huber(x, x)) == 0.0
    assert abs(float(fa.charbonnier(x, x, eps=0.25)) - 0.25) < 1e-9
    assert abs(float(fa.psnr(x, x, eps=1e-10)) - (10 * math.log10(255.0 ** 2) + 100)) < 1e-9


@pytest.mark.parametrize("mode", ["bt601", "bt709", "matlab"])
@pytest.mark.parametrize("cb", [0, 4])
def test_luma_crop_psnr(golden, mode, cb):
    a, b = T(golden["luma_a"])[None], T(golden["luma_b"])[None]
    got = float(fa.psnr(a, b, data_range=255.0, luma=mode, crop_border=cb))
    assert abs(got - float(golden[f"luma_{mode}_{cb}_psnr"])) < 1e-6


@pytest.mark.parametrize("dt", [torch.uint8, torch.float32])
def test_luma_crop_all_ops_vs_oracle(dt):
    a, b = baseline_pair((3, 3, 45, 67), 11.0, seed=9)
    x, y = T(a, dt), T(b, dt)
    for name, fn, kw, par in [("mse", fa.mse, {}, 0.0), ("l1", fa.l1, {}, 0.0),
                              ("charbonnier", fa.charbonnier, {"eps": 0.5}, 0.5),
                              ("huber", fa.huber, {"delta": 2.0}, 2.0)]:
        got = fn(x, y, luma="matlab", crop_border=3, reduction="none", **kw).cpu().numpy()
        want = O.pixel(a, b, name, par, reduction="none", luma="matlab", crop_border=3)
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-9)
        got = fn(x, y, crop_border=2, **kw)
        assert abs(float(got) - O.pixel(a, b, name, par, crop_border=2)) < 1e-6


@pytest.mark.parametrize("name,param", [("mse", 0.0), ("l1", 0.0), ("charbonnier", 0.3),
                                        ("huber", 0.5)])
@pytest.mark.parametrize("luma", [None, "bt709"])
def test_pixel_loss_gradients(name, param, luma):
    torch.manual_seed(0)
    x = torch.rand(2, 3, 19, 23, device="cuda", dtype=torch.float64, requires_grad=True)
    y = torch.rand(2, 3, 19, 23, device="cuda", dtype=torch.float64, requires_grad=True)
    fn = {"mse": fa.mse, "l1": fa.l1, "charbonnier": fa.charbonnier, "huber": fa.huber}[name]
    kw = {"charbonnier": {"eps": param}, "huber": {"delta": param}}.get(name, {})
    out = fn(x, y, luma=luma, reduction="none", **kw)
    w = torch.tensor([0.3, -1.7], dtype=torch.float64, device="cuda")
    gx, gy = torch.autograd.grad((out * w).sum(), (x, y))
    # float64 torch reference of the same penalty
    xr, yr = x.detach().clone().requires_grad_(), y.detach().clone().requires_grad_()
    xa, ya = xr, yr
    if luma:
        k = fa.LUMA_COEFFS[luma]
        xa = k[0] * xr[:, 0:1] + k[1] * xr[:, 1:2] + k[2] * xr[:, 2:3]
        ya = k[0] * yr[:, 0:1] + k[1] * yr[:, 1:2] + k[2] * yr[:, 2:3]
    d = xa - ya
    t = {"mse": d * d, "l1": d.abs(), "charbonnier": torch.sqrt(d * d + param ** 2),
         "huber": torch.where(d.abs() <= param, 0.5 * d * d, param * (d.abs() - 0.5 * param))}[name]
    ref = t.flatten(1).mean(1)
    rx, ry = torch.autograd.grad((ref * w).sum(), (xr, yr))
    torch.testing.assert_close(gx, rx, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(gy, ry, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("op", ["mse", "l1", "charbonnier", "huber"])
@pytest.mark.parametrize("reduction", ["mean", "none"])
@pytest.mark.parametrize("shape", [(2, 3, 40, 64), (3, 1, 17, 23)])
def test_fused_pixel_loss_grad_matches_two_pass(op, reduction, shape):
    """A float32 pixel loss with gradient from one read equals the reduction
    followed by the separate backward kernel (vector and scalar paths)."""
    fn = getattr(fa, op)
    g = torch.Generator().manual_seed(2)
    a = torch.rand(shape, generator=g).cuda()
    b = torch.rand(shape, generator=g).cuda()
    up = torch.randn(shape[0], generator=g, dtype=torch.float64).cuda() if reduction == "none" else None
    res = {}
    for fused in (True, False):
        fa.set_fused_loss_grad(fused)
        try:
            x = a.clone().requires_grad_(True)
            y = b.clone().requires_grad_(True)
            v = fn(x, y, reduction=reduction)
            (v.sum() if up is None else (v * up).sum()).backward()
            res[fused] = (v.detach(), x.grad, y.grad)
        finally:
            fa.set_fused_loss_grad(True)
    (v1, gx1, gy1), (v0, gx0, gy0) = res[True], res[False]
    # MSE sums every float term in float64 on both paths; for the other
    # penalties the forward kernel adds four float terms before going to
    # float64, the fused one adds each: ~1e-8 relative
    rtol = 1e-12 if op == "mse" else 1e-7
    torch.testing.assert_close(v1, v0, rtol=rtol, atol=1e-15)
    torch.testing.assert_close(v1, fn(a, b, reduction=reduction), rtol=rtol, atol=1e-15)
    for g1, g0 in ((gx1, gx0), (gy1, gy0)):
        torch.testing.assert_close(g1, g0, rtol=1e-6, atol=1e-6 * float(g0.abs().max()))


def test_fused_pixel_loss_second_backward():
    g = torch.Generator().manual_seed(3)
    a = torch.rand((2, 3, 32, 48), generator=g).cuda()
    y = torch.rand((2, 3, 32, 48), generator=g).cuda().requires_grad_(True)
    loss = fa.mse(a, y)
    loss.backward(retain_graph=True)
    first = y.grad.clone()
    loss.backward()
    torch.testing.assert_close(y.grad, 2 * first, rtol=1e-6, atol=1e-12)
    torch.testing.assert_close(first, 2 * (y.detach() - a) / a.numel(), rtol=1e-5, atol=1e-12)

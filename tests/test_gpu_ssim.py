"""SSIM / MS-SSIM forward and backward on the GPU against the oracle and the
reference's goldens.  Tolerances are the reference's own (validate.py:24-26,
test_metrics.py:130-171): SSIM scalar 5e-6, map 5e-5, gradients 1e-4 relative."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import baseline_pair, natural_pair

import frame_analytics_b200 as fa

pytestmark = pytest.mark.gpu
V = ["v0", "v1", "v2", "v3"]
TOL_SSIM, TOL_MAP = 5e-6, 5e-5


def T(a, dt=torch.uint8):
    return torch.as_tensor(np.asarray(a), dtype=dt, device="cuda")


@pytest.mark.parametrize("k", V)
@pytest.mark.parametrize("dt", [torch.uint8, torch.float32, torch.float16, torch.float64])
def test_ssim_matches_golden(golden, k, dt):
    a, b = T(golden[f"{k}_a"], dt), T(golden[f"{k}_b"], dt)
    assert abs(float(fa.ssim(a, b, data_range=255.0)) - float(golden[f"{k}_ssim"])) < TOL_SSIM
    if f"{k}_map" in golden:
        m = fa.ssim(a, b, data_range=255.0, return_map=True)[0, 0].double().cpu().numpy()
        assert np.abs(m - golden[f"{k}_map"]).max() < TOL_MAP
    for ksz in (3, 5, 7, 9):
        got = float(fa.ssim(a, b, data_range=255.0, win_size=ksz))
        assert abs(got - float(golden[f"{k}_ssim_k{ksz}"])) < TOL_SSIM


def test_config0(golden):
    a, b = baseline_pair((1, 3, 512, 512), 8.0, seed=0)
    assert abs(float(fa.ssim(T(a), T(b))) - float(golden["cfg0_ssim"])) < 1e-6


def test_input_ranks_agree():
    a, b = natural_pair()
    x, y = T(a), T(b)
    v2 = float(fa.ssim(x, y, data_range=255.0))
    assert v2 == float(fa.ssim(x[None], y[None], data_range=255.0))
    assert v2 == float(fa.ssim(x[None, None], y[None, None], data_range=255.0))


def test_batch_channels_and_reduction_none():
    a, b = baseline_pair((3, 2, 70, 90), 10.0, seed=2)
    x, y = T(a), T(b)
    per = fa.ssim(x, y, reduction="none").cpu().numpy()
    np.testing.assert_allclose(per, O.ssim(a, b, reduction="none"), atol=TOL_SSIM)
    assert abs(float(fa.ssim(x, y)) - O.ssim(a, b)) < TOL_SSIM
    m = fa.ssim(x, y, return_map=True)
    assert tuple(m.shape) == (3, 2, 60, 80)
    np.testing.assert_allclose(m.double().cpu().numpy(), O.ssim(a, b, return_map=True), atol=TOL_MAP)
    assert abs(float(m.double().mean()) - O.ssim(a, b)) < TOL_SSIM


@pytest.mark.parametrize("shape", [(1, 1, 11, 11), (1, 1, 12, 400), (2, 1, 400, 13),
                                   (1, 2, 353, 17), (1, 1, 700, 353), (1, 1, 365, 365)])
@pytest.mark.parametrize("ksz", [11, 3])
def test_odd_shapes_and_strip_edges(shape, ksz):
    """Sizes at and around the kernels' strip and chunk boundaries."""
    a, b = baseline_pair(shape, 15.0, seed=sum(shape))
    got = fa.ssim(T(a), T(b), win_size=ksz, return_map=True).double().cpu().numpy()
    want = O.ssim(a, b, win_size=ksz, return_map=True)
    assert np.abs(got - want).max() < TOL_MAP


def test_identity_and_flat():
    a, _ = baseline_pair((2, 3, 64, 64), 1.0)
    x = T(a)
    assert abs(float(fa.ssim(x, x)) - 1.0) < 1e-6
    f = torch.full((1, 1, 33, 41), 128, dtype=torch.uint8, device="cuda")
    assert abs(float(fa.ssim(f, f)) - 1.0) < 1e-6


@pytest.mark.parametrize("mode", ["bt601", "bt709", "matlab"])
@pytest.mark.parametrize("cb", [0, 4])
def test_luma_crop_ssim(golden, mode, cb):
    a, b = T(golden["luma_a"])[None], T(golden["luma_b"])[None]
    got = float(fa.ssim(a, b, data_range=255.0, luma=mode, crop_border=cb))
    assert abs(got - float(golden[f"luma_{mode}_{cb}_ssim"])) < TOL_SSIM


def test_full_hd_plane_vs_oracle():
    """One 1080p plane at full size against the float64 oracle."""
    a, b = baseline_pair((1, 1, 1080, 1920), 8.0, seed=0)
    got = float(fa.ssim(T(a), T(b)))
    assert abs(got - O.ssim(a, b)) < 1e-6


# ---------------------------------------------------------------------------- #
# backward
# ---------------------------------------------------------------------------- #

def _grad_case(shape=(2, 3, 40, 52), seed=0):
    rng = np.random.default_rng(seed)
    a = rng.random(shape)
    b = np.clip(a + 0.05 * rng.standard_normal(shape), 0, 1)
    return a, b


def _rel(got, want):
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


@pytest.mark.parametrize("need", ["x", "y", "both"])
@pytest.mark.parametrize("ksz", [11, 7, 3])
def test_backward_scalar_vs_oracle(need, ksz):
    a, b = _grad_case()
    x = T(a, torch.float32).requires_grad_(need in ("x", "both"))
    y = T(b, torch.float32).requires_grad_(need in ("y", "both"))
    loss = 1 - fa.ssim(x, y, data_range=1.0, win_size=ksz)
    loss.backward()
    dx, dy = O.ssim_grad(a, b, data_range=1.0, win_size=ksz)
    if need in ("x", "both"):
        assert _rel(-x.grad.double().cpu().numpy(), dx) < 1e-4
    if need in ("y", "both"):
        assert _rel(-y.grad.double().cpu().numpy(), dy) < 1e-4


@pytest.mark.parametrize("shape", [(1, 1, 11, 11), (1, 1, 13, 400), (1, 2, 345, 29),
                                   (1, 1, 700, 343), (2, 1, 64, 700)])
def test_backward_strip_edges(shape):
    a, b = _grad_case(shape, seed=3)
    x = T(a, torch.float32).requires_grad_()
    y = T(b, torch.float32).requires_grad_()
    fa.ssim(x, y, data_range=1.0).backward()
    dx, dy = O.ssim_grad(a, b, data_range=1.0)
    assert _rel(x.grad.double().cpu().numpy(), dx) < 1e-4
    assert _rel(y.grad.double().cpu().numpy(), dy) < 1e-4


def test_backward_through_map_and_per_image():
    a, b = _grad_case((2, 2, 37, 45), seed=5)
    x = T(a, torch.float32).requires_grad_()
    y = T(b, torch.float32)
    m = fa.ssim(x, y, data_range=1.0, return_map=True)
    w = torch.randn(m.shape, generator=torch.Generator().manual_seed(0)).to("cuda")
    (m * w).sum().backward()
    dx, _ = O.ssim_grad(a, b, data_range=1.0, upstream=w.double().cpu().numpy())
    assert _rel(x.grad.double().cpu().numpy(), dx) < 1e-4

    x.grad = None
    per = fa.ssim(x, y, data_range=1.0, reduction="none")
    wn = torch.tensor([0.7, -1.3], device="cuda", dtype=torch.float64)
    (per * wn).sum().backward()
    hw = 27 * 35
    up = np.broadcast_to((wn.cpu().numpy() / (2 * hw))[:, None, None, None], (2, 2, 27, 35))
    dx, _ = O.ssim_grad(a, b, data_range=1.0, upstream=up)
    assert _rel(x.grad.double().cpu().numpy(), dx) < 1e-4


def test_backward_vs_central_differences_on_reference():
    """test_metrics.py:148-171: the gradient against finite differences of the
    float64 oracle (a 1e-4 relative bar on the largest components)."""
    a, b = _grad_case((1, 1, 24, 26), seed=11)
    y = T(b, torch.float32).requires_grad_()
    fa.ssim(T(a, torch.float32), y, data_range=1.0).backward()
    g = y.grad.double().cpu().numpy()
    idx = np.unravel_index(np.argsort(-np.abs(g).ravel())[:6], g.shape)
    h = 1e-5
    for t in zip(*idx):
        p, m = b.copy(), b.copy()
        p[t] += h
        m[t] -= h
        fd = (O.ssim(a, p, data_range=1.0) - O.ssim(a, m, data_range=1.0)) / (2 * h)
        assert abs(g[t] - fd) <= 1e-4 * abs(fd) + 1e-7


def test_backward_does_not_sync():
    a, b = _grad_case((1, 3, 128, 128))
    y = T(b, torch.float32).requires_grad_()
    x = T(a, torch.float32)
    loss = 1 - fa.ssim(x, y, data_range=1.0)
    torch.cuda.synchronize()
    torch.cuda._sleep(200_000_000)  # keep the stream busy
    ev = torch.cuda.Event()
    loss.backward()
    ev.record()
    assert not ev.query(), "backward synchronised with the device"
    torch.cuda.synchronize()


def test_double_backward_refuses_loudly():
    a, b = _grad_case((1, 1, 64, 64))
    x = T(a, torch.float32).requires_grad_()
    with pytest.raises(RuntimeError, match="twice differentiable"):
        g, = torch.autograd.grad(fa.ssim(x, T(b, torch.float32), data_range=1.0), x,
                                 create_graph=True)
        torch.autograd.grad(g.sum(), x)


# ---------------------------------------------------------------------------- #
# MS-SSIM
# ---------------------------------------------------------------------------- #

@pytest.mark.parametrize("k", ["m0", "m1", "m2"])
def test_ms_ssim_matches_golden(golden, k):
    a, b = T(golden[f"{k}_a"])[None, None], T(golden[f"{k}_b"])[None, None]
    assert abs(float(fa.ms_ssim(a, b, data_range=255.0)) - float(golden[f"{k}_ms_ssim"])) < TOL_SSIM


def test_ms_ssim_channels_and_batch():
    a, b = baseline_pair((2, 3, 180, 200), 12.0, seed=8)
    got = fa.ms_ssim(T(a), T(b), reduction="none").cpu().numpy()
    np.testing.assert_allclose(got, O.ms_ssim(a, b, reduction="none"), atol=TOL_SSIM)
    with pytest.raises(ValueError):
        fa.ms_ssim(T(a)[..., :175, :], T(b)[..., :175, :])


def test_ms_ssim_backward_vs_finite_differences():
    # a quick float64-input check; the reference's own bars (1e-3 against
    # central differences, 2e-4 against float64 autograd, at float32-exact
    # inputs) are held in tests/test_gpu_configs.py
    rng = np.random.default_rng(2)
    a = rng.random((1, 1, 176, 180))
    b = np.clip(a + 0.1 * rng.standard_normal(a.shape), 0, 1)
    y = T(b, torch.float32).requires_grad_()
    fa.ms_ssim(T(a, torch.float32), y, data_range=1.0).backward()
    g = y.grad.double().cpu().numpy()
    idx = np.unravel_index(np.argsort(-np.abs(g).ravel())[:4], g.shape)
    h = 1e-5
    for t in zip(*idx):
        p, m = b.copy(), b.copy()
        p[t] += h
        m[t] -= h
        fd = (O.ms_ssim(a, p, data_range=1.0) - O.ms_ssim(a, m, data_range=1.0)) / (2 * h)
        assert abs(g[t] - fd) <= 2e-3 * abs(fd) + 1e-8


@pytest.mark.parametrize("reduction", ["mean", "none"])
@pytest.mark.parametrize("hw", [(67, 90), (120, 129)])
@pytest.mark.parametrize("which", ["x", "y", "both"])
def test_fused_loss_grad_matches_two_pass(reduction, hw, which):
    """Value + unit gradient in one launch (then scaled by the upstream
    gradient) equals the forward followed by the separate backward."""
    g = torch.Generator().manual_seed(3)
    a = torch.rand((2, 3) + hw, generator=g).cuda()
    b = (a + 0.05 * torch.randn(a.shape, generator=g).cuda()).clamp(0, 1)
    up = torch.randn(2, generator=g, dtype=torch.float64).cuda() if reduction == "none" else None
    res = {}
    for fused in (True, False):
        fa.set_fused_loss_grad(fused)
        try:
            x = a.clone().requires_grad_(which in ("x", "both"))
            y = b.clone().requires_grad_(which in ("y", "both"))
            v = fa.ssim(x, y, data_range=1.0, reduction=reduction)
            (1.0 - v).sum().backward() if up is None else (v * up).sum().backward()
            res[fused] = (v.detach(), x.grad, y.grad)
        finally:
            fa.set_fused_loss_grad(True)
    (v1, gx1, gy1), (v0, gx0, gy0) = res[True], res[False]
    # the fused kernel owns 32K-(K-1)-column strips, the forward 32K-column
    # ones: float per-batch partials group differently (~1e-9)
    torch.testing.assert_close(v1, v0, rtol=0, atol=1e-7)
    for g1, g0 in ((gx1, gx0), (gy1, gy0)):
        assert (g1 is None) == (g0 is None)
        if g1 is not None:
            # the two paths apply the upstream gradient at different points:
            # rounding differs, relative to the gradient's scale
            torch.testing.assert_close(g1, g0, rtol=1e-5, atol=1e-5 * float(g0.abs().max()))


@pytest.mark.parametrize("shape", [(3, 2, 17, 31), (2, 3, 64, 96)])
@pytest.mark.parametrize("per_image", [False, True])
def test_grad_scale(shape, per_image):
    from frame_analytics_b200 import backend
    u = torch.randn(shape, device="cuda")
    g = torch.randn(shape[0] if per_image else (), dtype=torch.float64, device="cuda")
    got = backend.grad_scale(u, g, per_image=per_image, mult=shape[0])
    f = (g * shape[0]).to(torch.float32)
    ref = u * (f.view(-1, 1, 1, 1) if per_image else f)
    assert torch.equal(got, ref)


def _torch_ssim_mean(x, y, w, shift, C1, C2):
    """float64 torch SSIM batch mean with an arbitrary separable window."""
    k = w.numel()
    xs, ys = x - shift, y - shift
    n, c, h, wd = x.shape

    def blur(t):
        t = t.reshape(n * c, 1, h, wd)
        t = torch.nn.functional.conv2d(t, w.view(1, 1, k, 1))
        t = torch.nn.functional.conv2d(t, w.view(1, 1, 1, k))
        return t
    ux, uy = blur(xs), blur(ys)
    sxx = blur(xs * xs) - ux * ux
    syy = blur(ys * ys) - uy * uy
    sxy = blur(xs * ys) - ux * uy
    mx, my = ux + shift, uy + shift
    s = ((2 * mx * my + C1) * (2 * sxy + C2)) / ((mx * mx + my * my + C1) * (sxx + syy + C2))
    return s.mean()


@pytest.mark.parametrize("taps", [[0.1, 0.2, 0.4, 0.2, 0.1], [0.05, 0.15, 0.5, 0.2, 0.1],
                                  [0.2, 0.3, 0.5]])
@pytest.mark.parametrize("fused", [True, False])
def test_backward_symmetric_and_asymmetric_windows(taps, fused):
    """Symmetric windows take the warp-specialised kernel, asymmetric ones the
    general one; both match float64 torch autograd."""
    from frame_analytics_b200 import backend
    g = torch.Generator().manual_seed(11)
    a = torch.rand((2, 2, 40, 72), generator=g).cuda()
    b = (a + 0.05 * torch.randn(a.shape, generator=g).cuda()).clamp(0, 1)
    win = backend.Taps(taps)
    C1, C2, shift = 1e-4, 9e-4, 0.5
    if fused:
        _, _, dx, dy = backend.ssim_loss_grad(a, b, win, shift=shift, C1=C1, C2=C2)
    else:
        one = torch.ones((), device="cuda")
        dx, dy = backend.ssim_backward(a, b, win, shift=shift, C1=C1, C2=C2, gscalar=one)
    xd, yd = a.double().requires_grad_(True), b.double().requires_grad_(True)
    wt = torch.tensor(taps, dtype=torch.float64, device="cuda")
    _torch_ssim_mean(xd, yd, wt, shift, C1, C2).backward()
    for got, ref in ((dx, xd.grad), (dy, yd.grad)):
        torch.testing.assert_close(got.double(), ref, rtol=1e-3, atol=2e-3 * float(ref.abs().max()))


@pytest.mark.parametrize("reduction", ["mean", "none"])
def test_fused_loss_grad_second_backward(reduction):
    """The first backward hands the fused kernel's buffer to autograd; a second
    backward through the same graph recomputes and accumulates the same."""
    g = torch.Generator().manual_seed(5)
    a = torch.rand((2, 3, 60, 80), generator=g).cuda()
    b = (a + 0.05 * torch.randn(a.shape, generator=g).cuda()).clamp(0, 1)
    y = b.clone().requires_grad_(True)
    v = fa.ssim(a, y, data_range=1.0, reduction=reduction)
    loss = (1.0 - v).sum()
    loss.backward(retain_graph=True)
    first = y.grad.clone()
    loss.backward()
    torch.testing.assert_close(y.grad, 2 * first, rtol=1e-5, atol=1e-5 * float(first.abs().max()))
    fa.set_fused_loss_grad(False)
    try:
        y2 = b.clone().requires_grad_(True)
        (1.0 - fa.ssim(a, y2, data_range=1.0, reduction=reduction)).sum().backward()
    finally:
        fa.set_fused_loss_grad(True)
    torch.testing.assert_close(first, y2.grad, rtol=1e-5, atol=1e-5 * float(first.abs().max()))

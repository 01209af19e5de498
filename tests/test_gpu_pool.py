"""MS-SSIM pyramid pooling on the GPU: the 2x2 mean-pool kernel and its
adjoint against torch's avg_pool2d (the reference's own pooling,
functional.py:717-725), and MS-SSIM through it against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import fa_oracle as O
from conftest import natural_pair

import frame_analytics_b200 as fa
from frame_analytics_b200 import backend

pytestmark = pytest.mark.gpu


def _pair(n, c, h, w, noise, seed):
    """Stack of natural_pair planes shaped (n, c, h, w), uint8 values."""
    ps = [natural_pair(h, w, seed=seed + i, noise=noise) for i in range(n * c)]
    a = np.stack([p[0] for p in ps]).reshape(n, c, h, w).astype(np.uint8)
    b = np.stack([p[1] for p in ps]).reshape(n, c, h, w).astype(np.uint8)
    return a, b


def _rand(shape, dt, seed=0):
    g = torch.Generator().manual_seed(seed)
    if dt == torch.uint8:
        return torch.randint(0, 256, shape, generator=g, dtype=torch.uint8).cuda()
    return (torch.rand(shape, generator=g, dtype=torch.float64) * 255).to(dt).cuda()


@pytest.mark.parametrize("shape", [(1, 1, 2, 2), (2, 3, 37, 53), (1, 3, 64, 129), (3, 1, 131, 66),
                                   (2, 3, 34, 64), (1, 2, 7, 32), (1, 1, 6, 96)])
@pytest.mark.parametrize("dt", [torch.uint8, torch.float16, torch.bfloat16, torch.float32])
def test_pool2_bitwise_vs_avg_pool2d(shape, dt):
    x = _rand(shape, dt)
    got = backend.pool2(x)
    ref = F.avg_pool2d(x.to(torch.float32), 2)
    assert got.dtype == torch.float32 and got.shape == ref.shape
    assert torch.equal(got, ref)


def test_pool2_float64_input():
    """float64 planes pool in float64 (the MS-SSIM pyramid of float64 frames)."""
    x = _rand((2, 2, 41, 30), torch.float64)
    got = backend.pool2(x)
    assert got.dtype == torch.float64
    torch.testing.assert_close(got, F.avg_pool2d(x, 2), rtol=0, atol=1e-12)


def test_pool2_vector_path_with_row_padding():
    """16-byte aligned row pitch wider than the row: the vector path with strides."""
    for dt in (torch.uint8, torch.float16, torch.float32):
        x = _rand((2, 3, 41, 80), dt)[..., :64]
        assert not x.is_contiguous()
        assert torch.equal(backend.pool2(x), F.avg_pool2d(x.float(), 2))


def test_pool2_strided_views():
    x = _rand((2, 3, 80, 100), torch.uint8)
    crop = x[:, :, 3:-5, 7:-2]
    assert not crop.is_contiguous()
    assert torch.equal(backend.pool2(crop), F.avg_pool2d(crop.float(), 2))
    nhwc = _rand((2, 50, 60, 3), torch.float32).permute(0, 3, 1, 2)
    assert torch.equal(backend.pool2(nhwc), F.avg_pool2d(nhwc.contiguous(), 2))


@pytest.mark.parametrize("mode", ["bt601", "bt709"])
def test_pool2_luma(mode):
    x = _rand((2, 3, 45, 62), torch.uint8)
    lum = fa.rgb_to_luma(x, mode, data_range=255.0)
    ref = F.avg_pool2d(lum.to(torch.float32), 2)
    from frame_analytics_b200.functional import _luma_k
    got = backend.pool2(x, luma=_luma_k(mode, 255.0))
    torch.testing.assert_close(got, ref, rtol=0, atol=2e-4)


@pytest.mark.parametrize("shape", [(1, 1, 2, 2), (2, 3, 37, 53), (1, 2, 64, 129)])
def test_pool2_backward_bitwise(shape):
    x = _rand(shape, torch.float32).requires_grad_(True)
    y = F.avg_pool2d(x, 2)
    g = torch.randn_like(y)
    (ref,) = torch.autograd.grad(y, x, g)
    got = backend.pool2_backward(g, shape)
    assert torch.equal(got, ref)


def test_pool2_rejects_bad_input():
    with pytest.raises(Exception):
        backend.pool2(_rand((1, 1, 1, 8), torch.float32))
    with pytest.raises(Exception):
        backend.pool2(_rand((1, 2, 8, 8), torch.uint8), luma=(0.3, 0.5, 0.2, 0.0))


@pytest.mark.parametrize("luma", [None, True, "bt709"])
@pytest.mark.parametrize("hw", [(176, 176), (193, 241)])
def test_ms_ssim_vs_oracle(luma, hw):
    a, b = _pair(2, 3, *hw, 12.0, seed=5)
    got = fa.ms_ssim(torch.as_tensor(a).cuda(), torch.as_tensor(b).cuda(), luma=luma,
                     reduction="none").cpu().numpy()
    np.testing.assert_allclose(got, O.ms_ssim(a, b, luma=luma, reduction="none"), atol=5e-6)


def test_ms_ssim_grad_matches_torch_pooling():
    """Gradient through the pool kernels equals the one through avg_pool2d."""
    a, b = _pair(1, 3, 180, 200, 10.0, seed=9)
    x0 = torch.as_tensor(a, dtype=torch.float32).cuda() / 255
    y = torch.as_tensor(b, dtype=torch.float32).cuda() / 255
    x = x0.clone().requires_grad_(True)
    fa.ms_ssim(x, y, data_range=1.0).backward()
    xr = x0.clone().requires_grad_(True)
    from frame_analytics_b200 import functional as fn
    orig = fn._Pool2Fn.apply
    try:
        fn._Pool2Fn.apply = staticmethod(lambda t: F.avg_pool2d(t.float(), 2))
        fa.ms_ssim(xr, y, data_range=1.0).backward()
    finally:
        fn._Pool2Fn.apply = orig
    torch.testing.assert_close(x.grad, xr.grad, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("f", [2, 3, 4, 5])
@pytest.mark.parametrize("hw", [(37, 53), (64, 96), (101, 80)])
def test_box_downsample_vs_oracle(f, hw):
    x = _rand((2, 3) + hw, torch.uint8)
    got = backend.box_downsample(x, f).double().cpu().numpy()
    ref = O.matlab_downsample(x.double().cpu().numpy(), f)
    assert got.shape == ref.shape
    # float32 sums of values up to 255 with an inexact 1/f^2 (f = 3, 5): a few
    # float32 ulp, as in the reference's own float32 conv
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-5)


def test_box_downsample_luma_and_strides():
    x = _rand((2, 3, 90, 120), torch.uint8)
    xc = x[:, :, 3:-2, 5:-4]
    lk = (0.299, 0.587, 0.114, 0.0)
    got = backend.box_downsample(xc, 3, luma=lk).double().cpu().numpy()
    lum = np.tensordot(np.array(lk[:3]), xc.double().cpu().numpy(), axes=([0], [1]))[:, None]
    np.testing.assert_allclose(got, O.matlab_downsample(lum, 3), rtol=2e-6, atol=1e-5)


@pytest.mark.parametrize("f", [2, 3, 4])
@pytest.mark.parametrize("hw", [(37, 53), (64, 96)])
def test_box_downsample_backward(f, hw):
    # float64 reference: cuDNN may run a float32 conv2d in TF32
    x = _rand((1, 2) + hw, torch.float64).requires_grad_(True)
    pad = f // 2
    ker = torch.full((1, 1, f, f), 1.0 / (f * f), device="cuda", dtype=torch.float64)
    xp = F.pad(x.reshape(2, 1, *hw), (pad, pad, pad, pad), mode="replicate")
    d = F.conv2d(xp, ker)[:, :, ::f, ::f]
    y = d.reshape(1, 2, d.shape[-2], d.shape[-1])
    g = torch.randn_like(y)
    (ref,) = torch.autograd.grad(y, x, g)
    got = backend.box_downsample_backward(g.float(), tuple(x.shape), f)
    torch.testing.assert_close(got.double(), ref, rtol=1e-5, atol=1e-6)


def test_ssim_matlab_downsample_mode():
    a, b = _pair(1, 3, 600, 800, 10.0, seed=2)  # min side 600 -> f = 2
    got = float(fa.ssim(torch.as_tensor(a).cuda(), torch.as_tensor(b).cuda(), downsample=True))
    da = O.matlab_downsample(a.astype(np.float64), 2)
    db = O.matlab_downsample(b.astype(np.float64), 2)
    assert abs(got - O.ssim(da, db)) < 5e-6
    # luma folded into the downsample kernel
    got_l = float(fa.ssim(torch.as_tensor(a).cuda(), torch.as_tensor(b).cuda(), downsample=True,
                          luma="bt601"))
    la = O.rgb_to_luma(a.astype(np.float64), "bt601", 255.0)
    lb = O.rgb_to_luma(b.astype(np.float64), "bt601", 255.0)
    assert abs(got_l - O.ssim(O.matlab_downsample(la, 2), O.matlab_downsample(lb, 2))) < 5e-6


def test_ssim_matlab_downsample_gradient():
    """Training through the downsample: the native adjoint against autograd
    through the torch formulation of the same downsample."""
    a, b = _pair(1, 3, 520, 530, 8.0, seed=4)
    y0 = torch.as_tensor(b, dtype=torch.float32).cuda() / 255
    x = torch.as_tensor(a, dtype=torch.float32).cuda() / 255
    y = y0.clone().requires_grad_(True)
    fa.ssim(x, y, data_range=1.0, downsample=True).backward()
    y2 = y0.clone().requires_grad_(True)
    f = 2
    ker = torch.full((1, 1, f, f), 0.25, device="cuda", dtype=torch.float64)

    def down(t):  # float64 conv (no TF32), result back to float32
        tp = F.pad(t.double().reshape(3, 1, 520, 530), (1, 1, 1, 1), mode="replicate")
        d = F.conv2d(tp, ker)[:, :, ::2, ::2]
        return d.reshape(1, 3, d.shape[-2], d.shape[-1]).float()
    fa.ssim(down(x), down(y2), data_range=1.0).backward()
    torch.testing.assert_close(y.grad, y2.grad, rtol=1e-3, atol=1e-3 * float(y2.grad.abs().max()))

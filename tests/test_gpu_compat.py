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


def _gauss(k, sigma):
    c = torch.arange(k, dtype=torch.float64) - (k - 1) / 2
    g = torch.exp(-(c * c) / (2 * sigma * sigma))
    return (g / g.sum()).float()


def _compat_ssim(lib, x, y, w, k, stream):
    n, c, h, wd = x.shape
    bpp = ctypes.c_int(0)
    assert lib.fa_cuda_ssim_workspace(h, wd, k, ctypes.byref(bpp)) == 0
    part = torch.empty((n * c, bpp.value), dtype=torch.float64, device="cuda")
    tot = torch.empty((), dtype=torch.float64, device="cuda")
    rc = lib.fa_cuda_ssim(x.data_ptr(), y.data_ptr(), 0, n, c, h, wd, w.data_ptr(), k,
                          127.5, (0.01 * 255) ** 2, (0.03 * 255) ** 2, None, part.data_ptr(),
                          bpp.value, None, tot.data_ptr(), 0, stream)
    assert rc == 0
    return tot, part


def test_compat_window_reread_at_the_same_address():
    """The window is read on the device at every call: a window freed and
    replaced by a different one at the same address gives the new result."""
    lib = _cabi.load()
    a, b = baseline_pair((1, 2, 64, 80), 9.0, seed=5)
    x, y = T(a), T(b)
    buf = torch.empty(64, dtype=torch.float32, device="cuda")
    w = buf[:11]
    got = []
    for sigma in (1.5, 0.8):
        w.copy_(_gauss(11, sigma).cuda())  # same device address, new taps
        tot, _ = _compat_ssim(lib, x, y, w, 11, _st())
        got.append(float(tot))
    for v, sigma in zip(got, (1.5, 0.8)):
        assert abs(v - O.ssim(a, b, sigma=sigma)) < 5e-6
    # a released window's block handed out again by the caching allocator
    w1 = _gauss(11, 1.5).cuda()
    p1 = w1.data_ptr()
    tot1, _ = _compat_ssim(lib, x, y, w1, 11, _st())
    v1 = float(tot1)
    del w1
    w2 = torch.empty(11, dtype=torch.float32, device="cuda")
    if w2.data_ptr() == p1:
        w2.copy_(_gauss(11, 2.5).cuda())
        tot2, _ = _compat_ssim(lib, x, y, w2, 11, _st())
        assert abs(float(tot2) - O.ssim(a, b, sigma=2.5)) < 5e-6
    assert abs(v1 - O.ssim(a, b, sigma=1.5)) < 5e-6


def test_compat_ssim_captured_on_its_first_call():
    """The compat SSIM call makes no host synchronisation, so its very first
    call in a process can be recorded into a CUDA graph."""
    import subprocess
    import sys
    import textwrap
    from conftest import REPO
    code = textwrap.dedent(f"""
        import ctypes, sys, torch
        sys.path.insert(0, {str(REPO)!r})
        from frame_analytics_b200 import _cabi
        lib = _cabi.load()
        g = torch.Generator().manual_seed(0)
        x = torch.randint(0, 256, (1, 3, 64, 96), generator=g, dtype=torch.uint8).cuda()
        y = torch.randint(0, 256, (1, 3, 64, 96), generator=g, dtype=torch.uint8).cuda()
        c = torch.arange(11, dtype=torch.float64) - 5
        w = torch.exp(-c * c / 4.5); w = (w / w.sum()).float().cuda()
        bpp = ctypes.c_int(0)
        assert lib.fa_cuda_ssim_workspace(64, 96, 11, ctypes.byref(bpp)) == 0
        part = torch.empty((3, bpp.value), dtype=torch.float64, device="cuda")
        tot = torch.zeros((), dtype=torch.float64, device="cuda")
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            rc = lib.fa_cuda_ssim(x.data_ptr(), y.data_ptr(), 0, 1, 3, 64, 96, w.data_ptr(), 11,
                                  127.5, 6.5025, 58.5225, None, part.data_ptr(), bpp.value,
                                  None, tot.data_ptr(), 0, s.cuda_stream)
        assert rc == 0, rc
        graph.replay()
        torch.cuda.synchronize()
        print(float(tot))
    """)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 256, (1, 3, 64, 96), generator=g, dtype=torch.uint8).numpy()
    b = torch.randint(0, 256, (1, 3, 64, 96), generator=g, dtype=torch.uint8).numpy()
    assert abs(float(out.stdout.strip().splitlines()[-1]) - O.ssim(a, b)) < 5e-6


@pytest.mark.parametrize("taps", [[0.1, 0.2, 0.4, 0.2, 0.1], [0.05, 0.15, 0.5, 0.2, 0.1]])
def test_compat_backward_with_device_window(taps):
    """fa_cuda_ssim_backward reads its (possibly asymmetric) window on the
    device; the gradient matches the extended entry point given host taps."""
    from frame_analytics_b200 import backend
    lib = _cabi.load()
    g = torch.Generator().manual_seed(4)
    x = torch.rand((2, 2, 40, 72), generator=g).cuda()
    y = (x + 0.05 * torch.randn(x.shape, generator=g).cuda()).clamp(0, 1)
    w = torch.tensor(taps, dtype=torch.float32, device="cuda")
    one = torch.ones((), device="cuda")
    C1, C2, shift = 1e-4, 9e-4, 0.5
    dx = torch.empty_like(x)
    dy = torch.empty_like(y)
    rc = lib.fa_cuda_ssim_backward(x.data_ptr(), y.data_ptr(), None, one.data_ptr(),
                                   w.data_ptr(), len(taps), 2, 2, 40, 72, shift, C1, C2, None,
                                   dx.data_ptr(), dy.data_ptr(), 0, _st())
    assert rc == 0
    rx, ry = backend.ssim_backward(x, y, backend.Taps(taps), shift=shift, C1=C1, C2=C2,
                                   gscalar=one)
    torch.testing.assert_close(dx, rx, rtol=1e-5, atol=1e-6 * float(rx.abs().max()))
    torch.testing.assert_close(dy, ry, rtol=1e-5, atol=1e-6 * float(ry.abs().max()))


def test_wait_timeout_is_reported_by_the_next_call():
    """A bounded device wait that runs out (here: a phase nothing completes,
    with no copy in flight) is returned as FA_E_TIMEOUT by the next call, and
    the context stays usable."""
    lib = _cabi.load()
    a, b = baseline_pair((1, 1, 32, 48), 5.0, seed=3)
    x, y = T(a), T(b)
    assert lib.fa_b200_wait_selftest(2_000_000, 0, _st()) == 0  # 2 ms
    torch.cuda.synchronize()
    n = 1
    bpi = ctypes.c_int(0)
    assert lib.fa_cuda_pixel_workspace(n, 32 * 48, 0, ctypes.byref(bpi)) == 0
    part = torch.empty((n, bpi.value), dtype=torch.float64, device="cuda")
    tot = torch.empty((), dtype=torch.float64, device="cuda")
    args = (x.data_ptr(), y.data_ptr(), 0, n, 32 * 48, 0, 0.0, -1e300, part.data_ptr(),
            bpi.value, None, tot.data_ptr(), None, None, 0, _st())
    assert lib.fa_cuda_pixel_reduce(*args) == _cabi.FA_E_TIMEOUT
    # reported once; the library and the context keep working
    assert lib.fa_cuda_pixel_reduce(*args) == 0
    torch.cuda.synchronize()
    assert float(tot) == O.pixel(a, b, "mse")
    with pytest.raises(_cabi.KernelError, match="timed out"):
        lib.fa_b200_wait_selftest(1_000_000, 0, _st())
        torch.cuda.synchronize()
        _cabi.check(lib.fa_cuda_pixel_reduce(*args))

"""The C port timed as the CPU baseline (oracle/ssim_port.c) against the
float64 oracle: the SSIM sum and both gradients on small shapes.  The port is
the denominator of every CPU-vs-GPU ratio the bench reports, so it is held to
the same bars as the GPU path (value 5e-6, gradient 1e-4 relative)."""

from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest

import fa_oracle as O
from conftest import REPO

SO = REPO / "oracle" / "_build" / "libssim_port.so"


@pytest.fixture(scope="module")
def port():
    subprocess.run(["make", "-C", str(REPO / "oracle"), "port"], check=True,
                   stdout=subprocess.DEVNULL)
    lib = ctypes.CDLL(str(SO))
    lib.ssim_port_fwd_bwd.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                      ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int]
    lib.ssim_port_fwd_bwd.restype = ctypes.c_int
    return lib


@pytest.mark.parametrize("shape,ksz", [((2, 3, 40, 52), 11), ((1, 2, 64, 33), 7),
                                       ((1, 1, 11, 11), 11), ((3, 1, 29, 70), 3)])
def test_port_matches_oracle(port, shape, ksz):
    rng = np.random.default_rng(sum(shape) + ksz)
    a = rng.random(shape).astype(np.float32)
    b = np.clip(a + 0.05 * rng.standard_normal(shape), 0, 1).astype(np.float32)
    n, c, h, w = shape
    planes, hw = n * c, (h - ksz + 1) * (w - ksz + 1)
    win = O.gaussian_window_1d(ksz, 1.5).astype(np.float64)
    out = np.zeros(planes, np.float64)
    dx = np.zeros(shape, np.float32)
    dy = np.zeros(shape, np.float32)
    g = 1.0 / (planes * hw)
    rc = port.ssim_port_fwd_bwd(a.ctypes.data, b.ctypes.data, planes, h, w, win.ctypes.data,
                                ksz, 1e-4, 9e-4, g, out.ctypes.data, dx.ctypes.data,
                                dy.ctypes.data, 2)
    assert rc == 0
    ad, bd = a.astype(np.float64), b.astype(np.float64)
    assert abs(out.sum() / (planes * hw) - O.ssim(ad, bd, data_range=1.0, win_size=ksz)) < 5e-6
    wx, wy = O.ssim_grad(ad, bd, data_range=1.0, win_size=ksz)
    for got, want in ((dx, wx), (dy, wy)):
        assert float(np.abs(got - want).max() / np.abs(want).max()) < 1e-4

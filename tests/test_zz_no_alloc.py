"""The allocation-free pixel reduction, fa_b200_pixel_reduce_noalloc.

It exists for callers that cannot allocate device memory (plugins that only
see a host application's frame buffers, code where cudaMalloc is not
available): its scratch is a fixed array inside the library.  Checked
through the C ABI against fa_b200_pixel_reduce, twice in a row, because the
shared scratch keeps the previous call's contents.  This file is named so
that pytest collects it last."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import baseline_pair

from frame_analytics_b200 import _cabi, backend

pytestmark = pytest.mark.gpu


def _views(x, y):
    vx, x = backend.as_view(x)
    vy, y = backend.as_view(y)
    return vx, vy, x, y


def _noalloc(x, y, op, param, psnr_bias, luma=None):
    lib = _cabi.load()
    vx, vy, x, y = _views(x, y)
    n = vx.n
    per = torch.empty(n, dtype=torch.float64, device=x.device)
    tot = torch.empty((), dtype=torch.float64, device=x.device)
    ppi = torch.empty(n, dtype=torch.float64, device=x.device)
    ptot = torch.empty((), dtype=torch.float64, device=x.device)
    isum = torch.empty(n, dtype=torch.int64, device=x.device)
    lk = None if luma is None else (ctypes.c_double * 4)(*luma)
    rc = lib.fa_b200_pixel_reduce_noalloc(
        ctypes.byref(vx), ctypes.byref(vy), lk, op, float(param), float(psnr_bias),
        per.data_ptr(), tot.data_ptr(), ppi.data_ptr(), ptot.data_ptr(), isum.data_ptr(),
        x.device.index or 0, torch.cuda.current_stream().cuda_stream)
    return rc, per, tot, ppi, ptot, isum


def _existing(x, y, op, param, psnr_bias, luma=None):
    per = backend.pixel(x, y, op=op, param=param, per_image=True, luma=luma)
    tot = backend.pixel(x, y, op=op, param=param, per_image=False, luma=luma)
    _, isum = backend.pixel(x, y, op=op, param=param, per_image=True, luma=luma, want_isum=True)
    p = backend.pixel(x, y, op=op, per_image=True, psnr_bias=psnr_bias, luma=luma) \
        if op == backend.OP_MSE else None
    return per, tot, isum, p


@pytest.mark.parametrize("dtype", [torch.uint8, torch.float32])
@pytest.mark.parametrize("op,param", [(0, 0.0), (1, 0.0), (2, 1e-6), (3, 2.0)])
def test_noalloc_matches_existing_entry_point_twice(dtype, op, param):
    a, b = baseline_pair((5, 3, 67, 131), 9.0, seed=op)
    x = torch.as_tensor(a, device="cuda").to(dtype)
    y = torch.as_tensor(b, device="cuda").to(dtype)
    bias = 10 * np.log10(255.0 ** 2)
    want_per, want_tot, want_isum, want_p = _existing(x, y, op, param, bias)
    for _ in range(2):  # the shared scratch keeps the last call's contents
        rc, per, tot, ppi, _, isum = _noalloc(x, y, op, param, bias)
        assert rc == 0
        torch.testing.assert_close(per, want_per, rtol=1e-12, atol=1e-12)
        torch.testing.assert_close(tot, want_tot, rtol=1e-12, atol=1e-12)
        if dtype == torch.uint8 and op in (0, 1):
            assert torch.equal(isum, want_isum)  # exact integer sums
        if want_p is not None:
            torch.testing.assert_close(ppi, want_p, rtol=1e-12, atol=1e-12)


def test_noalloc_luma_and_crop():
    a, b = baseline_pair((2, 3, 50, 70), 7.0, seed=3)
    x = torch.as_tensor(a, device="cuda")[..., 4:-4, 4:-4]
    y = torch.as_tensor(b, device="cuda")[..., 4:-4, 4:-4]
    k = (65.481 / 255, 128.553 / 255, 24.966 / 255, 16.0)
    want = backend.pixel(x, y, op=0, per_image=True, luma=k)
    for _ in range(2):
        rc, per, *_ = _noalloc(x, y, 0, 0.0, backend.PSNR_NONE, luma=k)
        assert rc == 0
        torch.testing.assert_close(per, want, rtol=1e-12, atol=1e-12)


def test_noalloc_rejects_batches_beyond_its_scratch():
    x = torch.zeros((4097, 1, 2, 2), dtype=torch.uint8, device="cuda")
    rc, *_ = _noalloc(x, x.clone(), 0, 0.0, backend.PSNR_NONE)
    assert rc == 2  # FA_E_SHAPE: more images than FA_B200_NOALLOC_MAX_IMAGES
    x = torch.zeros((4096, 1, 2, 2), dtype=torch.uint8, device="cuda")
    rc, per, *_ = _noalloc(x, x.clone(), 0, 0.0, backend.PSNR_NONE)
    assert rc == 0 and float(per.abs().max()) == 0.0

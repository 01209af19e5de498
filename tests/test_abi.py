"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares with the reference-compatible names, and validates arguments
before touching a device."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import REPO

from frame_analytics_b200 import _cabi

HEADER = REPO / "include" / "fa_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FA_B200_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", text)))


def test_header_declares_the_reference_entry_points():
    syms = declared_symbols()
    ref = ["fa_cuda_abi_version", "fa_cuda_error_string", "fa_cuda_device_count",
           "fa_cuda_pixel_workspace", "fa_cuda_pixel_reduce", "fa_cuda_ssim_workspace",
           "fa_cuda_ssim", "fa_cuda_ssim_cs", "fa_cuda_ssim_backward",
           "fa_cuda_ssim_cs_backward", "fa_cuda_gmsd_workspace", "fa_cuda_gmsd"]
    for s in ref:
        assert s in syms, s


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_cabi.library_path()))
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # and the Python binding declares a prototype for each
    assert set(declared_symbols()) <= set(_cabi.PROTOTYPES), \
        set(declared_symbols()) - set(_cabi.PROTOTYPES)


def test_load_and_versions():
    lib = _cabi.load()
    assert lib.fa_cuda_abi_version() == 1
    assert lib.fa_b200_abi_version() == 1
    assert lib.fa_cuda_error_string(5) == b"invalid argument"
    assert lib.fa_cuda_error_string(3) == b"unsupported window size"


def test_workspace_queries_validate():
    lib = _cabi.load()
    out = ctypes.c_int(0)
    assert lib.fa_cuda_ssim_workspace(64, 64, 4, ctypes.byref(out)) == 3   # even window
    assert lib.fa_cuda_ssim_workspace(64, 64, 13, ctypes.byref(out)) == 3  # too wide
    assert lib.fa_cuda_ssim_workspace(8, 64, 11, ctypes.byref(out)) == 2   # smaller than window
    assert lib.fa_cuda_ssim_workspace(64, 64, 11, None) == 5
    assert lib.fa_cuda_gmsd_workspace(4, 4, 1, ctypes.byref(out)) == 2
    assert lib.fa_cuda_pixel_workspace(0, 10, 0, ctypes.byref(out)) == 2
    sz = ctypes.c_size_t(0)
    assert lib.fa_b200_ssim_workspace_bytes(1, 1, 64, 64, 6, 0, ctypes.byref(sz)) == 3
    assert lib.fa_b200_gmsd_workspace_bytes(1, 1, 5, 5, 1, 0, ctypes.byref(sz)) == 2


def test_entry_points_reject_null_arguments_before_any_launch():
    lib = _cabi.load()
    assert lib.fa_cuda_pixel_reduce(None, None, 0, 1, 16, 0, 0.0, -1e300, None, 1,
                                    None, None, None, None, 0, None) == 5
    assert lib.fa_cuda_pixel_reduce(1, 1, 0, 1, 16, 9, 0.0, -1e300, 1, 1,
                                    None, None, None, None, 0, None) == 4
    assert lib.fa_cuda_ssim(None, None, 0, 1, 1, 64, 64, None, 11, 0.5, 1e-4, 9e-4,
                            None, None, 1, None, None, 0, None) == 5
    assert lib.fa_b200_pixel_reduce(None, None, None, 0, 0.0, -1e300, None, 0,
                                    None, None, None, None, None, 0, None) == 5
    assert lib.fa_b200_ssim(None, None, None, None, 11, 0.5, 1e-4, 9e-4, None, None, 0,
                            None, None, None, None, 0, None) == 5

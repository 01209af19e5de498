"""ctypes binding of libfa_b200.so.

Plays the role of the reference's loader (frame_analytics/_cabi.py:414-530):
open the shared library, declare every prototype, check the ABI version.
Unlike the reference there is exactly one library, built in-tree for sm_100a,
and no fallback: a missing or stale library raises, loudly.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Optional

HERE = Path(__file__).resolve().parent
DEFAULT_LIB = HERE / "_lib" / "libfa_b200.so"

ABI_VERSION = 1        # FA_ABI_VERSION, reference-compatible block
B200_ABI_VERSION = 1   # FA_B200_ABI_VERSION, extended block

# status codes, include/fa_b200.h (same values as the reference's fa_abi.h:56-64)
FA_OK = 0
_STATUS = {
    1: "unsupported dtype",
    2: "unsupported shape",
    3: "unsupported window size",
    4: "unknown pixel op",
    5: "invalid argument",
    6: "internal error",
    7: "no CUDA device",
    8: "a device-side wait timed out; the results of the kernel that waited are invalid",
}
FA_E_TIMEOUT = 8


class KernelError(RuntimeError):
    """A native entry point returned a non-zero status (frame_analytics/_cabi.py:60-74)."""

    def __init__(self, code: int, text: str):
        super().__init__(f"frame_analytics_b200 kernel error {code}: {text}")
        self.code = code


class fa_view(ctypes.Structure):
    """Mirror of ``struct fa_view`` in include/fa_b200.h."""

    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("c", ctypes.c_int32),
        ("h", ctypes.c_int32),
        ("w", ctypes.c_int32),
        ("pad_", ctypes.c_int32),
        ("stride_n", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
    ]


_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_d = ctypes.c_double
_sz = ctypes.c_size_t
_pview = ctypes.POINTER(fa_view)

# name -> argtypes (restype int unless listed in _RESTYPE)
PROTOTYPES = {
    # reference-compatible block
    "fa_cuda_abi_version": [],
    "fa_cuda_error_string": [_i],
    "fa_cuda_device_count": [_vp],
    "fa_cuda_pixel_workspace": [_i64, _i64, _i, _vp],
    "fa_cuda_pixel_reduce": [_vp, _vp, _i, _i64, _i64, _i, _d, _d, _vp, _i,
                             _vp, _vp, _vp, _vp, _i, _vp],
    "fa_cuda_ssim_workspace": [_i, _i, _i, _vp],
    "fa_cuda_ssim": [_vp, _vp, _i, _i, _i, _i, _i, _vp, _i, _d, _d, _d,
                     _vp, _vp, _i, _vp, _vp, _i, _vp],
    "fa_cuda_ssim_cs": [_vp, _vp, _i, _i, _i, _i, _i, _vp, _i, _d, _d, _d,
                        _vp, _vp, _i, _vp, _vp, _i, _vp],
    "fa_cuda_ssim_backward": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                              _d, _d, _d, _vp, _vp, _vp, _i, _vp],
    "fa_cuda_ssim_cs_backward": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                 _d, _d, _d, _vp, _vp, _vp, _i, _vp],
    "fa_cuda_gmsd_workspace": [_i, _i, _i, _vp],
    "fa_cuda_gmsd": [_vp, _vp, _i, _i, _i, _i, _i, _d, _d, _i, _vp, _vp, _i,
                     _vp, _vp, _i, _vp],
    # extended block
    "fa_b200_abi_version": [],
    "fa_b200_pixel_workspace_bytes": [_i, _i, _vp],
    "fa_b200_pixel_reduce": [_pview, _pview, _vp, _i, _d, _d, _vp, _sz,
                             _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "fa_b200_ssim_workspace_bytes": [_i, _i, _i, _i, _i, _i, _vp],
    "fa_b200_ssim": [_pview, _pview, _vp, _vp, _i, _d, _d, _d, _vp, _vp, _sz,
                     _vp, _vp, _vp, _vp, _i, _vp],
    "fa_b200_ssim_backward": [_vp, _vp, _i, _i, _i, _i, _vp, _i, _d, _d, _d,
                              _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "fa_b200_gmsd_workspace_bytes": [_i, _i, _i, _i, _i, _i, _vp],
    "fa_b200_gmsd": [_pview, _pview, _vp, _d, _d, _i, _vp, _sz, _vp, _vp, _vp,
                     _i, _vp],
    "fa_b200_pixel_reduce_noalloc": [_pview, _pview, _vp, _i, _d, _d, _vp, _vp, _vp, _vp,
                                     _vp, _i, _vp],
    "fa_b200_gmsd_backward": [_vp, _vp, _i, _i, _i, _i, _i, _d, _d, _vp, _vp, _vp, _vp,
                              _vp, _vp, _i, _vp],
    "fa_b200_pixel_backward": [_vp, _vp, _i, _i, _i, _i, _vp, _i, _d, _vp, _i,
                               _vp, _vp, _i, _vp],
    "fa_b200_ssim_mse": [_pview, _pview, _vp, _i, _d, _d, _d, _d, _vp, _sz, _vp, _vp, _vp,
                         _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "fa_b200_ssim_loss_grad_workspace_bytes": [_i, _i, _i, _i, _i, _i, _vp],
    "fa_b200_ssim_loss_grad": [_vp, _vp, _i, _i, _i, _i, _vp, _i, _d, _d, _d, _d, _vp, _sz,
                               _vp, _vp, _vp, _vp, _vp, _i, _vp],
    "fa_b200_grad_scale": [_vp, ctypes.c_longlong, _i, _vp, _i, _d, _vp, _i, _vp],
    "fa_b200_box_downsample": [_pview, _vp, _i, _vp, _i, _vp],
    "fa_b200_box_downsample_backward": [_vp, _i, _i, _i, _i, _i, _vp, _i, _vp],
    "fa_b200_pixel_loss_grad": [_vp, _vp, _i, _i64, _i, _d, _i, _vp, _sz, _vp, _vp, _vp, _vp,
                                _i, _vp],
    "fa_b200_pool2": [_pview, _vp, _vp, _i, _vp],
    "fa_b200_pool2_backward": [_vp, _i, _i, _i, _i, _vp, _i, _vp],
    "fa_b200_wait_selftest": [ctypes.c_ulonglong, _i, _vp],
    "fa_b200_ssim_gmsd_fusable": [_pview, _pview, _i, _i, _vp],
    "fa_b200_ssimulacra2_workspace_bytes": [_i, _i, _i, _i, _vp],
    "fa_b200_ssimulacra2": [_pview, _pview, _d, _i, _vp, _vp, _sz, _vp, _vp, _i, _vp],
    "fa_b200_ssim64_workspace_bytes": [_i, _i, _i, _i, _i, _i, _vp],
    "fa_b200_ssim64": [_pview, _pview, _vp, _vp, _i, _d, _d, _vp, _sz, _vp, _vp, _vp, _vp, _vp,
                       _i, _vp],
    "fa_b200_ssim64_backward": [_vp, _vp, _i, _i, _i, _i, _vp, _i, _d, _d, _vp, _vp, _vp, _vp,
                                _vp, _vp, _vp, _i, _vp],
    "fa_b200_pool64": [_vp, _i, _i, _i, _vp, _i, _vp],
    "fa_b200_pool64_backward": [_vp, _i, _i, _i, _vp, _i, _vp],
    "fa_b200_gmsd64_workspace_bytes": [_i, _i, _i, _i, _i, _i, _i, _vp],
    "fa_b200_gmsd64": [_pview, _pview, _vp, _d, _d, _i, _vp, _sz, _vp, _vp, _vp, _i, _vp],
    "fa_b200_gmsd64_backward": [_vp, _vp, _i, _i, _i, _i, _i, _d, _d, _vp, _vp, _vp, _vp, _vp,
                                _vp, _vp, _i, _vp],
    "fa_b200_ssim_gmsd": [_pview, _pview, _vp, _i, _d, _d, _d, _d, _d, _d, _vp, _sz,
                          _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp],
}
_RESTYPE = {"fa_cuda_error_string": ctypes.c_char_p}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    env = os.environ.get("FA_B200_LIB")
    return Path(env) if env else DEFAULT_LIB


def bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    """Declare every prototype on an opened library; missing symbols raise."""
    for name, args in PROTOTYPES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is absent
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    return lib


def load() -> ctypes.CDLL:
    """Open (once) and return the bound library.  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libfa_b200.so not found at {path}; build it with "
                "`python -m frame_analytics_b200._build`")
        lib = bind(ctypes.CDLL(str(path)))
        if lib.fa_cuda_abi_version() != ABI_VERSION or \
                lib.fa_b200_abi_version() != B200_ABI_VERSION:
            raise RuntimeError(f"{path} has a different ABI version; rebuild it")
        _lib = lib
        return lib


def status_text(code: int) -> str:
    if code < 0 and _lib is not None:
        s = _lib.fa_cuda_error_string(code)
        return s.decode() if s else f"CUDA error {-code}"
    return _STATUS.get(code, f"status {code}")


def check(code: int) -> None:
    if code != FA_OK:
        raise KernelError(code, status_text(code))

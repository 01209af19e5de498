"""Marshalling between torch tensors and the C ABI of libfa_b200.so.

Counterpart of the reference's frame_analytics/backend.py, without its tiers:
there is one backend (the sm_100a kernels) and no fallback.  A call the
kernels cannot serve raises instead of quietly taking another path.

Every buffer a kernel writes is allocated here through torch's caching
allocator (outputs per call; scratch once per device and stream), so no
native call allocates and the calls stay legal inside CUDA-graph capture
(backend.py:145-153 in the reference states the same rule).
"""

from __future__ import annotations

import contextlib
import contextvars
import ctypes
import functools
import math
from typing import Optional, Tuple

import torch

from . import _cabi
from ._cabi import KernelError, fa_view  # noqa: F401

DTYPE_CODE = {
    torch.uint8: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.float32: 3,
    torch.float64: 4,
    torch.uint16: 5,  # extension code: read natively, exact integer MSE / L1
}
PSNR_NONE = -1.0e300
OP_MSE, OP_L1, OP_CHARB, OP_HUBER = 0, 1, 2, 3
KERNEL_WINDOWS = (3, 5, 7, 9, 11)


def lib():
    return _cabi.load()


def status() -> dict:
    try:
        lib()
        return {"available": True, "cuda": torch.cuda.is_available(),
                "library": str(_cabi.library_path()), "error": None}
    except Exception as exc:  # pragma: no cover - environment dependent
        return {"available": False, "cuda": False,
                "library": str(_cabi.library_path()), "error": str(exc)}


# --------------------------------------------------------------------------- #
# input checks
# --------------------------------------------------------------------------- #

def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise TypeError(
                "frame_analytics_b200 computes on CUDA tensors only "
                f"(got a {t.device} tensor); move the inputs to the GPU")


def kernel_dtype(t: torch.Tensor) -> torch.Tensor:
    """Inputs the kernels read natively pass through; other integer types
    (int16/int32/uint16) are widened to float32 on the device first."""
    if t.dtype in DTYPE_CODE:
        return t
    return t.to(torch.float32)


def _row_ok(t: torch.Tensor) -> bool:
    return t.shape[-1] == 1 or t.stride(-1) == 1


def as_view(t: torch.Tensor) -> Tuple[fa_view, torch.Tensor]:
    """A 4-D tensor as an ``fa_view`` (strided; W stride must be 1).

    Returns the view and the tensor that owns its memory (a contiguous copy
    only when the innermost stride is not 1)."""
    if not _row_ok(t):
        t = t.contiguous()
    n, c, h, w = t.shape
    v = fa_view()
    v.data = t.data_ptr()
    v.dtype = DTYPE_CODE[t.dtype]
    v.n, v.c, v.h, v.w = int(n), int(c), int(h), int(w)
    v.stride_n, v.stride_c, v.stride_h = int(t.stride(0)), int(t.stride(1)), int(t.stride(2))
    return v, t


def same_layout(x: torch.Tensor, y: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """The kernels take one set of strides for both operands."""
    if x.stride() != y.stride() or not _row_ok(x):
        x, y = x.contiguous(), y.contiguous()
    return x, y


def _dev(t: torch.Tensor) -> int:
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _luma_arg(luma) -> Optional[ctypes.Array]:
    if luma is None:
        return None
    return (ctypes.c_double * 4)(*[float(v) for v in luma])


# --------------------------------------------------------------------------- #
# scratch
#
# Every kernel's first 256 workspace bytes are completion counters that must
# be zero on entry and are left zero on exit.  One zero-initialised buffer per
# (device, stream) therefore serves every call issued in order on that stream;
# it only ever grows.  Calls that may overlap on the GPU without being ordered
# on one stream (CUDA-graph replays of different owners, say) need separate
# buffers: private_workspaces gives an owner its own table.
# --------------------------------------------------------------------------- #

_ws: dict = {}
# A caller that replays its own CUDA graphs (StreamingMetrics) routes its calls
# to a pool of its own, so graphs and eager calls never share counters.
_ws_pool: contextvars.ContextVar = contextvars.ContextVar("fa_b200_ws_pool", default=None)


@contextlib.contextmanager
def private_workspaces(pool: dict):
    """Within this block, every workspace comes from `pool` (keyed by device
    and stream like the shared one) instead of the process-wide table."""
    token = _ws_pool.set(pool)
    try:
        yield pool
    finally:
        _ws_pool.reset(token)


def _pool() -> dict:
    p = _ws_pool.get()
    return _ws if p is None else p


def workspace(t: torch.Tensor, nbytes: int) -> torch.Tensor:
    pool = _pool()
    key = (_dev(t), _stream(t))
    buf = pool.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(int(nbytes), 1 << 16)
        if buf is not None:
            size = max(size, 2 * buf.numel())
        buf = torch.zeros(size, dtype=torch.uint8, device=t.device)
        pool[key] = buf
    return buf


def _drop_workspace(t: torch.Tensor) -> None:
    # a failed launch may leave a counter non-zero: never reuse that buffer
    _pool().pop((_dev(t), _stream(t)), None)


def _call(t: torch.Tensor, fn, *args) -> None:
    code = fn(*args)
    if code != 0:
        _drop_workspace(t)
        _cabi.check(code)


def _ws_query(fn, *args) -> int:
    out = ctypes.c_size_t(0)
    _cabi.check(fn(*args, ctypes.byref(out)))
    return int(out.value)


_wsq_cache: dict = {}


def _cached_ws(kind: str, fn, *args) -> int:
    key = (kind,) + args
    v = _wsq_cache.get(key)
    if v is None:
        v = _ws_query(fn, *args)
        _wsq_cache[key] = v
    return v


def _f64(t: torch.Tensor, *shape) -> torch.Tensor:
    return torch.empty(shape, dtype=torch.float64, device=t.device)


# --------------------------------------------------------------------------- #
# pixel reductions
# --------------------------------------------------------------------------- #

def pixel(x: torch.Tensor, y: torch.Tensor, *, op: int, param: float = 0.0,
          per_image: bool, psnr_bias: float = PSNR_NONE, luma=None,
          want_isum: bool = False):
    """One-launch pixel reduction.  Returns the (N,) or 0-d float64 result
    (PSNR when ``psnr_bias`` is given) and, if asked, the exact integer sums."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    vx, x = as_view(x)
    vy, y = as_view(y)
    n = vx.n
    dev = _dev(x)
    nb = _cached_ws("pix", L.fa_b200_pixel_workspace_bytes, n, dev)
    ws = workspace(x, nb)
    out = _f64(x, n) if per_image else _f64(x)
    want_psnr = psnr_bias != PSNR_NONE
    sinks = [None, None, None, None]
    sinks[(2 if want_psnr else 0) + (0 if per_image else 1)] = out
    isum = torch.empty(n, dtype=torch.int64, device=x.device) if want_isum else None
    _call(x, L.fa_b200_pixel_reduce, ctypes.byref(vx), ctypes.byref(vy),
          _luma_arg(luma), int(op), float(param), float(psnr_bias),
          ws.data_ptr(), ws.numel(), _ptr(sinks[0]), _ptr(sinks[1]),
          _ptr(sinks[2]), _ptr(sinks[3]), _ptr(isum), dev, _stream(x))
    return (out, isum) if want_isum else out


# --------------------------------------------------------------------------- #
# SSIM
# --------------------------------------------------------------------------- #

class Taps:
    """The 1-D Gaussian window as host taps: float32 for the float32 kernels
    (they take them by value in their launch parameters, so no device window
    is read) and float64 for the float64 kernels."""

    __slots__ = ("k", "arr", "values", "arr64")

    def __init__(self, values, values64=None):
        self.values = tuple(float(v) for v in values)
        self.k = len(self.values)
        self.arr = (ctypes.c_float * self.k)(*self.values)
        v64 = self.values if values64 is None else tuple(float(v) for v in values64)
        self.arr64 = (ctypes.c_double * self.k)(*v64)


@functools.lru_cache(maxsize=64)
def gaussian_taps(win_size: int, sigma: float) -> Tuple[float, ...]:
    """The SSIM window in float64: exp(-t^2 / (2 sigma^2)) at
    t = -(K-1)/2 .. (K-1)/2, divided by its sum (functional.py:397-420 of the
    reference)."""
    half = 0.5 * (win_size - 1)
    raw = [math.exp(-0.5 * ((i - half) / sigma) ** 2) for i in range(win_size)]
    total = math.fsum(raw)
    return tuple(v / total for v in raw)


@functools.lru_cache(maxsize=64)
def host_taps(win_size: int, sigma: float) -> Taps:
    """gaussian_taps rounded to float32: the same numbers as
    functional.gaussian_window_1d(..., dtype=torch.float32)."""
    g = gaussian_taps(int(win_size), float(sigma))
    f32 = torch.tensor(g, dtype=torch.float64).to(torch.float32)
    return Taps(f32.tolist(), g)


def ssim_forward(x: torch.Tensor, y: torch.Tensor, win: Taps, *,
                 shift: float, C1: float, C2: float, luma=None,
                 want_map: bool = False, want_plane: bool = False,
                 want_cs: bool = False, want_per_image: bool = False,
                 want_total: bool = False) -> dict:
    """Fused SSIM forward, one launch.  ``win`` holds the window taps.
    Returns a dict with the requested outputs.  float64 frames go to the
    float64 kernels (everything, the map included, in double)."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    if x.dtype == torch.float64:
        return _ssim64_forward(x, y, win, C1=C1, C2=C2, luma=luma, want_map=want_map,
                               want_plane=want_plane or want_cs, want_cs=want_cs,
                               want_per_image=want_per_image, want_total=want_total)
    vx, x = as_view(x)
    vy, y = as_view(y)
    k = win.k
    cm = 1 if luma is not None else vx.c
    hout, wout = vx.h - k + 1, vx.w - k + 1
    if hout <= 0 or wout <= 0:
        raise ValueError(f"image {(vx.h, vx.w)} smaller than window {k}x{k}")
    dev = _dev(x)
    nb = _cached_ws("ssim", L.fa_b200_ssim_workspace_bytes, vx.n, cm, vx.h, vx.w, k, dev)
    ws = workspace(x, nb)
    res = {}
    res["map"] = (torch.empty((vx.n, cm, hout, wout), dtype=torch.float32,
                              device=x.device) if want_map else None)
    res["plane_s"] = _f64(x, vx.n * cm) if (want_plane or want_cs) else None
    res["plane_cs"] = _f64(x, vx.n * cm) if want_cs else None
    res["per_image"] = _f64(x, vx.n) if want_per_image else None
    res["total"] = _f64(x) if want_total else None
    _call(x, L.fa_b200_ssim, ctypes.byref(vx), ctypes.byref(vy), _luma_arg(luma),
          win.arr, k, float(shift), float(C1), float(C2), _ptr(res["map"]),
          ws.data_ptr(), ws.numel(), _ptr(res["plane_s"]), _ptr(res["plane_cs"]),
          _ptr(res["per_image"]), _ptr(res["total"]), dev, _stream(x))
    return res


def ssim_mse(x: torch.Tensor, y: torch.Tensor, win: Taps, *, shift: float, C1: float,
             C2: float, psnr_bias: float, per_image: bool) -> dict:
    """SSIM, MSE and PSNR from one read of the frame pair (one launch).
    Returns a dict of float64 tensors, (N,) when ``per_image`` else 0-d; uint8
    input also gives the exact per-image sums of squared differences."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    vx, x = as_view(x)
    vy, y = as_view(y)
    k = win.k
    if vx.h - k + 1 <= 0 or vx.w - k + 1 <= 0:
        raise ValueError(f"image {(vx.h, vx.w)} smaller than window {k}x{k}")
    dev = _dev(x)
    nb = _cached_ws("ssim", L.fa_b200_ssim_workspace_bytes, vx.n, vx.c, vx.h, vx.w, k, dev)
    ws = workspace(x, nb)
    shape = (vx.n,) if per_image else ()
    res = {"ssim": _f64(x, *shape), "mse": _f64(x, *shape), "psnr": _f64(x, *shape)}
    res["ssd"] = (torch.empty(vx.n, dtype=torch.int64, device=x.device)
                  if x.dtype == torch.uint8 else None)
    pi = (lambda t: t) if per_image else (lambda t: None)
    tot = (lambda t: None) if per_image else (lambda t: t)
    _call(x, L.fa_b200_ssim_mse, ctypes.byref(vx), ctypes.byref(vy), win.arr, k,
          float(shift), float(C1), float(C2), float(psnr_bias), ws.data_ptr(), ws.numel(),
          None, _ptr(pi(res["ssim"])), _ptr(tot(res["ssim"])), _ptr(pi(res["mse"])),
          _ptr(tot(res["mse"])), _ptr(pi(res["psnr"])), _ptr(tot(res["psnr"])),
          _ptr(res["ssd"]), dev, _stream(x))
    return res


def ssim_gmsd_fusable(x: torch.Tensor, y: torch.Tensor, k: int) -> bool:
    """Whether ssim_gmsd serves this pair (see fa_b200_ssim_gmsd_fusable)."""
    L = lib()
    if kernel_dtype(x).dtype not in (torch.uint8, torch.float32):
        return False
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    vx, x = as_view(x)
    vy, y = as_view(y)
    ok = ctypes.c_int(0)
    _cabi.check(L.fa_b200_ssim_gmsd_fusable(ctypes.byref(vx), ctypes.byref(vy), int(k),
                                            _dev(x), ctypes.byref(ok)))
    return bool(ok.value)


def ssim_gmsd(x: torch.Tensor, y: torch.Tensor, win: Taps, *, shift: float, C1: float,
              C2: float, T: float, eps: float, psnr_bias: float, per_image: bool,
              want_mse: bool) -> dict:
    """SSIM and GMSD / GMS (2x2 pool) of one pair from ONE read (one launch),
    plus MSE / PSNR when ``want_mse``.  SSIM / MSE / PSNR are (N,) when
    ``per_image`` else 0-d; GMS and GMSD are always per image (N,)."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    vx, x = as_view(x)
    vy, y = as_view(y)
    k = win.k
    dev = _dev(x)
    nb = _cached_ws("ssim", L.fa_b200_ssim_workspace_bytes, vx.n, vx.c, vx.h, vx.w, k, dev)
    ws = workspace(x, nb)
    shape = (vx.n,) if per_image else ()
    res = {"ssim": _f64(x, *shape), "gms": _f64(x, vx.n), "gmsd": _f64(x, vx.n)}
    if want_mse:
        res["mse"], res["psnr"] = _f64(x, *shape), _f64(x, *shape)
        res["ssd"] = (torch.empty(vx.n, dtype=torch.int64, device=x.device)
                      if x.dtype == torch.uint8 else None)
    pi = (lambda t: t) if per_image else (lambda t: None)
    tot = (lambda t: None) if per_image else (lambda t: t)
    m, p_ = res.get("mse"), res.get("psnr")
    _call(x, L.fa_b200_ssim_gmsd, ctypes.byref(vx), ctypes.byref(vy), win.arr, k,
          float(shift), float(C1), float(C2), float(T), float(eps), float(psnr_bias),
          ws.data_ptr(), ws.numel(), None, _ptr(pi(res["ssim"])), _ptr(tot(res["ssim"])),
          _ptr(res["gms"]), _ptr(res["gmsd"]),
          _ptr(pi(m) if m is not None else None), _ptr(tot(m) if m is not None else None),
          _ptr(pi(p_) if p_ is not None else None), _ptr(tot(p_) if p_ is not None else None),
          _ptr(res.get("ssd")), dev, _stream(x))
    return res


def ssim_backward(x: torch.Tensor, y: torch.Tensor, win: Taps, *,
                  shift: float, C1: float, C2: float,
                  dmap: Optional[torch.Tensor] = None,
                  gscalar: Optional[torch.Tensor] = None,
                  gs: Optional[torch.Tensor] = None,
                  gcs: Optional[torch.Tensor] = None,
                  need_dx: bool = True, need_dy: bool = True):
    """Fused SSIM backward (no scratch).  x, y: float32 (N,C,H,W); float64
    frames take the float64 kernels (scratch: four coefficient planes)."""
    L = lib()
    if x.dtype == torch.float64:
        return _ssim64_backward(x, y, win, C1=C1, C2=C2, dmap=dmap, gscalar=gscalar, gs=gs,
                                gcs=gcs, need_dx=need_dx, need_dy=need_dy)
    x = x.detach().to(torch.float32).contiguous()
    y = y.detach().to(torch.float32).contiguous()
    n, c, h, w = x.shape
    k = win.k
    dx = torch.empty_like(x) if need_dx else None
    dy = torch.empty_like(y) if need_dy else None
    if dmap is not None:
        dmap = dmap.to(torch.float32).contiguous()
    if gscalar is not None:
        gscalar = gscalar.to(torch.float32).reshape(1).contiguous()
    if gs is not None:
        gs = gs.to(torch.float32).reshape(-1).contiguous()
        gcs = gcs.to(torch.float32).reshape(-1).contiguous()
    _call(x, L.fa_b200_ssim_backward, x.data_ptr(), y.data_ptr(), n, c, h, w,
          win.arr, k, float(shift), float(C1), float(C2), _ptr(dmap),
          _ptr(gscalar), _ptr(gs), _ptr(gcs), _ptr(dx), _ptr(dy), _dev(x), _stream(x))
    return dx, dy


def ssim_loss_grad(x: torch.Tensor, y: torch.Tensor, win: Taps, *, shift: float,
                   C1: float, C2: float, need_dx: bool = True, need_dy: bool = True,
                   want_per_image: bool = False, upstream: float = 1.0):
    """SSIM means and the gradient of the batch-mean SSIM for the upstream
    gradient ``upstream`` (1: the unit gradient), one launch.
    Returns ``(total, per_image or None, dx, dy)``; x, y float32 (N,C,H,W)."""
    L = lib()
    x = x.detach().to(torch.float32).contiguous()
    y = y.detach().to(torch.float32).contiguous()
    n, c, h, w = x.shape
    k = win.k
    if h - k + 1 <= 0 or w - k + 1 <= 0:
        raise ValueError(f"image {(h, w)} smaller than window {k}x{k}")
    dev = _dev(x)
    nb = _cached_ws("ssim_lg", L.fa_b200_ssim_loss_grad_workspace_bytes, n, c, h, w, k, dev)
    ws = workspace(x, nb)
    total = _f64(x)
    per_image = _f64(x, n) if want_per_image else None
    dx = torch.empty_like(x) if need_dx else None
    dy = torch.empty_like(y) if need_dy else None
    _call(x, L.fa_b200_ssim_loss_grad, x.data_ptr(), y.data_ptr(), n, c, h, w, win.arr, k,
          float(shift), float(C1), float(C2), float(upstream), ws.data_ptr(), ws.numel(), None,
          _ptr(per_image), total.data_ptr(), _ptr(dx), _ptr(dy), dev, _stream(x))
    return total, per_image, dx, dy


def grad_scale(unit: torch.Tensor, g: torch.Tensor, *, per_image: bool,
               mult: float = 1.0, inplace: bool = False) -> torch.Tensor:
    """``unit * g * mult`` (``g`` one scalar, or one value per image when
    ``per_image``); ``g`` stays on the device.  A new float32 tensor, or
    ``unit`` itself rescaled when ``inplace`` (a factor of exactly 1 then
    costs no memory traffic)."""
    L = lib()
    n = unit.shape[0]
    gd = g.detach().to(torch.float64).reshape(-1).contiguous()
    out = unit if inplace else torch.empty_like(unit)
    _call(unit, L.fa_b200_grad_scale, unit.data_ptr(), unit.numel() // n, n, gd.data_ptr(),
          int(bool(per_image)), float(mult), out.data_ptr(), _dev(unit), _stream(unit))
    return out


# --------------------------------------------------------------------------- #
# GMSD
# --------------------------------------------------------------------------- #

# --------------------------------------------------------------------------- #
# float64 frames
# --------------------------------------------------------------------------- #

def _ssim64_forward(x, y, win: Taps, *, C1, C2, luma, want_map, want_plane, want_cs,
                    want_per_image, want_total) -> dict:
    L = lib()
    vx, x = as_view(x)
    vy, y = as_view(y)
    k = win.k
    cm = 1 if luma is not None else vx.c
    hout, wout = vx.h - k + 1, vx.w - k + 1
    if hout <= 0 or wout <= 0:
        raise ValueError(f"image {(vx.h, vx.w)} smaller than window {k}x{k}")
    nb = _cached_ws("ssim64", L.fa_b200_ssim64_workspace_bytes, vx.n, vx.c, vx.h, vx.w, k,
                    int(luma is not None))
    ws = workspace(x, nb)
    res = {"map": _f64(x, vx.n, cm, hout, wout) if want_map else None,
           "plane_s": _f64(x, vx.n * cm) if want_plane else None,
           "plane_cs": _f64(x, vx.n * cm) if want_cs else None,
           "per_image": _f64(x, vx.n) if want_per_image else None,
           "total": _f64(x) if want_total else None}
    _call(x, L.fa_b200_ssim64, ctypes.byref(vx), ctypes.byref(vy), _luma_arg(luma), win.arr64,
          k, float(C1), float(C2), ws.data_ptr(), ws.numel(), _ptr(res["map"]),
          _ptr(res["plane_s"]), _ptr(res["plane_cs"]), _ptr(res["per_image"]),
          _ptr(res["total"]), _dev(x), _stream(x))
    return res


def _ssim64_backward(x, y, win: Taps, *, C1, C2, dmap, gscalar, gs, gcs, need_dx, need_dy):
    L = lib()
    x = x.detach().contiguous()
    y = y.detach().contiguous()
    n, c, h, w = x.shape
    k = win.k
    coef = torch.empty((4, n * c, h - k + 1, w - k + 1), dtype=torch.float64, device=x.device)
    dx = torch.empty_like(x) if need_dx else None
    dy = torch.empty_like(y) if need_dy else None

    def d64(t, flat=True):
        if t is None:
            return None
        t = t.detach().to(torch.float64)
        return (t.reshape(-1) if flat else t).contiguous()

    _call(x, L.fa_b200_ssim64_backward, x.data_ptr(), y.data_ptr(), n, c, h, w, win.arr64, k,
          float(C1), float(C2), _ptr(d64(dmap)), _ptr(d64(gscalar)), _ptr(d64(gs)),
          _ptr(d64(gcs)), coef.data_ptr(), _ptr(dx), _ptr(dy), _dev(x), _stream(x))
    return dx, dy


def _gmsd64(x, y, *, T, eps, downsample, luma, want_map):
    L = lib()
    vx, x = as_view(x)
    vy, y = as_view(y)
    cm = 1 if luma is not None else vx.c
    nb = _cached_ws("gmsd64", L.fa_b200_gmsd64_workspace_bytes, vx.n, vx.c, vx.h, vx.w,
                    int(bool(downsample)), int(luma is not None), _dev(x))
    ws = workspace(x, nb)
    mean, std = _f64(x, vx.n), _f64(x, vx.n)
    qmap = None
    if want_map:
        hd = vx.h // 2 if downsample else vx.h
        wd = vx.w // 2 if downsample else vx.w
        qmap = _f64(x, vx.n, cm, hd - 2, wd - 2)
    _call(x, L.fa_b200_gmsd64, ctypes.byref(vx), ctypes.byref(vy), _luma_arg(luma), float(T),
          float(eps), int(bool(downsample)), ws.data_ptr(), ws.numel(), _ptr(qmap),
          mean.data_ptr(), std.data_ptr(), _dev(x), _stream(x))
    return (mean, std, qmap) if want_map else (mean, std)


def _gmsd64_backward(x, y, *, T, eps, downsample, mean, std, g_mean, g_std, need_dx, need_dy):
    L = lib()
    x = x.detach().contiguous()
    y = y.detach().contiguous()
    n, c, h, w = x.shape
    hd, wd = (h // 2, w // 2) if downsample else (h, w)
    coef = torch.empty((4, n * c, hd - 2, wd - 2), dtype=torch.float64, device=x.device)
    dx = torch.empty_like(x) if need_dx else None
    dy = torch.empty_like(y) if need_dy else None
    zero = torch.zeros(n, dtype=torch.float64, device=x.device)

    def d64(t):
        return zero if t is None else t.detach().to(torch.float64).reshape(-1).contiguous()

    _call(x, L.fa_b200_gmsd64_backward, x.data_ptr(), y.data_ptr(), n, c, h, w,
          int(bool(downsample)), float(T), float(eps), d64(g_mean).data_ptr(),
          d64(g_std).data_ptr(), d64(mean).data_ptr(), d64(std).data_ptr(), coef.data_ptr(),
          _ptr(dx), _ptr(dy), _dev(x), _stream(x))
    return dx, dy


def gmsd(x: torch.Tensor, y: torch.Tensor, *, T: float, eps: float,
         downsample: bool, luma=None, want_map: bool = False):
    """``(gms_mean, gmsd)`` per image, float64, one launch (plus the float32
    GMS map when ``want_map``; float64 frames: the float64 kernels, float64
    map)."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    if x.dtype == torch.float64:
        return _gmsd64(x, y, T=T, eps=eps, downsample=downsample, luma=luma, want_map=want_map)
    vx, x = as_view(x)
    vy, y = as_view(y)
    cm = 1 if luma is not None else vx.c
    dev = _dev(x)
    nb = _cached_ws("gmsd", L.fa_b200_gmsd_workspace_bytes, vx.n, cm, vx.h, vx.w,
                    int(bool(downsample)), dev)
    ws = workspace(x, nb)
    mean = _f64(x, vx.n)
    std = _f64(x, vx.n)
    qmap = None
    if want_map:
        hd = vx.h // 2 if downsample else vx.h
        wd = vx.w // 2 if downsample else vx.w
        qmap = torch.empty((vx.n, cm, hd - 2, wd - 2), dtype=torch.float32, device=x.device)
    _call(x, L.fa_b200_gmsd, ctypes.byref(vx), ctypes.byref(vy), _luma_arg(luma),
          float(T), float(eps), int(bool(downsample)), ws.data_ptr(), ws.numel(),
          _ptr(qmap), mean.data_ptr(), std.data_ptr(), dev, _stream(x))
    if want_map:
        return mean, std, qmap
    return mean, std


def gms_map(x, y, *, T: float, eps: float, downsample: bool, luma=None) -> torch.Tensor:
    """The (N, C', H'-2, W'-2) GMS map (float32; float64 for float64 frames)."""
    return gmsd(x, y, T=T, eps=eps, downsample=downsample, luma=luma, want_map=True)[2]


# --------------------------------------------------------------------------- #
# SSIMULACRA 2
# --------------------------------------------------------------------------- #

def ssimulacra2(x: torch.Tensor, y: torch.Tensor, *, data_range: float, f64: bool, weights,
                per_image: bool) -> torch.Tensor:
    """SSIMULACRA 2 of (N, 3, H, W) sRGB pairs (any dtype and strides; channel
    stride 0 for a replicated gray plane): float64 scores, (N,) or 0-d."""
    L = lib()
    x, y = same_layout(kernel_dtype(x), kernel_dtype(y))
    vx, x = as_view(x)
    vy, y = as_view(y)
    nb = _cached_ws("su2", L.fa_b200_ssimulacra2_workspace_bytes, vx.n, vx.h, vx.w, int(f64))
    ws = workspace(x, nb)
    out = _f64(x, vx.n) if per_image else _f64(x)
    _call(x, L.fa_b200_ssimulacra2, ctypes.byref(vx), ctypes.byref(vy), float(data_range),
          int(f64), weights, ws.data_ptr(), ws.numel(), _ptr(out) if per_image else None,
          None if per_image else out.data_ptr(), _dev(x), _stream(x))
    return out


# --------------------------------------------------------------------------- #
# MS-SSIM pyramid pooling
# --------------------------------------------------------------------------- #

def pool2(x: torch.Tensor, luma=None) -> torch.Tensor:
    """2x2 mean pool to float32 (``F.avg_pool2d(x.float(), 2)``), one read of
    ``x`` in its own dtype and strides; ``luma`` projects RGB first.  float64
    planes pool to float64 (no luma: project first)."""
    L = lib()
    if x.dtype == torch.float64:
        if luma is not None:
            raise ValueError("float64 pooling takes luma planes, not RGB")
        x = x.contiguous()
        n, c, h, w = x.shape
        out = torch.empty((n, c, h // 2, w // 2), dtype=torch.float64, device=x.device)
        _call(x, L.fa_b200_pool64, x.data_ptr(), n * c, h, w, out.data_ptr(), _dev(x),
              _stream(x))
        return out
    vx, x = as_view(kernel_dtype(x))
    cm = 1 if luma is not None else vx.c
    out = torch.empty((vx.n, cm, vx.h // 2, vx.w // 2), dtype=torch.float32, device=x.device)
    _call(x, L.fa_b200_pool2, ctypes.byref(vx), _luma_arg(luma), out.data_ptr(), _dev(x),
          _stream(x))
    return out


def box_downsample(x: torch.Tensor, f: int, luma=None) -> torch.Tensor:
    """MATLAB-mode f x f box downsample (replicated borders) to float32."""
    L = lib()
    vx, x = as_view(kernel_dtype(x))
    cm = 1 if luma is not None else vx.c
    pad = f // 2
    ho = (vx.h + 2 * pad - f + 1 + f - 1) // f
    wo = (vx.w + 2 * pad - f + 1 + f - 1) // f
    out = torch.empty((vx.n, cm, ho, wo), dtype=torch.float32, device=x.device)
    _call(x, L.fa_b200_box_downsample, ctypes.byref(vx), _luma_arg(luma), int(f),
          out.data_ptr(), _dev(x), _stream(x))
    return out


def box_downsample_backward(g: torch.Tensor, shape, f: int) -> torch.Tensor:
    """Adjoint of :func:`box_downsample` for a float32 input of ``shape``."""
    L = lib()
    g = g.detach().to(torch.float32).contiguous()
    n, c, h, w = shape
    dx = torch.empty((n, c, h, w), dtype=torch.float32, device=g.device)
    _call(g, L.fa_b200_box_downsample_backward, g.data_ptr(), n, c, h, w, int(f),
          dx.data_ptr(), _dev(g), _stream(g))
    return dx


def pool2_backward(g: torch.Tensor, shape) -> torch.Tensor:
    """Adjoint of :func:`pool2` for an input of ``shape`` (float32, or
    float64 when ``g`` is float64)."""
    L = lib()
    if g.dtype == torch.float64:
        g = g.detach().contiguous()
        n, c, h, w = shape
        dx = torch.empty((n, c, h, w), dtype=torch.float64, device=g.device)
        _call(g, L.fa_b200_pool64_backward, g.data_ptr(), n * c, h, w, dx.data_ptr(), _dev(g),
              _stream(g))
        return dx
    g = g.detach().to(torch.float32).contiguous()
    n, c, h, w = shape
    dx = torch.empty((n, c, h, w), dtype=torch.float32, device=g.device)
    _call(g, L.fa_b200_pool2_backward, g.data_ptr(), n, c, h, w, dx.data_ptr(), _dev(g),
          _stream(g))
    return dx


# --------------------------------------------------------------------------- #
# pixel-loss backward
# --------------------------------------------------------------------------- #

def pixel_loss_grad(x: torch.Tensor, y: torch.Tensor, *, op: int, param: float,
                    per_image: bool, need_dx: bool = True, need_dy: bool = True):
    """A pixel loss and its gradient (for an upstream gradient of 1) from one
    read; x, y contiguous float32 (N, ...).  Returns (value, dx, dy)."""
    L = lib()
    n = x.shape[0]
    per = x.numel() // n
    dev = _dev(x)
    nb = _cached_ws("pix", L.fa_b200_pixel_workspace_bytes, n, dev)
    ws = workspace(x, nb)
    out = _f64(x, n) if per_image else _f64(x)
    dx = torch.empty_like(x) if need_dx else None
    dy = torch.empty_like(y) if need_dy else None
    _call(x, L.fa_b200_pixel_loss_grad, x.data_ptr(), y.data_ptr(), n, per, int(op),
          float(param), int(bool(per_image)), ws.data_ptr(), ws.numel(),
          _ptr(out) if per_image else None, None if per_image else out.data_ptr(),
          _ptr(dx), _ptr(dy), dev, _stream(x))
    return out, dx, dy


def pixel_backward(x, y, g, *, op: int, param: float, per_image: bool, luma=None,
                   need_dx: bool = True, need_dy: bool = True):
    """Gradients of a pixel reduction w.r.t. x and y, in the inputs' dtypes."""
    L = lib()
    xf = x.detach().to(torch.float32).contiguous()
    yf = y.detach().to(torch.float32).contiguous()
    n, c, h, w = xf.shape
    gd = g.detach().to(torch.float64).reshape(-1).contiguous()
    dx = torch.empty_like(xf) if need_dx else None
    dy = torch.empty_like(yf) if need_dy else None
    _call(xf, L.fa_b200_pixel_backward, xf.data_ptr(), yf.data_ptr(), n, c, h, w,
          _luma_arg(luma), int(op), float(param), gd.data_ptr(), int(bool(per_image)),
          _ptr(dx), _ptr(dy), _dev(xf), _stream(xf))
    return (dx.to(x.dtype) if need_dx else None, dy.to(y.dtype) if need_dy else None)


def gmsd_backward(x, y, *, T: float, eps: float, downsample: bool, mean, std,
                  g_mean=None, g_std=None, need_dx: bool = True, need_dy: bool = True):
    """Gradients of the per-image GMS (mean) and GMSD (std) w.r.t. x and y."""
    L = lib()
    if x.dtype == torch.float64:
        return _gmsd64_backward(x, y, T=T, eps=eps, downsample=downsample, mean=mean, std=std,
                                g_mean=g_mean, g_std=g_std, need_dx=need_dx, need_dy=need_dy)
    xf = x.detach().to(torch.float32).contiguous()
    yf = y.detach().to(torch.float32).contiguous()
    n, c, h, w = xf.shape
    odd = downsample and (h % 2 or w % 2)
    alloc = torch.zeros_like if odd else torch.empty_like
    dx = alloc(xf) if need_dx else None
    dy = alloc(yf) if need_dy else None

    def d64(t):
        return None if t is None else t.detach().to(torch.float64).reshape(-1).contiguous()

    gm, gs, mu, sd = d64(g_mean), d64(g_std), d64(mean), d64(std)
    _call(xf, L.fa_b200_gmsd_backward, xf.data_ptr(), yf.data_ptr(), n, c, h, w,
          int(bool(downsample)), float(T), float(eps), _ptr(gm), _ptr(gs), _ptr(mu), _ptr(sd),
          _ptr(dx), _ptr(dy), _dev(xf), _stream(xf))
    return (dx.to(x.dtype) if need_dx else None, dy.to(y.dtype) if need_dy else None)

"""Planar video frames: zero-copy plane views and the per-frame scorer of the
reference's VapourSynth binding, without VapourSynth.

The reference's ``vapoursynth._Runner.scores`` (frame_analytics/vapoursynth.py:
275-338) turns each plane of a clip's frame into a ``(1, 1, H, W)`` tensor --
8-bit as uint8, 10-16-bit widened to float32 after the copy -- then runs the
per-plane metrics on every plane (property ``<prop>_y`` / ``_cb`` / ``_cr``)
and the image metrics on the luma plane of GRAY/YUV clips or on all three
channels of RGB clips.  Here:

* :func:`frame_planes` cuts the planes of one packed planar frame buffer
  (GRAY, YUV 4:2:0 / 4:2:2 / 4:4:4, planar RGB; uint8 or uint16) into views
  without copying anything;
* :class:`PlaneScorer` scores a pair of frames the way ``_Runner.scores``
  does, with the same feature ids, names and property names.  uint16 planes
  are read as they are (exact integer MSE) instead of being widened to
  float32 first, and the luma plane is read directly, with no RGB projection.

The VapourSynth clip / frame plumbing itself (``vs`` module, frame props,
logging) is not part of this package.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import functional as F

__all__ = ["FEATURES", "available_features", "resolve_features", "frame_planes",
           "PlaneScorer", "LAYOUTS"]


class Feature:
    """One scorable feature: ``kind`` is ``per_plane`` (every plane at its
    own resolution, property gets a plane suffix), ``image`` (luma of a
    GRAY/YUV frame, all channels of an RGB frame) or ``rgb`` (RGB only)."""

    __slots__ = ("id", "name", "kind", "prop", "takes_range")

    def __init__(self, id_: int, name: str, kind: str, prop: str, takes_range: bool = True):
        self.id, self.name, self.kind, self.prop = id_, name, kind, prop
        self.takes_range = takes_range


# Ids, names and property names of the reference's feature table
# (vapoursynth.py:148-183), which follow the VapourSynth-VMAF plugin.
FEATURES: Tuple[Feature, ...] = (
    Feature(0, "psnr", "per_plane", "psnr"),
    Feature(2, "ssim", "image", "float_ssim"),
    Feature(3, "ms_ssim", "image", "float_ms_ssim"),
    Feature(5, "gmsd", "image", "gmsd"),
    Feature(6, "gms", "image", "gms"),
    Feature(7, "mse", "per_plane", "mse", takes_range=False),
    Feature(8, "l1", "per_plane", "l1", takes_range=False),
    Feature(9, "charbonnier", "per_plane", "charbonnier", takes_range=False),
    Feature(10, "huber", "per_plane", "huber", takes_range=False),
    Feature(12, "ssimulacra2", "rgb", "ssimulacra2"),
)
_NAMED = {f.name: f for f in FEATURES}
_NUMBERED = {f.id: f for f in FEATURES}
# features of the reference this package does not compute, with why
_ABSENT = {1: "psnr_hvs (a libvmaf feature)", 4: "ciede2000 (a libvmaf feature)",
           11: "lpips (not part of this package)"}
_SUFFIXES = {"gray": ("_y",), "yuv": ("_y", "_cb", "_cr"), "rgb": ("_r", "_g", "_b")}


def available_features() -> Dict[str, int]:
    """``{name: id}`` of every feature :class:`PlaneScorer` computes."""
    return {f.name: f.id for f in FEATURES}


def resolve_features(feature) -> List[Feature]:
    """An id, a name, or a sequence of them -> the features, in order and
    without repeats (vapoursynth.py:186-235 of the reference: same errors)."""
    if feature is None:
        raise ValueError(f"feature is required (an id or a name); available: {sorted(_NAMED)}")
    if isinstance(feature, (str, int, np.integer)) and not isinstance(feature, bool):
        feature = [feature]
    if not isinstance(feature, Iterable):
        raise TypeError(f"feature must be an int, a str or a sequence of them, "
                        f"got {type(feature).__name__}")
    out: List[Feature] = []
    for item in feature:
        if isinstance(item, str):
            key = item.strip().lower().replace("-", "_")
            if key == "lpips":
                raise ValueError(f"feature {item!r}: {_ABSENT[11]}")
            if key not in _NAMED:
                raise ValueError(f"unknown feature {item!r}; expected one of {sorted(_NAMED)}")
            f = _NAMED[key]
        elif isinstance(item, (int, np.integer)) and not isinstance(item, bool):
            i = int(item)
            if i in _ABSENT:
                raise ValueError(f"feature {i} is {_ABSENT[i]}; no implementation here")
            if i not in _NUMBERED:
                raise ValueError(f"unknown feature id {i}; expected one of {sorted(_NUMBERED)}")
            f = _NUMBERED[i]
        else:
            raise TypeError(f"feature entries must be int or str, got {type(item).__name__}")
        if f not in out:
            out.append(f)
    if not out:
        raise ValueError("feature is empty; nothing to compute")
    return out


# planar layouts: family, (chroma width divisor, chroma height divisor)
LAYOUTS = {
    "gray": ("gray", None),
    "yuv420p": ("yuv", (2, 2)),
    "yuv422p": ("yuv", (2, 1)),
    "yuv444p": ("yuv", (1, 1)),
    "rgbp": ("rgb", (1, 1)),
}


def frame_planes(buf: torch.Tensor, width: int, height: int,
                 layout: str = "yuv420p") -> Tuple[torch.Tensor, ...]:
    """Views of the planes of one packed planar frame (no copy).

    ``buf`` is a 1-D uint8 or uint16 tensor holding the planes back to back
    (Y then Cb then Cr for YUV; R, G, B for ``rgbp``), as a decoder or a
    frame server hands them over; chroma planes of 4:2:0 / 4:2:2 have
    ceil(width / 2) columns (and ceil(height / 2) rows for 4:2:0).  Each
    plane comes back as ``(1, 1, h, w)``, ready for the metric functions."""
    if layout not in LAYOUTS:
        raise ValueError(f"unknown layout {layout!r}; expected one of {sorted(LAYOUTS)}")
    if buf.ndim != 1:
        raise ValueError(f"frame buffer must be 1-D, got shape {tuple(buf.shape)}")
    fam, sub = LAYOUTS[layout]
    sizes = [(height, width)]
    if sub is not None:
        cw, ch = -(-width // sub[0]), -(-height // sub[1])
        sizes += [(ch, cw), (ch, cw)]
    need = sum(h * w for h, w in sizes)
    if buf.numel() < need:
        raise ValueError(f"a {width}x{height} {layout} frame needs {need} samples, "
                         f"the buffer holds {buf.numel()}")
    out, off = [], 0
    for h, w in sizes:
        out.append(buf.narrow(0, off, h * w).view(1, 1, h, w))
        off += h * w
    return tuple(out)


_PER_PLANE = {"psnr": F.psnr, "mse": F.mse, "l1": F.l1, "charbonnier": F.charbonnier,
              "huber": F.huber}
_IMAGE = {"ssim": F.ssim, "ms_ssim": F.ms_ssim, "gmsd": F.gmsd, "gms": F.gms,
          "ssimulacra2": F._ssimulacra2()}


class PlaneScorer:
    """Per-frame scores of a reference / distorted pair of planar frames, as
    the reference's VapourSynth ``Metric`` reports them (frame property name
    -> float).

    ``family`` is ``"gray"``, ``"yuv"`` or ``"rgb"``; ``bits`` the sample
    depth of integer planes (``data_range`` defaults to 2**bits - 1, 1.0 for
    float planes); ``options`` maps a feature name to extra keyword arguments
    of its function."""

    def __init__(self, feature, family: str = "yuv", *, bits: Optional[int] = None,
                 data_range: Optional[float] = None, crop_border: int = 0,
                 options: Optional[Dict[str, dict]] = None):
        if family not in _SUFFIXES:
            raise ValueError(f"family must be one of {sorted(_SUFFIXES)}, got {family!r}")
        self.features = resolve_features(feature)
        self.family = family
        self.bits = bits
        self.data_range = data_range
        self.crop_border = int(crop_border)
        self.options = dict(options or {})
        for f in self.features:
            if f.kind == "rgb" and family != "rgb":
                raise ValueError(f"{f.name} needs RGB planes")

    @property
    def prop_names(self) -> List[str]:
        names = []
        n = len(_SUFFIXES[self.family])
        for f in self.features:
            if f.kind == "per_plane":
                names += [f.prop + s for s in _SUFFIXES[self.family][:n]]
            else:
                names.append(f.prop)
        return names

    def _range(self, t: torch.Tensor) -> float:
        if self.data_range is not None:
            return float(self.data_range)
        if t.is_floating_point():
            return 1.0
        bits = self.bits if self.bits is not None else 8 * t.element_size()
        return float((1 << bits) - 1)

    def _kw(self, f: Feature, L: float) -> dict:
        kw = {"crop_border": self.crop_border}
        if f.takes_range:
            kw["data_range"] = L
        kw.update(self.options.get(f.name, {}))
        return kw

    def scores(self, ref: Sequence[torch.Tensor], dist: Sequence[torch.Tensor]) -> Dict[str, float]:
        """``ref`` / ``dist``: the planes of one frame each (Y[, Cb, Cr] or
        R, G, B), any of (H, W) / (1, H, W) / (1, 1, H, W), on the device."""
        ref, dist = list(ref), list(dist)
        nplanes = len(_SUFFIXES[self.family])
        if len(ref) != nplanes or len(dist) != nplanes:
            raise ValueError(f"a {self.family} frame has {nplanes} planes; got "
                             f"{len(ref)} and {len(dist)}")
        out: Dict[str, float] = {}
        L = self._range(ref[0])
        per = [f for f in self.features if f.kind == "per_plane"]
        with torch.inference_mode():
            for i, sfx in enumerate(_SUFFIXES[self.family]):
                x, y = ref[i], dist[i]
                for f in per:
                    out[f.prop + sfx] = float(_PER_PLANE[f.name](x, y, **self._kw(f, L)))
            image = [f for f in self.features if f.kind in ("image", "rgb")]
            if image:
                if self.family == "rgb":
                    x = torch.cat([F._as_nchw(p) for p in ref], 1)
                    y = torch.cat([F._as_nchw(p) for p in dist], 1)
                else:  # the luma plane, read in place
                    x, y = ref[0], dist[0]
                for f in image:
                    out[f.prop] = float(_IMAGE[f.name](x, y, **self._kw(f, L)))
        return out

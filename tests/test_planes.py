"""Planar frames without a GPU: plane views of packed buffers and the feature
table of the reference's VapourSynth binding (vapoursynth.py:148-235)."""

from __future__ import annotations

import pytest
import torch

from frame_analytics_b200 import planes


@pytest.mark.parametrize("layout,w,h,chroma", [("yuv420p", 7, 5, (3, 4)),
                                               ("yuv422p", 8, 6, (6, 4)),
                                               ("yuv444p", 5, 3, (3, 5)),
                                               ("gray", 9, 4, None)])
@pytest.mark.parametrize("dt", [torch.uint8, torch.uint16])
def test_frame_planes_are_views(layout, w, h, chroma, dt):
    n = h * w + (0 if chroma is None else 2 * chroma[0] * chroma[1])
    buf = torch.arange(n, dtype=torch.int32).to(dt)
    ps = planes.frame_planes(buf, w, h, layout)
    assert ps[0].shape == (1, 1, h, w)
    assert ps[0].data_ptr() == buf.data_ptr()
    assert torch.equal(ps[0].reshape(-1), buf[:h * w])
    if chroma is not None:
        assert ps[1].shape == ps[2].shape == (1, 1) + chroma
        off = h * w + chroma[0] * chroma[1]
        assert ps[2].data_ptr() == buf.data_ptr() + off * buf.element_size()
    with pytest.raises(ValueError):
        planes.frame_planes(buf[:-1], w, h, layout)


def test_feature_resolution_matches_the_reference_table():
    assert [f.prop for f in planes.resolve_features([0, "ssim", 3, "gmsd"])] == \
        ["psnr", "float_ssim", "float_ms_ssim", "gmsd"]
    assert [f.id for f in planes.resolve_features(["PSNR", 0, "ms-ssim"])] == [0, 3]
    for bad in (1, 4, 99, "vmaf", "lpips", []):
        with pytest.raises(ValueError):
            planes.resolve_features(bad)
    with pytest.raises(TypeError):
        planes.resolve_features([True])
    s = planes.PlaneScorer([0, 2, 7], family="yuv")
    assert s.prop_names == ["psnr_y", "psnr_cb", "psnr_cr", "float_ssim",
                            "mse_y", "mse_cb", "mse_cr"]

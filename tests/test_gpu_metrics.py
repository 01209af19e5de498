"""SSIM + MSE + PSNR from one kernel (``fa.metrics``) against the separate
metric functions, and ``StreamingMetrics`` (the reference's streaming scorer,
modules.py:308-451) with and without CUDA-graph capture."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import fa_oracle as O
from conftest import baseline_pair

import frame_analytics_b200 as fa
from frame_analytics_b200 import backend

pytestmark = pytest.mark.gpu


def _u8(shape, sigma=8.0, seed=0):
    a, b = baseline_pair(shape, sigma, seed=seed)
    return torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()


@pytest.mark.parametrize("shape", [(2, 3, 64, 96), (1, 1, 37, 53), (3, 2, 131, 66),
                                   (2, 3, 1080, 1920), (1, 3, 11, 11)])
@pytest.mark.parametrize("reduction", ["mean", "none"])
def test_fused_uint8_matches_separate(shape, reduction):
    x, y = _u8(shape)
    got = fa.metrics(x, y, ("mse", "psnr", "ssim"), reduction=reduction)
    # exact integer sums: MSE and PSNR equal the standalone kernels bit for bit
    assert torch.equal(got["mse"], fa.mse(x, y, reduction=reduction))
    assert torch.equal(got["psnr"], fa.psnr(x, y, reduction=reduction))
    # the SSIM kernel is the same code with the same partition
    assert torch.equal(got["ssim"], fa.ssim(x, y, reduction=reduction))
    # reference in host doubles (a CUDA tensor divided by a scalar is a
    # multiplication by its reciprocal, which can differ in the last bit)
    ssd = ((x.long() - y.long()) ** 2).flatten(1).sum(1).tolist()
    per = x[0].numel()
    ref = [v / per for v in ssd] if reduction == "none" else [sum(ssd) / (per * x.shape[0])]
    assert got["mse"].reshape(-1).tolist() == ref


def test_fused_exact_ssd_backend():
    x, y = _u8((3, 3, 200, 333))
    r = backend.ssim_mse(x, y, backend.host_taps(11, 1.5), shift=127.5, C1=(0.01 * 255) ** 2,
                         C2=(0.03 * 255) ** 2, psnr_bias=20 * math.log10(255), per_image=True)
    ref = ((x.long() - y.long()) ** 2).flatten(1).sum(1)
    assert torch.equal(r["ssd"], ref)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("shape", [(2, 3, 70, 96), (1, 2, 45, 61)])
def test_fused_float_matches_separate(dt, shape):
    g = torch.Generator().manual_seed(1)
    a = torch.rand(shape, generator=g, dtype=torch.float64)
    b = (a + 0.05 * torch.randn(shape, generator=g, dtype=torch.float64)).clamp(0, 1)
    x, y = a.to(dt).cuda(), b.to(dt).cuda()
    got = fa.metrics(x, y, ("mse", "psnr", "ssim"), data_range=1.0, reduction="none")
    torch.testing.assert_close(got["mse"], fa.mse(x, y, reduction="none"), rtol=1e-12, atol=0)
    torch.testing.assert_close(got["psnr"], fa.psnr(x, y, data_range=1.0, reduction="none"),
                               rtol=1e-12, atol=1e-12)
    assert torch.equal(got["ssim"], fa.ssim(x, y, data_range=1.0, reduction="none"))


def test_fused_strided_views():
    x, y = _u8((2, 3, 90, 120))
    xc, yc = x[:, :, 4:-4, 4:-4], y[:, :, 4:-4, 4:-4]
    got = fa.metrics(xc, yc, ("mse", "ssim"), reduction="none")
    assert torch.equal(got["mse"], fa.mse(xc, yc, reduction="none"))
    assert torch.equal(got["ssim"], fa.ssim(xc, yc, reduction="none"))


def test_identical_inputs():
    x, _ = _u8((1, 3, 64, 64))
    got = fa.metrics(x, x.clone(), ("mse", "psnr", "ssim"))
    assert float(got["mse"]) == 0.0
    assert math.isinf(float(got["psnr"]))
    assert abs(float(got["ssim"]) - 1.0) < 1e-6


def test_other_metrics_and_errors():
    x, y = _u8((2, 3, 200, 200))
    got = fa.metrics(x, y, ("gmsd", "l1", "ssim", "ms_ssim"))
    assert torch.equal(got["gmsd"], fa.gmsd(x, y))
    assert torch.equal(got["l1"], fa.l1(x, y))
    assert torch.equal(got["ms_ssim"], fa.ms_ssim(x, y))
    with pytest.raises(ValueError):
        fa.metrics(x, y, ("vmaf",))


@pytest.mark.parametrize("use_graph", [True, False])
def test_streaming_metrics(use_graph):
    shape = (1, 3, 120, 160)
    sm = fa.StreamingMetrics(shape, metrics=("mse", "psnr", "ssim", "gmsd"),
                             use_cuda_graph=use_graph)
    assert sm.graph_captured == use_graph, sm.capture_error
    for seed in range(3):
        a, b = baseline_pair(shape, 6.0, seed=seed)
        got = sm.update(a, b)  # host numpy frames through pinned staging
        x, y = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        assert got["mse"] == float(fa.mse(x, y))
        assert got["psnr"] == float(fa.psnr(x, y))
        assert got["ssim"] == float(fa.ssim(x, y))
        assert got["gmsd"] == float(fa.gmsd(x, y))
        got_dev = sm.update(x, y, as_float=False)  # device frames
        assert torch.equal(got_dev["ssim"], fa.ssim(x, y))


def test_streaming_metrics_rejects():
    with pytest.raises(NotImplementedError):
        fa.StreamingMetrics((1, 3, 64, 64), metrics=("lpips",), use_cuda_graph=False)
    with pytest.raises(ValueError):
        fa.StreamingMetrics((1, 3, 64, 64), metrics=("nope",), use_cuda_graph=False)


def test_streaming_ms_ssim_captures_with_side_streams():
    """MS-SSIM's coarse scales run on forked side streams; they join back into
    the capturing stream, so the CUDA graph still captures and replays."""
    shape = (1, 3, 256, 320)
    sm = fa.StreamingMetrics(shape, metrics=("ms_ssim", "psnr"))
    assert sm.graph_captured
    for seed in range(2):
        a, b = baseline_pair(shape, 6.0, seed=seed)
        got = sm.update(a, b)
        x, y = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        assert abs(got["ms_ssim"] - float(fa.ms_ssim(x, y))) < 1e-12


def test_streaming_instances_replay_concurrently_on_two_streams():
    """Each StreamingMetrics owns its scratch and streams: two instances whose
    graph replays overlap on the GPU both return the single-call values."""
    shape = (2, 3, 192, 200)
    sms = [fa.StreamingMetrics(shape, metrics=("mse", "psnr", "ssim", "ms_ssim")) for _ in range(2)]
    assert all(s.graph_captured for s in sms), [s.capture_error for s in sms]
    pairs = [baseline_pair(shape, 6.0, seed=10 + i) for i in range(6)]
    dev = [(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()) for a, b in pairs]
    torch.cuda.synchronize()
    outs = []
    for i in range(0, 6, 2):  # both instances queued before either result is read
        outs.append(sms[0].update(*dev[i], as_float=False))
        outs.append(sms[1].update(*dev[i + 1], as_float=False))
    torch.cuda.synchronize()
    for (x, y), got in zip(dev, outs):
        assert float(got["mse"]) == float(fa.mse(x, y))
        assert float(got["ssim"]) == float(fa.ssim(x, y))
        assert abs(float(got["ms_ssim"]) - float(fa.ms_ssim(x, y))) < 1e-12


def test_streaming_overlapped_updates_keep_results_apart():
    """Back-to-back device-result updates alternate slots; every returned
    tensor holds its own pair's values."""
    shape = (1, 3, 96, 128)
    sm = fa.StreamingMetrics(shape)
    pairs = [baseline_pair(shape, 4.0 + i, seed=20 + i) for i in range(5)]
    res = [sm.update(a, b, as_float=False) for a, b in pairs]
    for (a, b), got in zip(pairs, res):
        x, y = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        assert float(got["psnr"]) == float(fa.psnr(x, y))


@pytest.mark.parametrize("shape", [(2, 3, 64, 96), (1, 1, 37, 53), (3, 2, 131, 717),
                                   (1, 1, 400, 1067), (1, 3, 2160, 3840)])
@pytest.mark.parametrize("dt", [torch.uint8, torch.float32])
def test_fused_ssim_gmsd_matches_separate_calls(shape, dt):
    """SSIM + GMSD (+ MSE / PSNR) from one launch equal the separate calls
    (GMSD within 5e-6, SSIM within 1e-7, MSE exact for uint8) and the oracle."""
    from frame_analytics_b200 import backend
    a, b = baseline_pair(shape, 9.0, seed=sum(shape))
    x, y = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    L = 255.0
    if dt == torch.float32:
        x, y, L = x.float() / 255.0, y.float() / 255.0, 1.0
    # rows a TMA map describes (16-byte strides) fuse
    assert backend.ssim_gmsd_fusable(x, y, 11) == (shape[-1] * x.element_size() % 16 == 0)
    for names in (("ssim", "gmsd", "gms"), ("mse", "psnr", "ssim", "gmsd")):
        for red in ("none", "mean"):
            got = fa.metrics(x, y, names, reduction=red, data_range=L, fuse_gmsd=True)
            for n in names:
                kw = {} if n == "mse" else {"data_range": L}
                want = getattr(fa, n)(x, y, reduction=red, **kw)
                tol = 0 if (n == "mse" and dt == torch.uint8) else (1e-7 if n == "ssim" else 5e-6)
                assert float((got[n] - want).abs().max()) <= tol, (n, red)
    if shape[-1] <= 1067:
        m, s = O.gmsd(a, b, eps=(1e-6 * 255.0) ** 2)
        got = fa.metrics(x, y, ("ssim", "gmsd", "gms"), reduction="none", data_range=L,
                         fuse_gmsd=True)
        np.testing.assert_allclose(got["gmsd"].cpu().numpy(), s, atol=5e-6)
        np.testing.assert_allclose(got["gms"].cpu().numpy(), m, atol=5e-6)


def test_fused_ssim_gmsd_falls_back_where_it_cannot_fuse():
    """A width whose GMS map overhangs the SSIM strips (W = 362), and a uint16
    pair, are served by separate launches with the same results."""
    from frame_analytics_b200 import backend
    a, b = baseline_pair((1, 2, 70, 362), 9.0, seed=1)
    x, y = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    assert not backend.ssim_gmsd_fusable(x, y, 11)
    got = fa.metrics(x, y, ("ssim", "gmsd"), reduction="none", fuse_gmsd=True)
    assert torch.equal(got["gmsd"], fa.gmsd(x, y, reduction="none"))
    assert torch.equal(got["ssim"], fa.ssim(x, y, reduction="none"))

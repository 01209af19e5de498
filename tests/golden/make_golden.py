"""Generate tests/golden/golden.npz from the reference itself.

Run once, in a container that has the reference checked out (read-only):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [/path/to/reference]

Inputs come from the reference's own test generators (tests/validate.py
make_pair, tests/test_training_metrics.py _pair) or from the seeded BASELINE
generators; expected values from the reference's float64 oracle
(frame_analytics/reference.py) and from its CPU library (fa_cpu.cpp, built by
oracle/Makefile into oracle/_ref/).  The GPU box never runs this script; it
only reads the .npz it wrote.
"""

from __future__ import annotations

import ctypes
import importlib.util
import sys
import json
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _reference_path() -> Path:
    """argv[1], else $FA_REFERENCE, else BASELINE.json's reference_path."""
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if args:
        return Path(args[0])
    if os.environ.get("FA_REFERENCE"):
        return Path(os.environ["FA_REFERENCE"])
    return Path(json.loads((REPO / "BASELINE.json").read_text())["reference_path"])


REF = _reference_path()


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


ref = _load("fa_reference_py", REF / "frame_analytics" / "reference.py")
sys.path.insert(0, str(REF / "tests"))
sys.dont_write_bytecode = True
validate = None
try:
    # validate.py imports the reference package; make it importable read-only
    sys.path.insert(0, str(REF))
    import validate  # noqa: E402
except Exception as exc:  # pragma: no cover
    raise SystemExit(f"cannot import the reference's validate.py: {exc}")


def cpu_lib():
    so = REPO / "oracle" / "_ref" / "libfa_cpu_ref.so"
    if not so.exists():
        raise SystemExit("build oracle/_ref first: make -C oracle")
    lib = ctypes.CDLL(str(so))
    lib.fa_cpu_set_num_threads(1)
    return lib


def win1d(k=11, s=1.5):
    c = np.arange(k, dtype=np.float64) - (k - 1) / 2
    g = np.exp(-(c * c) / (2 * s * s))
    return (g / g.sum()).astype(np.float32)


def cpu_ssim_planes(lib, x, y, k=11, data_range=255.0):
    """Reference CPU library: per-plane SSIM means of uint8 NCHW."""
    x = np.ascontiguousarray(x, dtype=np.uint8)
    y = np.ascontiguousarray(y, dtype=np.uint8)
    n, c, h, w = x.shape
    win = win1d(k)
    out = np.zeros(n * c, dtype=np.float64)
    L = data_range
    rc = lib.fa_cpu_ssim(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p),
                         0, n, c, h, w, win.ctypes.data_as(ctypes.c_void_p), k,
                         ctypes.c_double(L / 2), ctypes.c_double((0.01 * L) ** 2),
                         ctypes.c_double((0.03 * L) ** 2), None,
                         out.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0, rc
    return out / ((h - k + 1) * (w - k + 1))


def cpu_gmsd(lib, x, y, down=1, data_range=255.0):
    x = np.ascontiguousarray(x, dtype=np.uint8)
    y = np.ascontiguousarray(y, dtype=np.uint8)
    n, c, h, w = x.shape
    m = np.zeros(n)
    s = np.zeros(n)
    L = data_range
    rc = lib.fa_cpu_gmsd(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p),
                         0, n, c, h, w, ctypes.c_double(170.0 * (L / 255) ** 2),
                         ctypes.c_double((1e-6 * L) ** 2), down,
                         m.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0, rc
    return m, s


def baseline_pair(shape, sigma, seed=0):
    """BASELINE.json configs 0/1/3/4: a ~ U{0..255}, b = clip(a + round(N(0, s^2)))."""
    rng = np.random.default_rng(seed)
    a = rng.integers(0, 256, shape, dtype=np.uint8)
    b = np.clip(a.astype(np.int16) + np.round(rng.normal(0, sigma, shape)).astype(np.int16),
                0, 255).astype(np.uint8)
    return a, b


def main():
    lib = cpu_lib()
    out = {}
    eps_g = (1e-6 * 255.0) ** 2

    # 1. single-plane accuracy cases of the reference's accuracy gate
    cases = [(64, 64, "uniform", 20.0), (127, 233, "natural", 8.0),
             (256, 256, "natural", 3.0), (33, 41, "flat", 5.0)]
    for i, (h, w, kind, noise) in enumerate(cases):
        a, b = validate.make_pair(h, w, kind, noise, seed=h * w)
        key = f"v{i}"
        out[f"{key}_a"] = a.astype(np.uint8)
        out[f"{key}_b"] = b.astype(np.uint8)
        s, smap = ref.ssim_reference(a, b, 255.0, return_map=True)
        out[f"{key}_ssim"] = s
        if h * w <= 64 * 64:
            out[f"{key}_map"] = smap
        out[f"{key}_mse"] = ref.mse_reference(a, b)
        out[f"{key}_psnr"] = ref.psnr_reference(a, b, 255.0)
        out[f"{key}_l1"] = ref.l1_reference(a, b)
        out[f"{key}_charb"] = ref.charbonnier_reference(a, b, 1e-3)
        out[f"{key}_charb2"] = ref.charbonnier_reference(a, b, 2.0)
        out[f"{key}_huber"] = ref.huber_reference(a, b, 1.0)
        out[f"{key}_huber3"] = ref.huber_reference(a, b, 3.0)
        out[f"{key}_gmsd"] = ref.gmsd_reference(a, b, 255.0, eps=eps_g)
        out[f"{key}_gmsd_nodown"] = ref.gmsd_reference(a, b, 255.0, downsample=False, eps=eps_g)
        for ksz in (3, 5, 7, 9):
            out[f"{key}_ssim_k{ksz}"] = ref.ssim_reference(a, b, 255.0, win_size=ksz)
        out[f"{key}_cpu_ssim"] = cpu_ssim_planes(lib, a[None, None], b[None, None])[0]

    # 2. MS-SSIM / GMSD / pixel-loss cases of the accuracy gate
    for i, (h, w, kind, noise) in enumerate([(200, 232, "natural", 8.0),
                                             (257, 193, "natural", 20.0),
                                             (176, 176, "uniform", 12.0)]):
        a, b = validate.make_pair(h, w, kind, noise, seed=h + w)
        key = f"m{i}"
        out[f"{key}_a"] = a.astype(np.uint8)
        out[f"{key}_b"] = b.astype(np.uint8)
        out[f"{key}_ms_ssim"] = ref.ms_ssim_reference(a, b, 255.0)
        out[f"{key}_gmsd"] = ref.gmsd_reference(a, b, 255.0, eps=eps_g)
        out[f"{key}_l1"] = ref.l1_reference(a, b)
        out[f"{key}_charb"] = ref.charbonnier_reference(a, b)
        out[f"{key}_huber"] = ref.huber_reference(a, b)

    # 3. luma x crop (validate.py's SR-convention section generator)
    rng = np.random.default_rng(99)
    rgb = rng.integers(0, 256, (3, 180, 220)).astype(np.float64)
    rgb2 = np.clip(rgb + 9 * rng.standard_normal((3, 180, 220)), 0, 255).round()
    out["luma_a"] = rgb.astype(np.uint8)
    out["luma_b"] = rgb2.astype(np.uint8)
    for mode in ("bt601", "bt709", "matlab"):
        ya = ref.rgb_to_luma_reference(rgb, mode)
        yb = ref.rgb_to_luma_reference(rgb2, mode)
        for cb in (0, 4):
            la = ya[cb:ya.shape[0] - cb or None, cb:ya.shape[1] - cb or None]
            lb = yb[cb:yb.shape[0] - cb or None, cb:yb.shape[1] - cb or None]
            out[f"luma_{mode}_{cb}_ssim"] = ref.ssim_reference(la, lb, 255.0)
            out[f"luma_{mode}_{cb}_psnr"] = ref.psnr_reference(la, lb, 255.0)

    # 4. multi-channel GMSD pooling, pinned by the reference CPU library
    a, b = baseline_pair((2, 3, 64, 80), 8.0, seed=5)
    out["gm3_a"], out["gm3_b"] = a, b
    for down in (1, 0):
        m, s = cpu_gmsd(lib, a, b, down)
        out[f"gm3_cpu_mean_d{down}"] = m
        out[f"gm3_cpu_std_d{down}"] = s

    # 5. config 0 (uint8 1x3x512x512, sigma 8, seed 0): reference.py per plane
    a, b = baseline_pair((1, 3, 512, 512), 8.0, seed=0)
    planes = [ref.ssim_reference(a[0, c].astype(np.float64), b[0, c].astype(np.float64), 255.0)
              for c in range(3)]
    out["cfg0_ssim"] = float(np.mean(planes))
    out["cfg0_cpu_ssim"] = float(cpu_ssim_planes(lib, a, b).mean())
    out["cfg0_a_sum"] = int(a.astype(np.int64).sum())

    # 6. config 1 exact SSD (uint8 8x3x1080x1920, sigma 5, seed 0)
    a, b = baseline_pair((8, 3, 1080, 1920), 5.0, seed=0)
    d = a.astype(np.int64) - b.astype(np.int64)
    out["cfg1_ssd"] = (d * d).reshape(8, -1).sum(axis=1)
    out["cfg1_a_sum"] = int(a.astype(np.int64).sum())

    # 7. MATLAB-mode SSIM downsample, from the reference's own implementation
    #    (frame_analytics/functional.py _matlab_downsample, torch on the CPU)
    import torch
    from frame_analytics import functional as ref_f
    rng = np.random.default_rng(7)
    dsx = rng.integers(0, 256, (1, 2, 41, 58)).astype(np.float32)
    out["mdown_x"] = dsx
    for f in (2, 3, 4):
        out[f"mdown_f{f}"] = ref_f._matlab_downsample(torch.from_numpy(dsx), f).numpy()

    np.savez_compressed(HERE / "golden.npz", **out)
    print(f"wrote {HERE / 'golden.npz'}: {len(out)} arrays")


def _smooth_rgb(h, w, noise, seed):
    """A smooth colour image and a noisy copy (uint8 values), the kind of pair
    SSIMULACRA 2 is tuned on."""
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float64)
    base = 120 + 55 * np.sin(xx / 8.0) * np.cos(yy / 6.0)
    a = np.stack([np.clip(base + 25 * np.sin(xx / 21.0), 0, 255),
                  np.clip(0.75 * base + 45, 0, 255),
                  np.clip(1.1 * base - 12 + 18 * np.cos(yy / 15.0), 0, 255)]).round()
    b = np.clip(a + noise * rng.standard_normal(a.shape), 0, 255).round()
    return a.astype(np.uint8), b.astype(np.uint8)


def ssimulacra2_fixtures():
    """tests/golden/ssimulacra2.npz: pairs scored by the reference's float64
    transcription of libjxl (reference.ssimulacra2_reference, which runs the
    recursive Gaussian itself) and by its torch path (frame_analytics.
    ssimulacra2 on the CPU, float32 and float64)."""
    import torch
    import frame_analytics as ref_s2
    cases = {
        "s0": _smooth_rgb(64, 72, 6.0, 11),
        "s1": _smooth_rgb(100, 60, 20.0, 2),    # five scales
        "s2": _smooth_rgb(37, 45, 3.0, 5),      # odd sizes, three scales
        "s3": _smooth_rgb(8, 9, 10.0, 7),       # the 8x8 floor
    }
    rng = np.random.default_rng(4)
    a = rng.integers(0, 256, (3, 96, 128)).astype(np.uint8)
    cases["r0"] = (a, np.clip(a + np.round(rng.normal(0, 8, a.shape)), 0, 255).astype(np.uint8))
    g, gb = _smooth_rgb(48, 56, 8.0, 9)
    cases["g0"] = (g[:1], gb[:1])               # grayscale, replicated to RGB
    out = {}
    for k, (x, y) in cases.items():
        out[f"{k}_a"], out[f"{k}_b"] = x, y
        x3 = np.repeat(x, 3, axis=0) if x.shape[0] == 1 else x
        y3 = np.repeat(y, 3, axis=0) if y.shape[0] == 1 else y
        out[f"{k}_ref64"] = ref.ssimulacra2_reference(x3.astype(np.float64),
                                                     y3.astype(np.float64), 255.0)
        tx, ty = torch.from_numpy(x), torch.from_numpy(y)
        out[f"{k}_torch32"] = float(ref_s2.ssimulacra2(tx, ty, data_range=255.0))
        out[f"{k}_torch64"] = float(ref_s2.ssimulacra2(tx, ty, data_range=255.0,
                                                       dtype=torch.float64))
    np.savez_compressed(HERE / "ssimulacra2.npz", **out)
    print(f"wrote {HERE / 'ssimulacra2.npz'}: {len(out)} arrays")


if __name__ == "__main__":
    if "--ssimulacra2" in sys.argv:
        sys.argv.remove("--ssimulacra2")
        ssimulacra2_fixtures()
    else:
        main()

"""Shared fixtures.  `gpu` marks tests that need a CUDA device (B200)."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle"))

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


def baseline_pair(shape, sigma, seed=0):
    """BASELINE.json generator: a ~ U{0..255}, b = clip(a + round(N(0, sigma^2)))."""
    rng = np.random.default_rng(seed)
    a = rng.integers(0, 256, shape, dtype=np.uint8)
    b = np.clip(a.astype(np.int16) + np.round(rng.normal(0, sigma, shape)).astype(np.int16),
                0, 255).astype(np.uint8)
    return a, b


def natural_pair(h=97, w=131, seed=3, noise=7.0):
    """Smooth texture plus noise, the shape of image the metrics are tuned on."""
    rng = np.random.default_rng(seed)
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float64)
    a = np.clip(120 + 50 * np.sin(xx / 11.0) * np.cos(yy / 13.0)
                + 12 * rng.standard_normal((h, w)), 0, 255).round()
    b = np.clip(a + noise * rng.standard_normal((h, w)), 0, 255).round()
    return a, b

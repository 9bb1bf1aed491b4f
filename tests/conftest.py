import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; runs the sm_100a kernels")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def rel_err(a, b):
    """RMS relative error ||a - b|| / ||b|| (the ratio of utils/ela_utils.py:63-85)."""
    import torch

    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_err(a, b):
    """Largest absolute difference relative to the largest reference magnitude."""
    import torch

    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30)) if b.numel() else 0.0


def assert_close(a, b, tol, name="", max_tol=None):
    """RMS relative error below ``tol`` (1e-5 fp32, 2e-2 bf16) and the
    largest element error below ``max_tol`` (default 5 * tol) of the largest reference
    magnitude, so that a few badly wrong elements cannot hide inside a good RMS."""
    assert tuple(a.shape) == tuple(b.shape), (name, tuple(a.shape), tuple(b.shape))
    r = rel_err(a, b)
    m = max_err(a, b)
    assert r < tol, f"{name}: RMS relative error {r:.3e} >= {tol:.1e}"
    mt = 5 * tol if max_tol is None else max_tol
    assert m < mt, f"{name}: max error {m:.3e} of the largest magnitude >= {mt:.1e}"

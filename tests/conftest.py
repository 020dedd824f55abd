"""Shared pytest configuration.

``-m gpu`` tests need a B200 (sm_100) and the built library; ``-m "not gpu"``
tests run anywhere.  The oracle (``oracle/``) is imported here only as the
checker.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# The reference package, installed (unmodified) under baseline/_ref.  Tests
# that drive the reference's own modules through the cuda backend import it
# from there and skip when it is not installed.
REF_SITE = os.path.join(ROOT, "baseline", "_ref")
if os.path.isdir(os.path.join(REF_SITE, "omniweave")) and REF_SITE not in sys.path:
    sys.path.append(REF_SITE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from omniwave_b200 import _lib

    lib = _lib.load()  # raises if the library is missing: no silent fallback
    if not lib.ow_device_supported(0):
        pytest.skip("device 0 is not sm_100")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def omniweave():
    """The reference package with the cuda backend installed (integration.install())."""
    try:
        import omniweave as ow  # noqa: F401
    except ImportError:
        pytest.skip("reference package omniweave is not installed under baseline/_ref")
    from omniwave_b200 import integration

    return integration.install()


@pytest.fixture(autouse=True)
def _device_fault_word_stays_clear(request):
    """Every GPU test leaves the library's device fault word at 0 (no kernel
    gave up on a bounded wait)."""
    yield
    if "cuda_device" not in request.fixturenames or not torch.cuda.is_available():
        return
    from omniwave_b200 import _lib

    v = _lib.device_fault(0, reset=True)
    assert v == 0, f"device fault word was {v} after {request.node.name}"


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def rel_err(actual, expected) -> float:
    """max |a - e| / max |e| (the reference's bf16 gate normalisation)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    scale = max(float(np.abs(e).max()), 1e-30)
    return float(np.abs(a - e).max()) / scale

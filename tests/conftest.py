"""Test configuration: the `gpu` marker, import paths, and shared fixtures.

Tests marked gpu need a B200 and call the CUDA library through its C ABI; everything else
runs on the CPU (the oracle against golden vectors, host-side validation of the C ABI, the
.cvw format, and multi-rank host logic over gloo).
"""

from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cu-vit_b200"))
sys.path.insert(0, str(ROOT / "tests" / "golden"))
GOLDEN = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run with -m gpu on a B200)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as data:
        return {key: data[key] for key in data.files}


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    if not oracle.ORACLE_LIB.exists():
        oracle.build()
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device; the library must be built (no fallback exists)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import cuvit

    cuvit.library()
    return torch


@pytest.fixture(autouse=True)
def _device_clean(request):
    """After every GPU test: no kernel may have given up on a bounded wait."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from cuvit import kernels

    assert kernels.device_status() == 0

"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any host (oracle, host-side validation, ABI surface);
``-m gpu`` needs a B200 and exercises the CUDA library through its C-ABI.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "comfyui-h3-speedkit_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")


def pytest_sessionstart(session):
    """Build the kernel library and the oracles if they are missing or stale
    (no-op when up to date; nvcc and gcc are present on both hosts)."""
    sys.path.insert(0, str(PKG_DIR / "csrc"))
    import build as kernel_build
    kernel_build.build(force=False)
    from oracle import build as oracle_build
    oracle_build.build()


@pytest.fixture(scope="session")
def device():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("GPU tests need a CUDA device; run them on the B200 box")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        raise RuntimeError(f"GPU tests target B200 (sm_100), found sm_{major}{minor}")
    return torch.device("cuda", 0)

"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle pinning, host logic and C-ABI export checks on a CPU
box; ``-m gpu`` runs the parity tests proper through the C-ABI on a B200.
"""
import sys

import pytest
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="module")
def k3():
    """The built package on a CUDA device (GPU tests fail loudly without one)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from kimi_k3_mlx_macmini_b200 import build
    build.build()
    import kimi_k3_mlx_macmini_b200 as k
    return k

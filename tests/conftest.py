"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle pinning, host logic and C-ABI export checks on a CPU
box; ``-m gpu`` runs the parity tests proper through the C-ABI on a B200.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")

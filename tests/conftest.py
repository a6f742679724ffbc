"""Test configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the CPU suite (oracle vs golden fixtures, host logic, the
C ABI library's exports and host-side functions); ``-m gpu`` runs the parity
tests of the CUDA kernels against the oracle on a B200.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")

"""Test configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle checks, host logic and C-ABI load checks on
CPU; ``-m gpu`` runs the CUDA parity tests on a B200.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cyfa-jittor_b200")
for path in (ROOT, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")

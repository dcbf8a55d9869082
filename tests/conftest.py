"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on any host (oracle pins, host logic, C-ABI symbol checks,
gloo ranks); ``-m gpu`` runs the CUDA parity suite on a B200.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PARENT = os.path.join(ROOT, "cute-causal-conv1d_b200")
for p in (ROOT, PKG_PARENT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")

"""Shared pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle, host-logic and C-ABI load checks on any machine;
`-m gpu` runs the parity tests, which call the CUDA library through its C ABI on
a B200 and compare against the CPU oracle.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "thunderkittens-sm7x_b200")
for path in (ROOT, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a) and the built library")

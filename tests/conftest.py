"""Test configuration.

Markers: ``gpu`` -- needs a CUDA device (run on a B200 with ``-m gpu``);
everything else runs on the CPU (``-m "not gpu"``).  GPU tests are not
skipped when CUDA is missing: they fail, so a broken GPU environment shows.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "bt-3dgs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")

"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 and the built CUDA library; everything else
runs on CPU (oracle against the golden fixtures, host-side validation of the
C ABI, multi-process gloo tests of the sharding logic).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "oracle", "falcon-ocr-cpu_b200", os.path.join("tests", "golden")):
    path = os.path.join(ROOT, sub)
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built libfo_cuda.so")

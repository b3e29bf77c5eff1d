"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any CPU box (oracle vs golden vectors, host logic,
C-ABI exports); `-m gpu` needs a B200 and checks the CUDA path against the
oracle through the C ABI.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "remora-lab_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")

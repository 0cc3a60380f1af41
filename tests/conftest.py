"""Test configuration: the `gpu` marker and the repository root on sys.path.

`-m "not gpu"` runs on any host (oracle against the reference's known-answer
tests, host logic, the C-ABI library's exports); `-m gpu` needs a B200 and
runs the CUDA kernels through the C ABI against the oracle.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")

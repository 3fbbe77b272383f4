"""Test configuration: the ``gpu`` marker and the repository on sys.path.

Tests marked ``gpu`` need a B200 (sm_100a) and run with ``pytest -m gpu``;
everything else runs on a CPU-only machine (``pytest -m "not gpu"``).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device with sm_100a (B200)")
    config.addinivalue_line("markers", "slow: long-running test")

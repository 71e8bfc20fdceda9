"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device and the built ``libadakv_b200.so``; every
other test runs on CPU.  The repository root is put on ``sys.path`` so the
tests import the in-tree package and the oracle.
"""
import os
import sys

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")

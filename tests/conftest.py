"""Pytest configuration.

* ``gpu``: needs a B200 (sm_100a) and the built ``libsas.so``; the CPU suite
  runs with ``-m "not gpu"``.
* ``slow``: large CPU-oracle cases, skipped unless ``--runslow`` (the
  reference suite's convention, conftest.py:1-32 of the reference).
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_addoption(parser):
    parser.addoption("--runslow", action="store_true", default=False,
                     help="run slow cases (large CPU-oracle shapes)")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: large case; skipped unless --runslow is given")


def pytest_collection_modifyitems(config, items):
    if config.getoption("--runslow"):
        return
    skip_slow = pytest.mark.skip(reason="slow case; pass --runslow to run")
    for item in items:
        if "slow" in item.keywords:
            item.add_marker(skip_slow)

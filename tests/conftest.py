import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: longer CPU-only test")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (not skip) when selected without a GPU, so that a
    # run of `-m gpu` on a machine without one cannot pass silently.
    pass

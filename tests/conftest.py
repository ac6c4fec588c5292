import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run on the GPU box: pytest -m gpu)")
    config.addinivalue_line("markers", "slow: long CPU test")


def pytest_collection_modifyitems(config, items):
    # tests/test_zz_* files run last (a failure there leaves every other test already run), and the
    # no-allocation entry point's test after all of them.
    def rank(it):
        name = os.path.basename(str(it.fspath))
        return (name.startswith("test_zz_"), name == "test_zz_no_alloc.py")

    items.sort(key=rank)

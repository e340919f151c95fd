"""Test configuration: the `gpu` marker and the import path of the repository root."""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


# Each GPU test ends within 10 minutes (the whole GPU suite takes about 3). A test that runs past
# that limit is stopped by pytest-timeout's thread method: it prints the stack of every Python
# thread, naming the library call that did not return, and ends the run.
GPU_TEST_TIMEOUT_S = 600


def pytest_collection_modifyitems(config, items):
    if not config.pluginmanager.hasplugin("timeout"):
        return
    import pytest

    for item in items:
        if item.get_closest_marker("gpu") and not item.get_closest_marker("timeout"):
            item.add_marker(pytest.mark.timeout(GPU_TEST_TIMEOUT_S, method="thread"))

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.fixture(scope="session")
def api():
    from porch_b200.build import build as build_library

    build_library()
    from porch_b200 import api as porch_api

    return porch_api


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import build as obuild

    obuild.build_oracle()
    obuild.build_pb_runner()
    from oracle import graph

    graph.lib()
    return graph


@pytest.fixture(scope="session")
def gpu(api):
    """The CUDA path must run: no silent skip on a GPU box."""
    if not api.is_available():
        pytest.fail("CUDA JIT backend unavailable on a GPU test run (libcuda/NVRTC/device missing)")
    return api

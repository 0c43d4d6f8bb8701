import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def kat():
    """Known-answer vectors of the reference's own tests (tests/golden/make_golden.py)."""
    with open(os.path.join(ROOT, "tests", "golden", "reference_kat.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def dev():
    """The library initialised on cuda:0 (cuda_init / cuda_fini)."""
    import wukong_b200 as wk
    L = wk.lib()
    L.cuda_init(0)
    yield L
    L.cuda_fini()

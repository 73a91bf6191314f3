import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size CPU oracle run")


@pytest.fixture(scope="session")
def kats():
    import json
    with open(os.path.join(REPO, "tests", "golden", "ref_kats.json")) as f:
        return json.load(f)

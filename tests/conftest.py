import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_oracle():
    """The CPU checker (oracle/) is compiled once per session."""
    from oracle import oracle as O
    ref = os.environ.get("QUASAR_REFERENCE", "")
    if not O.available("oracle") or (ref and os.path.exists(os.path.join(ref, "sample.c")) and not O.available("ref")):
        O.build()
    yield

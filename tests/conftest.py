import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running (full-size model) test")


def _ensure_oracle():
    so = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(so):
        subprocess.check_call(["sh", os.path.join(ROOT, "oracle", "build.sh")])


@pytest.fixture(scope="session")
def orc():
    _ensure_oracle()
    from oracle import oracle as _o
    o = _o.get()
    o.set_mode(False)
    return o

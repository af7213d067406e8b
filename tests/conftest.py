"""Test configuration.

Markers: tests that need a B200 are marked ``gpu`` and call the library only
through its C ABI; everything else runs on CPU (the oracle against the
reference's known answers, host-side policy, the ABI's symbol table, gloo
multi-process host logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "hy-nomas-rs_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def nkv():
    import nomas_kv
    nomas_kv.lib()
    return nomas_kv

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle as O

    if not os.path.exists(O.ORACLE_SO):
        O.build()
    return O


@pytest.fixture(scope="session")
def ref_mod(oracle_mod):
    if not oracle_mod.ref_available("strict"):
        pytest.skip("reference harness library oracle/_ref/libqwref_strict.so not built")
    return oracle_mod

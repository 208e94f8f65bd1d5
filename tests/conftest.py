"""Shared pytest setup: the `gpu` marker and import paths for the oracle
(test infrastructure) and the product's ctypes binding."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "irodori-c_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)
if os.path.join(ROOT, "tests") not in sys.path:
    sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA C-ABI)")


@pytest.fixture(scope="session")
def ref_ieee():
    import oracle
    if not oracle.ref_available("ieee"):
        pytest.skip("reference build oracle/_ref is not present")
    return oracle

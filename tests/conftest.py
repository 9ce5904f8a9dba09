"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs the oracle pins, the golden vectors and the ABI checks on any
machine; `-m gpu` runs the CUDA path against the oracle on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built liblitemind_b200.so")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle as orc

    if not os.path.exists(orc.ORACLE_SO):
        orc.build()
    return orc.Oracle()


@pytest.fixture(scope="session")
def reference_lib():
    from oracle import oracle as orc

    if not orc.reference_available():
        if os.path.isdir(orc.REFERENCE_DIR):
            orc.build()
        else:
            pytest.skip("reference build (oracle/_ref) is not available on this machine")
    return orc.Reference()


@pytest.fixture(scope="session")
def v2lite_weights():
    """DeepSeek-V2-Lite-shaped layer weights, seed 0 (about 1.1 GB of host memory)."""
    from litemind_b200 import synthetic as syn

    return syn.layer_weights(syn.V2_LITE, seed=0)

"""Shared test setup. `-m gpu` tests need a CUDA device; everything else runs on CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _have_reference_lib():
    from oracle import oracle

    return os.path.exists(oracle.REF_SO) or oracle.build_ref()


@pytest.fixture(scope="session")
def ref():
    """The reference engine library (oracle/_ref), built from the reference sources here."""
    from oracle import oracle

    if not _have_reference_lib():
        pytest.skip("oracle/_ref/libmpref.so not built and reference sources absent")
    return oracle.RefLib()


@pytest.fixture(scope="session")
def built():
    """Builds (if stale) and returns the product libraries' directory."""
    from tinyinfer_b200 import build

    build.build()
    return build.HERE

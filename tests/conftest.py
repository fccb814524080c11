import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ferrite-strata_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

LIB = os.path.join(PKG, "libstrata_b200.so")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def _ensure_built():
    if not os.path.exists(LIB):
        import build  # ferrite-strata_b200/build.py
        build.build()
    from oracle import oracle as ora
    ora.lib()


@pytest.fixture(scope="session")
def plugin():
    _ensure_built()
    from strata_host import Plugin
    p = Plugin(LIB)
    yield p
    p.close()


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests fail loudly (rather than skip) when CUDA is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a visible CUDA device")
    _ensure_built()
    return torch

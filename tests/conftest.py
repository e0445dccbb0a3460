"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run on a B200 box;
everything else runs on the CPU-only build machine."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libchatnet_cuda)")


@pytest.fixture(scope="session")
def oracle():
    from tests import _oracle
    return _oracle.load()


@pytest.fixture(scope="session")
def ctx():
    import chatnet_b200 as cn
    c = cn.Context(0)
    yield c
    c.close()

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_kind():
    """'ref' when the reference build is present (this container, or shipped
    to the GPU host as oracle/_ref), else the restatement 'port'."""
    import oracle as orc
    if orc.available("stack", "ref"):
        return "ref"
    orc.build_oracles()
    return "port"


@pytest.fixture(scope="session")
def gpu_lib():
    from puffysics_b200 import build, engine
    build.build()
    return engine.lib()

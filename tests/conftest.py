import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    # build the in-tree libraries once (no-op when up to date)
    from godwit_b200 import build
    build.build_oracle()
    try:
        build.build_cuda()
    except Exception as e:  # the CPU suite can still run the oracle tests
        print(f"warning: CUDA library build failed: {e}", file=sys.stderr)


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ctx():
    from godwit_b200.runtime import Context
    c = Context(0)
    yield c
    c.close()

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA extension")


def pytest_collection_modifyitems(config, items):
    """GPU tests are skipped on a machine without a CUDA device; on a GPU box
    they run and fail loudly if the extension is missing."""
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def built_library():
    """Build the CUDA extension once if it is missing (nvcc cross-compiles
    without a GPU); an existing build is used as is."""
    from blocksparsefa_reorder_b200 import build

    if not build.LIB_PATH.exists():
        build.build()
    return build.LIB_PATH


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def dev():
    import torch
    return torch.device("cuda:0")

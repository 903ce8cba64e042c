import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200); the CUDA path, compared with the oracle")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(params=["dense", "in_place"])
def kv_path(request):
    """Runs a test with each way of reading the KV cache as the process
    default (pcp_set_kv_path(NULL, ...)); e4m3 caches take it, bf16 caches
    always use the dense path.  Restores the automatic choice afterwards."""
    from aws_training_study_b200 import _capi

    _capi.set_default_kv_path(request.param)
    try:
        yield request.param
    finally:
        _capi.set_default_kv_path("auto")

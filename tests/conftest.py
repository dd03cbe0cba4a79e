import os

import pytest

os.environ.setdefault("SDCGUARD_SIGN_SEED", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)

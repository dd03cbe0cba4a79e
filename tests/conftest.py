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


@pytest.fixture(autouse=True)
def _reduction_flags_restored():
    """The training guards switch off PyTorch's reduced-precision GEMM reductions on checked steps; a test that
    leaves them changed would change every later test's (and a user's) GEMMs."""
    import torch
    m = torch.backends.cuda.matmul
    before = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    yield
    after = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    assert after == before, f"a test left the cuBLAS reduction flags changed: {before} -> {after}"

"""NVTX ranges around this package's phases, for Nsight Systems timelines: `SDCGUARD_NVTX=1` turns them on (off,
they cost one attribute read). Ranges: sdcguard.generate / .prefill / .decode (serving engine), sdcguard.poll
(reading the check state), sdcguard.train_step and sdcguard.flush (training guard), sdcguard.replay (the replay
checks the decoder forks onto its side stream).

    from sdcguard_b200.utils.trace import nvtx_range
    with nvtx_range("sdcguard.prefill"):
        ...

Reference: the reference's profiling hooks (src/sdcguard/serve.py timing) and its cost tables; here the ranges are
what Nsight's CUDA timeline groups kernels by.
"""
from __future__ import annotations

import contextlib
import os

ENABLED = os.environ.get("SDCGUARD_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx_range(name: str):
    if not ENABLED:
        yield
        return
    import torch
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def set_enabled(on: bool) -> None:
    global ENABLED
    ENABLED = bool(on)

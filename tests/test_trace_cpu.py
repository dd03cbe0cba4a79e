"""NVTX ranges: off by default (no call into NVTX), on with set_enabled / SDCGUARD_NVTX=1."""
import torch

from sdcguard_b200.utils import trace


def test_nvtx_ranges(monkeypatch):
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: calls.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    trace.set_enabled(False)
    with trace.nvtx_range("a"):
        pass
    assert calls == []
    trace.set_enabled(True)
    try:
        with trace.nvtx_range("sdcguard.prefill"):
            with trace.nvtx_range("sdcguard.poll"):
                pass
    finally:
        trace.set_enabled(False)
    assert calls == [("push", "sdcguard.prefill"), ("push", "sdcguard.poll"), ("pop",), ("pop",)]

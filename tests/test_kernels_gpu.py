"""cuBLASLt kernel inventory of a real workload and its replay on a B200: `kernels record` of a few bf16 linear
layers (plain and transposed operands, one batched), then `kernels test` replays every call at its shape in a fresh
process and judges it against float64: no call is WRONG, and at least one ran the same kernel as the workload."""
import sys

import pytest

pytestmark = pytest.mark.gpu

WORKLOAD = """
import torch
d = torch.device('cuda')
x = torch.randn(96, 512, device=d, dtype=torch.bfloat16)
w = torch.randn(768, 512, device=d, dtype=torch.bfloat16)
torch.nn.functional.linear(x, w)
torch.matmul(x, torch.randn(512, 256, device=d, dtype=torch.bfloat16))
torch.bmm(torch.randn(4, 64, 128, device=d, dtype=torch.bfloat16), torch.randn(4, 128, 32, device=d,
                                                                               dtype=torch.bfloat16))
torch.cuda.synchronize()
"""


def test_record_and_replay(tmp_path):
    from sdcguard_b200.tools import kernels
    inv = kernels.record([sys.executable, "-c", WORKLOAD], str(tmp_path / "inv.json"), seconds=300)
    assert inv["exit_code"] == 0 and inv["calls"] >= 3, inv
    r = kernels.test_calls(inv, repeats=2, log_dir=str(tmp_path / "logs"))
    assert r["counts"]["WRONG"] == 0, r["calls"]
    assert r["counts"]["PASSED"] >= 1, r["calls"]
    assert r["shapes_replayed"] >= 3 and r["gpu"]

"""First-use verification: every kernel family passes its clean and corrupted cases on this B200, the report is
cached per device, and a checked engine carries it."""
import pytest
import torch

from sdcguard_b200.ops import verify

pytestmark = pytest.mark.gpu


def test_every_kernel_family_verifies():
    rep = verify.run(torch.device("cuda:0"))
    assert rep["ok"], rep
    assert set(rep["cases"]) == {"gemm", "norm", "attention", "spot"}
    assert rep["seconds"] < 30


def test_cached_and_required_by_the_engine():
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve.engine import LLMEngine
    a = verify.verified(torch.device("cuda:0"))
    assert verify.verified(torch.device("cuda:0")) is a
    eng = LLMEngine(TINY, device="cuda:0", checked=True, num_blocks=32, max_prefill_tokens=256, max_num_seqs=4,
                    max_model_len=256)
    assert eng.verification is a and a["ok"]

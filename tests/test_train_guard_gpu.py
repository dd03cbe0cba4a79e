"""Training guard: protected linear layers give the same outputs and gradients as plain PyTorch (fp32 reference
tolerance for bf16), raise no alarm on clean steps, and report an injected accumulator flip in each of the three
GEMMs of a layer (forward, dX, dW) at the right place."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 256)).cuda().bfloat16()


def test_checked_training_step_matches_plain_and_is_clean():
    from sdcguard_b200.train.guard import SDCGuard
    ref = _model()
    m = copy.deepcopy(ref)
    g = SDCGuard()
    g.protect(m)
    x = torch.randn(64, 256, device="cuda").bfloat16()
    xr = x.clone().requires_grad_(True)
    xm = x.clone().requires_grad_(True)
    ref(xr).float().pow(2).mean().backward()
    with g.at_step(0):
        m(xm).float().pow(2).mean().backward()
    for (n1, p1), (n2, p2) in zip(ref.named_parameters(), m.named_parameters()):
        err = (p1.grad.float() - p2.grad.float()).abs().max().item()
        assert err <= 0.02 * p1.grad.float().abs().max().item() + 1e-6, (n1, err)
    assert (xr.grad.float() - xm.grad.float()).abs().max().item() <= 0.02 * xr.grad.float().abs().max().item()
    cov = g.coverage()
    assert g.events == [] and cov["checks"] > 0 and cov["unchecked_calls"] == 0 and cov["worst_clean_z"] < 6


@pytest.mark.parametrize("phase,row,col", [("fwd", 5, 200), ("dx", 7, 130), ("dw", 3, 17)])
def test_injected_flip_in_each_training_gemm_is_reported(phase, row, col):
    from sdcguard_b200.train.guard import SDCGuard
    m = _model()
    g = SDCGuard()
    g.protect(m)
    x = torch.randn(64, 256, device="cuda").bfloat16().requires_grad_(True)
    g.inject_next("2", phase, row, col, 29)
    with g.at_step(0):
        m(x).float().pow(2).mean().backward()
    assert len(g.events) == 1, [e.detail for e in g.events]
    d = g.events[0].detail
    assert d["layer"] == "2" and d["phase"] == phase and d["row"] == row and d["block"] == col // 128

"""Attaching the serving guard to a plain PyTorch model on a B200: the selected bf16 nn.Linear layers run on the
checked tcgen05 GEMM (outputs match an fp32 reference within bf16 rounding), their checks run and read clean, an
accumulator flip is caught and captured, a changed weight shows in verify_weights until refresh, a share leaves the
other layers on PyTorch, gradients and fp32 inputs fall back, and detach restores the model."""
import pytest
import torch

from sdcguard_b200.serve.attach import attach
from sdcguard_b200.serve.settings import CheckSettings

pytestmark = pytest.mark.gpu


def _model(dev):
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 384, bias=False),
                            torch.nn.Linear(384, 256))
    return m.to(dev, torch.bfloat16)


def test_attached_model_runs_checked():
    dev = torch.device("cuda:0")
    m = _model(dev)
    ref = _model(dev)
    g = attach(m, settings=CheckSettings())
    assert g.model.check_coverage()["layers_checked"] == 3
    x = torch.randn(2, 37, 256, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        y = m(x)
        r = ref.float()(x.float())
    torch.testing.assert_close(y.float(), r, rtol=3e-2, atol=3e-2)
    assert g.poll() == []
    cov = g.coverage_report()
    assert cov["ops"] == 3 and cov["ops_checked"] == 3 and cov["checks"] > 0 and cov["alarms"] == 0
    assert g.verify_weights() == []
    # a changed weight: exact in verify_weights, forgiven after refresh
    with torch.no_grad():
        m[2].weight[5, 7] += 1.0
    assert g.verify_weights() == ["2"]
    assert g.refresh() == 3 and g.verify_weights() == []
    # gradients (training) and fp32 inputs take the original forward, counted
    n0 = g.model.fallback_calls
    m(x.float().to(torch.bfloat16).requires_grad_())
    assert g.model.fallback_calls > n0
    g.detach()
    assert type(m[0]) is torch.nn.Linear
    with torch.no_grad():
        torch.testing.assert_close(m(x), torch.nn.Sequential(*m)(x))


def test_share_and_alarm():
    from sdcguard_b200.ops import gemm
    dev = torch.device("cuda:0")
    m = _model(dev)
    g = attach(m, share=0.5, settings=CheckSettings())
    rep = g.layer_report()
    assert 1 <= sum(r["checked"] for r in rep) <= 2 and any("outside the share" in (r["reason"] or "") for r in rep)
    g.detach()
    m = _model(dev)
    g = attach(m, settings=CheckSettings())
    st = m[0].__dict__["_sdcguard_state"]
    x = torch.randn(64, 256, device=dev, dtype=torch.bfloat16)
    gemm.checked_linear(x, st.cw, g.model.state.state, st.slot, inject=(3, 100, 1 << 29))
    ev = g.poll()
    assert ev and ev[0].detector == "checksum" and ev[0].detail["row"] == 3
    g.detach()

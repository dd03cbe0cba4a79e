"""A protected model under torch.compile on the GPU: checked steps run the checked GEMMs through the custom
operators (checks counted, no false alarm, outputs and gradients as eager), unchecked steps run the plain graph,
and a flipped accumulator bit in a compiled checked step is reported."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_compiled_checked_steps():
    from sdcguard_b200.train.guard import SDCGuard
    dev = torch.device("cuda")
    torch.manual_seed(0)

    def make():
        torch.manual_seed(0)
        return torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 256)).to(
            dev, torch.bfloat16)
    m, ref = make(), make()
    g = SDCGuard(check_every=2, device=dev)
    g.protect(m)
    cm = torch.compile(m, fullgraph=True)
    x = torch.randn(128, 256, device=dev, dtype=torch.bfloat16)
    for step in range(4):
        with g.on_step(step):
            y = cm(x)
            y.float().pow(2).mean().backward()
    yr = ref(x)
    yr.float().pow(2).mean().backward()
    assert torch.allclose(y.float(), yr.float(), atol=2e-2, rtol=2e-2)
    cov = g.coverage()
    assert cov["alarms"] == 0 and cov["checked_calls"] == 4 and cov["steps_checked"] == 2
    assert cov["checks"] >= 2 * 5                      # two checked steps: 2 forward + 2 dX + 2 dW (first layer's dX unneeded)
    g.inject_next("2", "fwd", 3, 40, 29)
    with g.on_step(4):
        cm(x).float().sum().backward()
    assert len(g.events) == 1 and g.events[0].detail["layer"] == "2"

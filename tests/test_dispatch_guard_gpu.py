"""Operator-level guard on a B200: bf16 mm / addmm run on the checked tcgen05 GEMM (native path, the check in the
GEMM epilogue), bmm and torch._grouped_mm on PyTorch's kernels checked afterwards. Gradients match plain PyTorch
within bf16 tolerance, clean steps raise no alarm, and injected flips are reported in the right op and place."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


class Block(torch.nn.Module):
    def __init__(self, d=512, heads=4):
        super().__init__()
        self.qkv = torch.nn.Linear(d, 3 * d)
        self.o = torch.nn.Linear(d, d)
        self.up = torch.nn.Linear(d, 4 * d)
        self.down = torch.nn.Linear(4 * d, d)
        self.h = heads

    def forward(self, x):
        B, T, d = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.h, -1).permute(2, 0, 3, 1, 4).reshape(3, B * self.h, T, -1)
        att = (torch.bmm(q, k.transpose(1, 2)) * (q.shape[-1] ** -0.5)).softmax(-1)
        y = torch.bmm(att, v).view(B, self.h, T, -1).transpose(1, 2).reshape(B, T, d)
        x = x + self.o(y)
        return x + self.down(torch.nn.functional.gelu(self.up(x)))


def _setup():
    torch.manual_seed(0)
    ref = Block().cuda().bfloat16()
    return ref, copy.deepcopy(ref), torch.randn(4, 256, 512, device="cuda").bfloat16()


def test_clean_training_step_native_and_library_paths():
    from sdcguard_b200.train.dispatch import DispatchGuard
    ref, m, x = _setup()
    ref(x).float().pow(2).mean().backward()
    g = DispatchGuard()
    with g.at_step(0):
        m(x).float().pow(2).mean().backward()
    for (n1, p1), (_, p2) in zip(ref.named_parameters(), m.named_parameters()):
        err = (p1.grad.float() - p2.grad.float()).abs().max().item()
        assert err <= 0.03 * p1.grad.float().abs().max().item() + 1e-6, (n1, err)
    cov = g.coverage()
    assert g.events == [], [e.detail for e in g.events]
    # 4 linear layers x (fwd, dX, dW), minus dX of the first (its input needs no grad)
    assert cov["native"] == 11 and cov["checked"] >= 6 and cov["unchecked"] == 0, cov
    assert cov["worst_clean_z"] < 6 and cov["unjudged"] == 0


@pytest.mark.parametrize("which", ["native", "bmm"])
def test_injected_flip_reported(which):
    from sdcguard_b200.train.dispatch import DispatchGuard
    _, m, x = _setup()
    g = DispatchGuard()
    orig = g._checked
    fired = []

    def spy(name, func, args, kwargs):
        if not fired and ((which == "bmm" and name == "aten::bmm") or (which == "native" and name == "aten::addmm")):
            fired.append(name)
            if which == "bmm":
                g.inject_next(row=9, col=200, bit=14, batch=2)      # bf16 output, top exponent bit
            else:
                g.inject_next(row=9, col=260, bit=27)               # fp32 accumulator
        return orig(name, func, args, kwargs)
    g._checked = spy
    with g.at_step(0):
        m(x).float().pow(2).mean().backward()
    assert len(g.events) >= 1, g.coverage()
    d = g.events[0].detail
    if which == "bmm":
        assert d["op"].startswith("aten::bmm") and d["row"] == 2 * 256 + 9 and d["block"] == 1
    else:
        assert d["op"].startswith("aten::addmm") and d["row"] == 9 and d["block"] == 2


def test_grouped_mm_checked_per_group():
    from sdcguard_b200.train.dispatch import DispatchGuard
    torch.manual_seed(1)
    a = torch.randn(384, 256, device="cuda").bfloat16()
    w = torch.randn(3, 256, 512, device="cuda").bfloat16()
    offs = torch.tensor([128, 256, 384], device="cuda", dtype=torch.int32)
    g = DispatchGuard()
    with g.at_step(0):
        torch._grouped_mm(a, w, offs)
    assert g.events == [] and g.coverage()["checked"] == 3
    with g.at_step(1):
        g.inject_next(row=200, col=20, bit=14)       # group 1 holds rows 128..255
        torch._grouped_mm(a, w, offs)
    assert len(g.events) == 1

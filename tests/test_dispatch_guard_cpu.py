"""Operator-level guard (TorchDispatchMode) on CPU: every aten matmul of a training step is seen and checked on the
library path (PyTorch's product, checked afterwards), gradients are unchanged, clean steps raise no alarm, an
injected flip in a bmm or an mm is reported in the right op, unchecked matmuls are counted, and the guard is idle on
steps off its schedule."""
import copy

import pytest
import torch

from sdcguard_b200.train.dispatch import DispatchGuard


class Tiny(torch.nn.Module):
    def __init__(self, d=256, heads=2):
        super().__init__()
        self.q = torch.nn.Linear(d, d)
        self.k = torch.nn.Linear(d, d, bias=False)
        self.o = torch.nn.Linear(d, d)
        self.h = heads

    def forward(self, x):                       # (B, T, d) -> scalar
        B, T, d = x.shape
        q = self.q(x).view(B, T, self.h, -1).transpose(1, 2).reshape(B * self.h, T, -1)
        k = self.k(x).view(B, T, self.h, -1).transpose(1, 2).reshape(B * self.h, T, -1)
        att = torch.bmm(q, k.transpose(1, 2)).softmax(-1)
        y = torch.bmm(att, q).view(B, self.h, T, -1).transpose(1, 2).reshape(B, T, d)
        return self.o(y).float().pow(2).mean()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_clean_step_same_grads_no_alarm(dtype):
    torch.manual_seed(0)
    ref = Tiny().to(dtype)
    m = copy.deepcopy(ref)
    x = torch.randn(2, 160, 256, dtype=dtype)
    ref(x).backward()
    g = DispatchGuard(device="cpu")
    with g.at_step(0):
        m(x).backward()
    for p1, p2 in zip(ref.parameters(), m.parameters()):
        assert torch.equal(p1.grad, p2.grad)              # same library products: bit-identical
    cov = g.coverage()
    assert g.events == [], [e.detail for e in g.events]
    assert cov["checked"] >= 10 and cov["unchecked"] == 0 and cov["worst_clean_z"] < 3, cov
    assert cov["flop_coverage"] == 1.0


def test_injected_flip_in_bmm_is_reported():
    torch.manual_seed(1)
    m = Tiny().bfloat16()
    x = torch.randn(2, 160, 256, dtype=torch.bfloat16)
    g = DispatchGuard(device="cpu")
    with g.at_step(0):
        # linear layers run addmm/mm first: q, k; the first bmm is the 3rd checked op
        seen = []
        orig = g._checked

        def spy(name, func, args, kwargs):
            seen.append(name)
            if name == "aten::bmm" and seen.count("aten::bmm") == 1:
                g.inject_next(row=17, col=140, bit=14, batch=3)
            return orig(name, func, args, kwargs)
        g._checked = spy
        m(x).backward()
    assert len(g.events) == 1, [e.detail for e in g.events]
    d = g.events[0].detail
    assert d["op"].startswith("aten::bmm") and d["row"] == 3 * 160 + 17 and d["block"] == 1


def test_injected_flip_in_mm_precise_path():
    torch.manual_seed(2)
    a = torch.randn(96, 512, dtype=torch.bfloat16)
    b = torch.randn(512, 384, dtype=torch.bfloat16)
    g = DispatchGuard(device="cpu", precise=True)
    with g.at_step(0):
        c0 = a @ b
    assert g.events == [] and g.coverage()["worst_clean_z"] < 3
    with g.at_step(1):
        g.inject_next(row=5, col=300, bit=15)            # the fp32 bit just below bf16 precision
        c1 = a @ b
    assert len(g.events) == 1 and g.events[0].detail["row"] == 5 and g.events[0].detail["block"] == 2
    assert (c1.float() - c0.float()).abs().max() < 1.0


def test_other_matmul_ops_checked_and_unchecked_counted():
    torch.manual_seed(3)
    g = DispatchGuard(device="cpu")
    A = torch.randn(4, 32, 64)
    B = torch.randn(4, 64, 200)
    base = torch.randn(4, 32, 200)
    with g.at_step(0):
        torch.baddbmm(base, A, B, beta=0.5, alpha=2.0)
        torch.addbmm(base[0], A, B)
        torch.mv(A[0], B[0, :, 0])
        torch.addmv(base[0, :, 0], A[0], B[0, :, 1])
        torch.addmm(base[0], A[0], B[0], beta=0.25, alpha=3.0)
        torch._int_mm(torch.randint(-8, 8, (32, 64), dtype=torch.int8), torch.randint(-8, 8, (64, 32),
                      dtype=torch.int8))
    cov = g.coverage()
    assert g.events == [], [e.detail for e in g.events]
    assert cov["checked"] == 5 and cov["unchecked"] == 1 and cov["unchecked_ops"] == {"aten::_int_mm": 1}
    assert 0 < cov["flop_coverage"] < 1


def test_off_schedule_steps_are_untouched():
    g = DispatchGuard(device="cpu", check_every=4)
    a, b = torch.randn(16, 32), torch.randn(32, 16)
    for step in range(1, 4):
        with g.at_step(step):
            a @ b
    assert g.coverage()["checked"] == 0
    with g.at_step(4):
        a @ b
    assert g.coverage()["checked"] == 1 and g.coverage()["checks"] == 1


def test_reduced_precision_flags_restored():
    m = torch.backends.cuda.matmul
    before = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    g = DispatchGuard(device="cpu")
    with g.at_step(0):
        assert not m.allow_bf16_reduced_precision_reduction and not m.allow_fp16_reduced_precision_reduction
    assert (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction) == before


def test_schedule_windows_drive_on_step():
    g = DispatchGuard(device="cpu", check_every=100)
    a, b = torch.randn(8, 16), torch.randn(16, 8)
    g.after_restart(5, steps=2)
    for step in range(4, 9):
        with g.on_step(step) as checked:
            a @ b
        assert checked == (step in (5, 6))
    assert g.coverage()["checked"] == 2

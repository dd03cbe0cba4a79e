"""Weight-only quantized layers on the CPU: group quantization round trip and the effective weights' arithmetic
(rnd((q - z) s) in bf16, symmetric and zero-point formats, INT4 and INT8)."""
import pytest
import torch

from sdcguard_b200.ops.quant import QuantWeights


@pytest.mark.parametrize("bits,zp", [(4, False), (4, True), (8, False), (8, True)])
def test_effective_weight_cpu(bits, zp):
    torch.manual_seed(bits + zp)
    w = (torch.randn(64, 256) * 0.05).bfloat16()
    qw = QuantWeights.quantize(w, bits=bits, group=64, zero_points=zp)
    assert qw.codes.dtype == torch.uint8 and qw.codes.shape == (64, 256 // (2 if bits == 4 else 1))
    eff = qw.effective_weight()
    ref = qw.reference_weight()
    assert torch.equal(eff.double(), ref)
    # quantization error within a step of each group's scale (a rounded zero point can cost half a step at the ends)
    step = qw.scales.double().repeat_interleave(64, dim=1)
    assert bool(((eff.double() - w.double()).abs() <= 1.0 * step + 2 ** -8 * w.double().abs() + 1e-6).all())
    # the codes' fingerprint moves when one code bit flips
    fp0 = qw.fingerprint().clone()
    qw.codes[3, 5] ^= 1
    assert not torch.equal(qw.fingerprint(), fp0)

"""Weight-only quantized layers on the GPU: the dequantization kernel gives the effective weights bit for bit, the
checked GEMM on them matches a float64 product and checks clean, an injected flip is reported, and a flipped code
bit is seen by the codes' fingerprint."""
import pytest
import torch

from sdcguard_b200.numerics import abft
from sdcguard_b200.ops import gemm
from sdcguard_b200.ops.quant import CheckedQuantLinear, QuantWeights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,zp", [(4, False), (4, True), (8, False), (8, True)])
def test_quant_layer_checked(bits, zp):
    dev = torch.device("cuda")
    torch.manual_seed(bits * 2 + zp)
    w = (torch.randn(512, 1024, device=dev) * 0.03).bfloat16()
    qw = QuantWeights.quantize(w, bits=bits, group=128, zero_points=zp)
    eff = qw.effective_weight()
    assert torch.equal(eff.double().cpu(), qw.reference_weight())
    layer = CheckedQuantLinear(qw)
    st = gemm.StateTable(dev, 2)
    s0, s1 = st.add("quant (ABFT GEMM)", layer.cw.nb), st.add("inj (ABFT GEMM)", layer.cw.nb)
    x = torch.randn(256, 1024, device=dev).bfloat16()
    y = layer(x, st.state, s0)
    ref = x.double() @ eff.double().t()
    assert float(((y.double() - ref).abs() / (ref.abs() + 1e-2)).max()) < 2 ** -7
    layer(x, st.state, s1, inject=(17, 300, 1 << 29))
    rows = st.read()
    assert rows[0]["z"] < 6 and rows[0]["unjudged"] == 0
    assert rows[1]["z"] > abft.Z_ALARM and rows[1]["row"] == 17 and rows[1]["block"] == 2
    assert layer.weights_unchanged()
    qw.codes[10, 7] ^= 0x10
    assert not layer.weights_unchanged()

"""Weight-only quantized layers as vLLM lays them out (CPU): int32 words unpacked lowest bits first along the packed
dimension, layouts read from the parameters' input / output / packed dimensions, the three readings of zero points
against a float64 restatement written here, the unit-vector probe, and the layers this module refuses."""
from types import SimpleNamespace

import pytest
import torch

from sdcguard_b200.ops import quant


def _pack(q: torch.Tensor, bits: int, axis: int) -> torch.Tensor:
    """Independent packer: 32 / bits codes per int32 word along `axis`, lowest bits first."""
    per = 32 // bits
    q = q.to(torch.int64).movedim(axis, -1)
    q = q.reshape(*q.shape[:-1], q.shape[-1] // per, per)
    words = torch.zeros(q.shape[:-1], dtype=torch.int64)
    for j in range(per):
        words |= q[..., j] << (bits * j)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words.movedim(-1, axis)


def _param(t, **dims):
    p = torch.nn.Parameter(t, requires_grad=False)
    for name, v in dims.items():
        setattr(p, name, v)
    return p


def _wtype(bits, bias):
    return SimpleNamespace(size_bits=bits, bias=bias, is_integer=lambda: True, has_bias=lambda: bias != 0)


def _kernel(bits, bias, k, n, group, zero_points, g_idx=False, name="MarlinLinearKernel"):
    cfg = SimpleNamespace(weight_type=_wtype(bits, bias), group_size=group, zero_points=zero_points,
                          has_g_idx=g_idx, partition_weight_shape=(k, n))
    kernel = type(name, (), {})()          # the reader looks at the kernel class's name (Machete: "fma")
    kernel.config, kernel.w_q_name, kernel.w_s_name = cfg, "wq", "ws"
    kernel.w_zp_name = "wz" if zero_points else None
    kernel.w_gidx_name = "g_idx" if g_idx else None
    return kernel


def test_unpack_words_roundtrip():
    g = torch.Generator().manual_seed(0)
    for bits in (4, 8):
        q = torch.randint(0, 1 << bits, (16, 24), generator=g)
        for axis in (0, 1):
            if q.shape[axis] % (32 // bits):
                continue
            assert torch.equal(quant.unpack_words(_pack(q, bits, axis), bits, axis), q.to(torch.int32))


def test_gptq_layout_symmetric_int4():
    g = torch.Generator().manual_seed(1)
    n, k, group = 32, 256, 128
    q = torch.randint(0, 16, (n, k), generator=g)
    s = (torch.rand(n, k // group, generator=g) * 0.02 + 1e-3).to(torch.bfloat16)
    layer = torch.nn.Module()
    layer.wq = _param(_pack(q.t(), 4, 0), input_dim=0, output_dim=1, packed_dim=0, packed_factor=8)  # [k/8, n]
    layer.ws = _param(s.t().contiguous(), input_dim=0, output_dim=1)                                  # [k/g, n]
    qw = quant.from_vllm(layer, _kernel(4, 8, k, n, group, False))
    want = ((q.double() - 8) * s.double().repeat_interleave(group, 1)).to(torch.bfloat16)
    assert qw.zero_mode == "subtract" and torch.equal(qw.effective_weight(), want)


def test_compressed_tensors_layout_with_zero_points_and_modes():
    g = torch.Generator().manual_seed(2)
    n, k, group = 16, 256, 64
    q = torch.randint(0, 16, (n, k), generator=g)
    z = torch.randint(0, 16, (n, k // group), generator=g)
    s = (torch.rand(n, k // group, generator=g) * 3.0 + 0.01).to(torch.bfloat16)
    layer = torch.nn.Module()
    layer.wq = _param(_pack(q, 4, 1), input_dim=1, output_dim=0, packed_dim=1, packed_factor=8)       # [n, k/8]
    layer.ws = _param(s, input_dim=1, output_dim=0)                                                   # [n, k/g]
    layer.wz = _param(_pack(z, 4, 0), input_dim=1, output_dim=0, packed_dim=0, packed_factor=8)       # [n/8, k/g]
    assert quant.from_vllm(layer, _kernel(4, 0, k, n, group, True, name="MacheteLinearKernel")).zero_mode == "fma"
    qw = quant.from_vllm(layer, _kernel(4, 0, k, n, group, True))
    sd, zd, qd = s.double().repeat_interleave(group, 1), z.double().repeat_interleave(group, 1), q.double()
    assert torch.equal(qw.effective_weight(), ((qd - zd) * sd).to(torch.bfloat16))
    zs = -(s.double() * z.double()).to(torch.bfloat16).double().repeat_interleave(group, 1)
    fma = qw.with_zero_mode("fma")
    two = qw.with_zero_mode("two_roundings")
    assert torch.equal(fma.effective_weight(), (qd * sd + zs).to(torch.bfloat16))
    assert torch.equal(two.effective_weight(), ((qd * sd).to(torch.bfloat16).double() + zs).to(torch.bfloat16))
    for m in (qw, fma, two):
        assert torch.equal(m.effective_weight().double(), m.reference_weight())
    # one rounding or two: some weights differ between the readings
    assert not torch.equal(fma.effective_weight(), two.effective_weight())


def test_probe_and_refusals():
    g = torch.Generator().manual_seed(3)
    n, k, group = 24, 512, 128
    qw = quant.QuantWeights.quantize(torch.randn(n, k, generator=g), bits=4, group=group)
    w = qw.effective_weight()
    cols = quant.probe_columns(k, group, limit=32)
    assert len(cols) == 32 and {0, 127, 128, 511} <= set(cols) and len(set(cols)) == 32
    exact = lambda x: (x.double() @ w.double().t()).to(torch.bfloat16)          # noqa: E731
    assert quant.probe(exact, w, cols) == {"ok": True, "columns": 32, "mismatches": 0, "first": None}
    w2 = w.clone()
    w2[5, cols[3]] = -w2[5, cols[3]] if w2[5, cols[3]] != 0 else 1.0
    wrong = lambda x: (x.double() @ w2.double().t()).to(torch.bfloat16)        # noqa: E731
    r = quant.probe(wrong, w, cols)
    assert not r["ok"] and r["mismatches"] == 1 and r["first"]["input"] == cols[3] and r["first"]["output"] == 5
    layer = torch.nn.Module()
    layer.wq = _param(torch.zeros(k // 8, n, dtype=torch.int32), input_dim=0, output_dim=1, packed_dim=0)
    layer.ws = _param(torch.ones(1, n, dtype=torch.bfloat16), input_dim=0, output_dim=1)
    with pytest.raises(quant.Unsupported, match="after accumulating"):
        quant.from_vllm(layer, _kernel(4, 8, k, n, -1, False))
    layer.g_idx = torch.randperm(k, generator=g) // group
    with pytest.raises(quant.Unsupported, match="reordering"):
        quant.from_vllm(layer, _kernel(4, 8, k, n, group, False, g_idx=True))


def test_plugin_quant_hook_on_cpu():
    """The plugin's hook of quantized kernels: the layer is read before the kernel's own loading, the kernel is
    probed after it, and a layer that cannot be adopted keeps the kernel's path with its reason (on the CPU: no
    CUDA device; a kernel whose products contradict the restated weights; a layout the reader refuses)."""
    from sdcguard_b200.serve import vllm_plugin as vp
    n, k, group = 16, 256, 128
    g = torch.Generator().manual_seed(4)
    q = torch.randint(0, 16, (n, k), generator=g)
    s = (torch.rand(n, k // group, generator=g) * 0.02 + 1e-3).to(torch.bfloat16)
    w_eff = ((q.double() - 8) * s.double().repeat_interleave(group, 1)).to(torch.bfloat16)
    loads = []

    class FakeKernel:
        def __init__(self, group_size=group, skew=0.0):
            self.config = SimpleNamespace(weight_type=_wtype(4, 8), group_size=group_size, zero_points=False,
                                          has_g_idx=False, partition_weight_shape=(k, n))
            self.w_q_name, self.w_s_name, self.w_zp_name, self.w_gidx_name = "wq", "ws", None, None
            self.skew = skew

        def process_weights_after_loading(self, layer):
            loads.append(layer.prefix)
            layer.wq = torch.nn.Parameter(torch.zeros(1, dtype=torch.int32), requires_grad=False)   # "repacked"

        def apply_weights(self, layer, x, bias=None):
            w = w_eff.double().clone()
            w[0, 0] += self.skew
            return (x.double() @ w.t()).to(torch.bfloat16)

    assert vp._patch_quant([FakeKernel]) == [FakeKernel]

    def layer(prefix):
        m = torch.nn.Module()
        m.prefix = prefix
        m.wq = _param(_pack(q.t(), 4, 0), input_dim=0, output_dim=1, packed_dim=0, packed_factor=8)
        m.ws = _param(s.t().contiguous(), input_dim=0, output_dim=1)
        return m
    before = len(vp._LEFT_OUT)
    FakeKernel().process_weights_after_loading(layer("q.ok"))
    FakeKernel(skew=1.0).process_weights_after_loading(layer("q.skewed"))
    FakeKernel(group_size=-1).process_weights_after_loading(layer("q.channelwise"))
    assert loads == ["q.ok", "q.skewed", "q.channelwise"]
    why = {name: r for name, r, _ in vp._LEFT_OUT[before:]}
    assert "not on a CUDA device" in why["q.ok"]                       # read, probed bit-exact, then refused: CPU
    assert why["q.skewed"].startswith("quantized kernel differs") and "subtract: 1 of" in why["q.skewed"]
    assert why["q.channelwise"].startswith("quantized layer not read: Unsupported")
    x = torch.randn(3, k).to(torch.bfloat16)
    assert torch.equal(FakeKernel().apply_weights(layer("q.unadopted"), x), FakeKernel().apply_weights(None, x))

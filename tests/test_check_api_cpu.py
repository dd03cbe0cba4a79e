"""The reference-style public API on the CPU: check_matmul / check_linear on products another library computed
(clean, a flipped output value, bias / alpha / beta, batched, non-finite outputs, unsupported dtypes), SDCError from
a guard built with raise_on_alert, and the lazily imported top-level names."""
import math

import pytest
import torch

import sdcguard_b200 as sg


def _ab(m=64, k=256, n=384, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dtype)
    b = (torch.randn(k, n, generator=g) * 0.05).to(dtype)
    return a, b


def test_check_matmul_clean_and_flipped():
    a, b = _ab()
    c = a @ b
    r = sg.check_matmul(a, b, c)
    assert r.ok and r.judged and 0 <= r.max_z < 6 and not r.nonfinite
    bad = c.clone()
    bad[17, 200] += 0.5
    r = sg.check_matmul(a, b, bad)
    assert not r.ok and r.row == 17 and r.col_block == 200 // 128 and r.max_z > 6 and r.noise > 0


def test_check_linear_bf16_bias_and_alpha_beta():
    x, w_t = _ab(m=32, k=512, n=256, dtype=torch.bfloat16)
    w = w_t.t().contiguous()
    bias = torch.randn(256).to(torch.bfloat16)
    y = torch.nn.functional.linear(x.float(), w.float(), bias.float()).to(torch.bfloat16)
    assert sg.check_linear(x.view(4, 8, 512), w, bias, y.view(4, 8, 256)).ok
    y2 = y.clone()
    y2[3, 100] = y2[3, 100] * 2 + 1
    r = sg.check_linear(x, w, bias, y2)
    assert not r.ok and r.row == 3 and r.col_block == 0
    a, b = _ab()
    bias2 = torch.randn(384)
    c = 0.5 * bias2 + 2.0 * (a @ b)
    assert sg.check_matmul(a, b, c, bias2, alpha=2.0, beta=0.5).ok
    assert not sg.check_matmul(a, b, c, bias2, alpha=1.0, beta=0.5).ok


def test_check_matmul_batched_nonfinite_and_dtypes():
    g = torch.Generator().manual_seed(3)
    a = torch.randn(3, 16, 128, generator=g)
    b = torch.randn(3, 128, 256, generator=g) * 0.1
    c = torch.bmm(a, b)
    assert sg.check_matmul(a, b, c).ok
    c[2, 5, 130] = float("nan")
    r = sg.check_matmul(a, b, c)
    assert not r.ok and r.nonfinite and math.isinf(r.max_z) and (r.batch, r.row, r.col_block) == (2, 5, 1)
    a[1] = float("inf")                       # non-finite inputs: those blocks are not judged, not alarms
    c2 = torch.bmm(torch.randn(3, 16, 128, generator=g), b)
    assert sg.check_matmul(torch.full((16, 128), float("inf")), b[0], c2[0]).judged is False
    assert sg.check_matmul(a[0].to(torch.int32), b[0].to(torch.int32), c2[0].to(torch.int32)) is None


def test_sdc_error_and_top_level_names():
    from sdcguard_b200.train.guard import SDCError, SDCGuard
    assert sg.SDCError is SDCError and sg.SDCGuard is SDCGuard
    for name in sg.__all__:
        assert getattr(sg, name) is not None
    assert hasattr(sg.ServeGuard, "attach")
    e = SDCError("x", [1, 2])
    assert isinstance(e, RuntimeError) and e.events == [1, 2]
    with pytest.raises(AttributeError):
        sg.not_a_name


def test_guard_raise_on_alert_reads_then_raises():
    """A checked step whose state table holds an alarm: with raise_on_alert the read-back logs the alert, then
    raises SDCError carrying it (the state row is written here by hand, as the GEMM's epilogue would)."""
    import struct
    from sdcguard_b200.train.guard import SDCError, SDCGuard
    g = SDCGuard(device="cpu", raise_on_alert=True)
    slot = g.table.add("blocks.0.mlp.fwd (ABFT GEMM)", 2)
    zbits = struct.unpack("<I", struct.pack("<f", 40.0))[0]
    nbits = struct.unpack("<I", struct.pack("<f", 0.5))[0]
    g.table.state[slot] = torch.tensor([(zbits << 32) | 6, nbits, 3, 0], dtype=torch.int64)
    with pytest.raises(SDCError) as ei:
        g.flush(step=7)
    assert len(ei.value.events) == 1 and ei.value.events[0].detail["layer"] == "blocks.0.mlp"
    assert len(g.events) == 1 and "step 7" in str(ei.value)
    quiet = SDCGuard(device="cpu")
    s2 = quiet.table.add("blocks.0.mlp.fwd (ABFT GEMM)", 2)
    quiet.table.state[s2] = torch.tensor([(zbits << 32) | 6, nbits, 3, 0], dtype=torch.int64)
    assert len(quiet.flush(step=7)) == 1          # without raise_on_alert: events only

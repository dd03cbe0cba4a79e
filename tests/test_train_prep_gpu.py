"""Device-built checksum rows of the training GEMMs' B operands (csrc/train_prep.cu) against the float64 PyTorch
restatement (numerics.abft.weight_checksums), the transposes bit-exact, and a training step under bf16 autocast
checked with no false alarm and with an injected flip found."""
import pytest
import torch

from sdcguard_b200.numerics import abft
from sdcguard_b200.ops import gemm

pytestmark = pytest.mark.gpu


def _parts_value(wc: torch.Tensor) -> torch.Tensor:
    """(6 nb, k) bf16 parts -> (nb, 2, k) float64 plain / signed sums."""
    v = wc.double().view(-1, 2, 3, wc.shape[1]).sum(2)
    return v


@pytest.mark.parametrize("r,c", [(256, 384), (200, 136), (1024, 768)])
def test_rowblock_matches_reference(r, c):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(r + c)
    m = (torch.randn(r, c, device=dev, generator=g) * 0.5).bfloat16()
    cw = gemm.CheckedWeight.of_transpose(m)
    ref = abft.weight_checksums(m.t().contiguous())
    assert torch.equal(cw.weight, m.t().contiguous())
    a, b = _parts_value(cw.cs.wc), _parts_value(ref.wc)
    scale = b.abs().amax() + 1e-30
    assert float(((a - b).abs() / scale).max()) < 2 ** -20
    assert torch.allclose(cw.cs.wstat, ref.wstat, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("n,k", [(384, 256), (136, 200), (768, 1024)])
def test_colblock_matches_reference(n, k):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(n * 3 + k)
    w = (torch.randn(n, k, device=dev, generator=g) * 0.05).bfloat16()
    b = torch.randn(n, device=dev, generator=g) * 0.1
    cw = gemm.CheckedWeight.on_device(w, b)
    ref = abft.weight_checksums(w, b)
    a, r = _parts_value(cw.cs.wc), _parts_value(ref.wc)
    assert float(((a - r).abs() / (r.abs().amax() + 1e-30)).max()) < 2 ** -20
    assert torch.allclose(cw.cs.wstat, ref.wstat, rtol=1e-4, atol=1e-6)
    assert torch.allclose(cw.cs.bsum, ref.bsum) and cw.cs.bias_max == 0.0     # not read back (no host sync)
    # the checked GEMM with these checksums: clean
    x = torch.randn(256, k, device=dev, generator=g).bfloat16()
    st = gemm.StateTable(dev, 1)
    s = st.add("prep (ABFT GEMM)", cw.nb)
    y = gemm.checked_linear(x, cw, st.state, s)
    torch.cuda.synchronize()
    row = st.read()[0]
    assert row["z"] < 6 and row["unjudged"] == 0
    ref_y = x.double() @ w.double().t() + b.double()
    assert float(((y.double() - ref_y).abs() / (ref_y.abs() + 1e-2)).max()) < 2 ** -7


def test_prep_scratch_is_left_zero():
    """Each prep launch finalizes its own statistics and clears the shared scratch: back-to-back preps of different
    block counts give the same statistics as fresh ones (to the last bits, which the fp32 atomic accumulation
    leaves order-dependent; a scratch left uncleared would add a whole previous sum)."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(7)
    ws = [(torch.randn(n, 256, device=dev, generator=g) * 0.05).bfloat16() for n in (1024, 128, 640)]
    first = [gemm.CheckedWeight.on_device(w).cs.wstat.clone() for w in ws]
    for _ in range(3):
        for w, f in zip(ws, first):
            assert torch.allclose(gemm.CheckedWeight.on_device(w).cs.wstat, f, rtol=1e-5, atol=0)
            t = gemm.CheckedWeight.of_transpose(w)
            assert torch.allclose(t.cs.wstat, abft.weight_checksums(w.t().contiguous()).wstat, rtol=1e-4, atol=1e-6)
    acc = gemm._PREP_ACC[ws[0].device]
    torch.cuda.synchronize()
    assert int((acc != 0).sum()) == 0


def test_autocast_training_step_checked():
    from sdcguard_b200.train.guard import SDCGuard
    dev = torch.device("cuda")
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 256)).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    guard = SDCGuard(check_every=1, device=dev)
    guard.protect(model)
    x = torch.randn(128, 256, device=dev)
    for step in range(3):
        with guard.on_step(step):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = model(x).float().pow(2).mean()
            loss.backward()
        opt.step()
        opt.zero_grad()
    cov = guard.coverage()
    assert cov["alarms"] == 0 and cov["checked_calls"] == 6 and cov["unchecked_calls"] == 0
    assert all(p.grad is None for p in model.parameters())
    assert model[0].weight.dtype == torch.float32
    guard.inject_next("0", "dw", 5, 17, 29)
    with guard.on_step(3):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(x).float().pow(2).mean()
        loss.backward()
    assert len(guard.events) == 1 and guard.events[0].detail["phase"] == "dw"


def test_alarm_evidence_recheck_and_confirm(tmp_path):
    from sdcguard_b200.train.guard import SDCGuard
    from sdcguard_b200.utils.events import load_evidence
    dev = torch.device("cuda")
    torch.manual_seed(1)
    model = torch.nn.Sequential(torch.nn.Linear(256, 384), torch.nn.GELU(), torch.nn.Linear(384, 256)).to(
        dev, torch.bfloat16)
    guard = SDCGuard(check_every=1, device=dev, recompute=True, evidence_dir=str(tmp_path), confirm_runs=5)
    guard.protect(model)
    x = torch.randn(64, 256, device=dev, dtype=torch.bfloat16)
    with guard.on_step(0):
        y = guard.checkpoint(model, x)
        y.float().pow(2).mean().backward()
    assert guard.events == [] and guard.recompute.checks == 1
    guard.inject_next("2", "fwd", 7, 200, 29)         # one flipped exponent bit, this step only
    with guard.on_step(1):
        model(x).float().sum().backward()
    assert len(guard.events) == 1
    d = guard.events[0].detail
    assert d["captured"]["row"] == 7 and d["captured"]["block"] == 200 // 128
    assert d["recheck"]["verdict"] == "output_wrong"
    assert d["confirm"]["runs"] == 5 and d["confirm"]["reproduced"] is False    # a transient flip: not on replay
    ev = load_evidence(d["evidence"])
    assert ev["layer"] == "2" and ev["x_row"].shape == (384,) and ev["w_block"].shape == (128, 384)


def test_fused_optimizer_keeps_checks_current():
    """AdamW(fused=True) updates weights without bumping their version counters: every checked step must use the
    updated weights (its checked forward equals plain PyTorch on the current weights) and raise no alarm."""
    from sdcguard_b200.train.guard import SDCGuard
    dev = torch.device("cuda")
    torch.manual_seed(3)
    m = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(), torch.nn.Linear(512, 256)).to(dev)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-2, fused=True)
    guard = SDCGuard(check_every=1, device=dev)
    guard.protect(m)
    x = torch.randn(128, 256, device=dev)
    for step in range(4):
        with guard.on_step(step):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = m(x)
                loss = y.float().pow(2).mean()
            loss.backward()
        # the checked forward of this step against PyTorch on the weights it had (bf16 autocast arithmetic)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            h = torch.nn.functional.gelu(torch.nn.functional.linear(x, m[0].weight, m[0].bias))
            ref = torch.nn.functional.linear(h, m[2].weight, m[2].bias)
        assert float((y.float() - ref.float()).abs().max()) < 0.02 * float(ref.float().abs().max()), step
        opt.step()
        opt.zero_grad()
    assert guard.coverage()["alarms"] == 0


@pytest.mark.parametrize("r,c", [(256, 384), (200, 136), (16384, 768), (70, 50)])
def test_transpose_kernel(r, c):
    from sdcguard_b200.ops import gemm
    m = torch.randn(r, c, device="cuda").bfloat16()
    assert torch.equal(gemm.transpose(m), m.t().contiguous())
    big = torch.randn(r, c + 8, device="cuda").bfloat16()[:, 3:3 + c]     # a strided, unaligned view
    assert torch.equal(gemm.transpose(big), big.t().contiguous())

"""Block-scaled fp8 checked GEMM and the activation quantizer, against plain PyTorch fp32 computations of the same
ops: quantizer codes and scales exactly; GEMM output against the fp32 product of the dequantized operands; clean
scores below the alarm line; injected accumulator flips located; the quantizer's replay check."""
import math

import pytest
import torch

from sdcguard_b200.numerics import abft

pytestmark = pytest.mark.gpu


def _ref_quant(x):
    from sdcguard_b200.ops.fp8 import pow2_scale, to_e4m3
    m, k = x.shape
    xb = x.float().view(m, k // 128, 128)
    sa = pow2_scale(xb.abs().amax(-1))
    q = to_e4m3(xb / sa[..., None]).view(m, k)
    return q, sa


def test_quantizer_matches_torch_and_replay_check():
    from sdcguard_b200.ops.fp8 import quantize_act, sf_chunks
    torch.manual_seed(0)
    x = (torch.randn(300, 1024, device="cuda") * torch.logspace(-3, 2, 1024, device="cuda")).bfloat16()
    xa = quantize_act(x)
    q, sa = _ref_quant(x)
    assert torch.equal(xa.sa, sa)
    assert torch.equal(xa.q.view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(xa.sf, sf_chunks(sa))
    assert torch.allclose(xa.row_sq, xa.dequantized().pow(2).sum(-1), rtol=1e-4)
    st = torch.zeros(2, 4, dtype=torch.int64, device="cuda")
    rows = torch.tensor([3, 150, 299], dtype=torch.int32, device="cuda")
    quantize_act(x, out=xa, rows=rows, check=st[0])
    xa.q.view(torch.uint8)[150, 517] ^= 1
    quantize_act(x, out=xa, rows=rows, check=st[1])
    d0, d1 = (abft.decode_state_row(r) for r in st.cpu().tolist())
    assert d0["z"] == 0 and d0["checks"] == 1
    assert d1["z"] == math.inf and d1["flat"] == 150 * 1024 + 516     # the first column of the differing 4
    # a corrupted scale-factor byte of a sampled row (row 3, K block 2) is caught too
    xa.q.view(torch.uint8)[150, 517] ^= 1
    st.zero_()
    xa.sf[0, 2, 3 * 16 + 1] ^= 1
    quantize_act(x, out=xa, rows=rows, check=st[0])
    d = abft.decode_state_row(st[0].cpu().tolist())
    assert d["z"] == math.inf and d["flat"] == 3 * 1024 + 256, d


@pytest.mark.parametrize("m,n,k", [(256, 1024, 1024), (100, 384, 512), (64, 4096, 4096), (1000, 2048, 2048)])
def test_fp8_gemm_matches_dequantized_fp32_and_is_clean(m, n, k):
    from sdcguard_b200.ops import gemm
    from sdcguard_b200.ops.fp8 import Fp8Weight, checked_linear_fp8, quantize_act
    torch.manual_seed(1)
    # magnitudes that differ by row, by K block and by weight block: every scale factor must reach its own rows
    rs = torch.logspace(-2, 2, m, device="cuda")[torch.randperm(m, device="cuda")][:, None]
    ks = torch.logspace(-1, 1, k // 128, device="cuda").repeat_interleave(128)[None, :]
    x = (torch.randn(m, k, device="cuda") * rs * ks).bfloat16()
    ws = torch.logspace(-1, 1, n // 128, device="cuda").repeat_interleave(128)[:, None]
    w = (torch.randn(n, k, device="cuda") * 0.02 * ws * ks.flip(1)).bfloat16()
    fw = Fp8Weight(w)
    xa = quantize_act(x)
    st = gemm.StateTable("cuda", 2)
    slot = st.add("fp8", fw.nb)
    y = checked_linear_fp8(xa, fw, st.state, slot)
    torch.cuda.synchronize()
    ref = xa.dequantized() @ fw.dequantized().t()
    err = ((y.float() - ref).abs() / (ref.abs().amax(1, keepdim=True) + 1e-6)).max().item()
    assert err <= 2 ** -7, err
    d = st.read()[0]
    assert d["checks"] == 1 and d["unjudged"] == 0 and d["z"] < 2.0, d


@pytest.mark.parametrize("bit", [30, 27, 24, 31])
def test_fp8_gemm_injected_flip_is_located(bit):
    from sdcguard_b200.ops import gemm
    from sdcguard_b200.ops.fp8 import Fp8Weight, checked_linear_fp8, quantize_act
    torch.manual_seed(2)
    m, n, k = 512, 1024, 2048
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    fw = Fp8Weight(w)
    xa = quantize_act(x)
    st = gemm.StateTable("cuda", 2)
    slot = st.add("fp8", fw.nb)
    y0 = checked_linear_fp8(xa, fw, st.state, slot)
    st.read(reset=True)
    row = 301
    col = int(y0[row].float().abs().argmax())
    checked_linear_fp8(xa, fw, st.state, slot, inject=(row, col, 1 << bit))
    d = st.read()[0]
    assert d["z"] > abft.Z_ALARM and d["row"] == row and d["block"] == col // 128, d


def test_fp8_decoder_serves_clean_and_close_to_bf16():
    """The decoder with fp8 projections: same greedy tokens as bf16 on most steps, checks run, no alarm."""
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve.engine import LLMEngine
    prompts = torch.randint(0, TINY.vocab, (4, 96), generator=torch.Generator().manual_seed(0)).pin_memory()
    outs = {}
    for prec in ("bf16", "fp8"):
        eng = LLMEngine(TINY, device="cuda:0", checked=True, num_blocks=64, max_prefill_tokens=512, max_num_seqs=8,
                        sample_every=2, max_model_len=512, precision=prec)
        outs[prec] = eng.generate(prompts, [96, 80, 64, 33], 4)
        ev = eng.guard.poll()
        cov = eng.guard.coverage_report()
        assert not ev and cov["checks"] > 0 and cov["unjudged"] == 0, (prec, ev, cov)
        if prec == "fp8":
            assert any("fp8" in n for n in eng.model.state.names) and any("quant" in n for n in eng.model.state.names)
    assert (outs["bf16"] == outs["fp8"]).float().mean().item() >= 0.5

"""Serving plugin hooks: periodic polling, attribution of an alarm to the request whose row it was in, the
require rule, and the weight scan attached through the hooks."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(checked=True):
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve.engine import LLMEngine
    return LLMEngine(TINY, device="cuda:0", checked=checked, num_blocks=64, max_prefill_tokens=512, max_num_seqs=8,
                     sample_every=2, max_model_len=512)


def test_hooks_poll_and_attribute_a_weight_fault_to_requests():
    from sdcguard_b200.serve.plugin import register
    from sdcguard_b200.utils.inject import flip_bit_
    eng = _engine()
    hooks = register(eng, poll_every=2, require=True, scan_mb=64)
    prompts = torch.randint(0, 1024, (3, 40), generator=torch.Generator().manual_seed(0)).pin_memory()
    eng.generate(prompts, [40, 30, 20], 3)
    hooks.poll()
    assert hooks.alerts == [] and hooks.polls >= 1 and hooks.report()["coverage"]["checks"] > 0
    # a flipped exponent bit in a weight after registration: the GEMM checksum rows still describe the clean
    # weight, so the layer's check fires; the weight scan names the weight
    w = eng.model.layers[0].qkv
    flip_bit_(w, 5 * w.shape[1] + 17, 14)
    eng.generate(prompts, [40, 30, 20], 3)
    hooks.poll()
    dets = {a["detector"] for a in hooks.alerts}
    assert "checksum" in dets and "weights" in dets, hooks.alerts
    gemm = [a for a in hooks.alerts if a["detector"] == "checksum"]
    assert any(a["detail"]["layer"].startswith("layers.0.qkv") for a in gemm)
    assert all(a["request"] in (0, 1, 2) for a in gemm if a["request"] is not None)


def test_require_refuses_unchecked_model():
    from sdcguard_b200.serve.plugin import UncheckedServingRefused, register
    eng = _engine(checked=False)
    with pytest.raises(UncheckedServingRefused):
        register(eng, require=True)

"""Non-blocking poll: poll(wait=False) never waits for the GPU; an alarm raised before it is reported by the next
poll once the asynchronous read has landed, and a blocking poll reports everything up to now."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine():
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve.engine import LLMEngine
    return LLMEngine(TINY, device="cuda:0", checked=True, num_blocks=64, max_prefill_tokens=512, max_num_seqs=8,
                     max_model_len=512)


def test_nonblocking_poll_reports_one_poll_late():
    eng = _engine()
    prompts = torch.randint(0, 1000, (2, 64)).pin_memory()
    eng.generate(prompts, [64, 40], 2)
    assert eng.guard.poll() == []                              # clean, blocking
    eng.model.inject_next("L0.down", 3, 5, 1 << 30)           # an exponent bit of one accumulator element
    eng.generate(prompts, [64, 40], 2)
    first = eng.guard.poll(wait=False)                         # starts the read; nothing landed before it
    assert first == []
    torch.cuda.synchronize()
    second = eng.guard.poll(wait=False)                        # the read has landed
    hits = [e for e in second if e.detector == "checksum" and "layers.0.down" in e.detail["layer"]]
    assert hits and hits[0].detail["row"] == 3 and hits[0].detail["block"] == 0
    assert eng.guard.poll() == []                              # the alarm is reported once


def test_plugin_attributes_late_alarm_to_its_request():
    from sdcguard_b200.serve.plugin import register
    eng = _engine()
    hooks = register(eng, poll_every=1, require=True)
    prompts = torch.randint(0, 1000, (2, 64)).pin_memory()
    eng.model.inject_next("L1.qkv", 70, 9, 1 << 30)          # token 70 of the batch: the second request (64 + 6)
    eng.generate(prompts, [64, 40], 2)
    torch.cuda.synchronize()
    hooks.poll(wait=True)
    hits = [a for a in hooks.alerts if a["detector"] == "checksum"]
    assert hits and hits[0]["request"] == 1


def test_alarm_is_captured_and_rechecked_in_float64():
    eng = _engine()
    prompts = torch.randint(0, 1000, (2, 64)).pin_memory()
    eng.generate(prompts, [64, 40], 2)
    eng.guard.poll()
    # a compute fault: an exponent bit of one accumulator element of layer 0's down projection
    eng.model.inject_next("L0.down", 11, 130, 1 << 29)
    eng.generate(prompts, [64, 40], 2)
    ev = [e for e in eng.guard.poll() if e.detector == "checksum" and "layers.0.down" in e.detail["layer"]]
    assert ev and ev[0].detail["captured"]["row"] == 11 and ev[0].detail["captured"]["block"] == 1
    assert ev[0].detail["recheck"]["verdict"] == "output_wrong"
    # a memory fault: one weight bit of layer 1's qkv projection flipped after registration
    w = eng.model.layers[1].qkv
    w.view(torch.int16)[7, 3] ^= 1 << 13
    eng.generate(prompts, [64, 40], 2)
    ev = [e for e in eng.guard.poll() if e.detector == "checksum" and "layers.1.qkv" in e.detail["layer"]]
    assert ev and ev[0].detail["recheck"]["verdict"] == "weights_changed"

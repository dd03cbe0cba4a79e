"""Attaching the serving guard to a plain PyTorch model, host side: layer selection by share and offset, the reason
recorded for every layer left unchecked, and detach. (The checked forward itself runs in the GPU test.)"""
import pytest
import torch

from sdcguard_b200.serve.attach import attach
from sdcguard_b200.serve.guard import ServeGuard
from sdcguard_b200.serve.settings import CheckSettings, layer_selected


def _model():
    return torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.ReLU(), torch.nn.Linear(128, 64),
                               torch.nn.Linear(64, 24))


def test_attach_on_cpu_leaves_every_layer_unchecked_with_its_reason():
    m = _model()
    g = attach(m, settings=CheckSettings())
    rep = g.layer_report()
    assert [r["layer"] for r in rep] == ["0", "2", "3"]
    assert all(not r["checked"] and r["reason"] == "not on a CUDA device" for r in rep)
    assert g.model.check_coverage()["layers_checked"] == 0
    assert g.poll() == [] and g.coverage_report()["ops"] == 0
    x = torch.randn(3, 64)
    torch.testing.assert_close(m(x), m(x))
    g.detach()


def test_share_selection_matches_the_settings_rule():
    chosen = [i for i in range(64) if layer_selected(i, 0.25, 0)]
    assert 8 <= len(chosen) <= 24
    both = [i for i in range(64) if layer_selected(i, 0.5, 0) or layer_selected(i, 0.5, 1)]
    assert both == list(range(64))               # two replicas at share 1/2 cover every layer once
    assert not any(layer_selected(i, 0.5, 0) and layer_selected(i, 0.5, 1) for i in range(64))


def test_classmethod_entry_and_double_attach(monkeypatch):
    m = _model()
    g = ServeGuard.attach(m, settings=CheckSettings())
    assert isinstance(g, ServeGuard)
    from sdcguard_b200.train import swap
    swap.take_over(m[0], object())             # a layer that is already checked
    with pytest.raises(ValueError):
        attach(m, settings=CheckSettings())
    swap.give_back(m[0])

"""Check settings from the environment: share parsing, the replica partition of the layer share, switches."""
import pytest

from sdcguard_b200.serve.settings import CheckSettings, layer_selected, parse_share


def test_share_forms_and_bounds():
    assert parse_share("1/8") == parse_share("12.5%") == parse_share("0.125") == 0.125
    for bad in ("nan", "-0.1", "1.5", "x", "1/0"):
        with pytest.raises((ValueError, ZeroDivisionError)):
            parse_share(bad)


@pytest.mark.parametrize("share", [1 / 8, 1 / 4, 1 / 2, 1 / 3])
def test_offsets_partition_every_layer_once(share):
    n = 28 * 4
    replicas = int(round(1 / share))
    owners = [[o for o in range(replicas) if layer_selected(i, share, o)] for i in range(n)]
    assert all(len(x) == 1 for x in owners)                 # every layer exactly once across replicas
    counts = [sum(1 for x in owners if x[0] == o) for o in range(replicas)]
    assert max(counts) - min(counts) <= 3                   # spread evenly
    # every projection kind appears in every replica's share (the golden-ratio stride, not every R-th layer)
    for o in range(replicas):
        kinds = {i % 4 for i in range(n) if layer_selected(i, share, o)}
        assert kinds == {0, 1, 2, 3}


def test_environment_switches(monkeypatch):
    monkeypatch.setenv("SDCGUARD_SHARE", "1/4")
    monkeypatch.setenv("SDCGUARD_OFFSET", "2")
    monkeypatch.setenv("SDCGUARD_ATTN", "0")
    monkeypatch.setenv("SDCGUARD_SPOT", "off")
    monkeypatch.setenv("SDCGUARD_NORMS", "maybe")           # unreadable: stays on
    monkeypatch.setenv("SDCGUARD_Z", "-3")                  # unreadable: 6
    s = CheckSettings.from_env()
    assert s.share == 0.25 and s.offset == 2 and not s.attn and not s.spot and s.norms and s.z_alarm == 6.0
    assert s.gemm_checked(0, 0) == layer_selected(0, 0.25, 2)
    monkeypatch.setenv("SDCGUARD_SHARE", "lots")
    assert CheckSettings.from_env().share == 1.0             # unreadable: every layer

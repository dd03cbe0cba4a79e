"""Model-free search of real threaded code (lifetime.realsearch over lifetime.toys) and component conformance of
serve/pd.py with CPU mocks: the buggy toys are found with the rule they break, the fixed toys are clean, and the
pd.py components conform (the misuse scenario is caught)."""
import pytest

from sdcguard_b200.lifetime import conformance, realsearch, toys


@pytest.mark.parametrize("toy,rule", [("push", "R1"), ("pull", "R1"), ("wakeup", "liveness")])
def test_buggy_toy_found(toy, rule):
    r = realsearch.search(lambda: toys.TOYS[toy](fixed=False))
    assert r.baseline_clean
    assert any(rule in f.rules for f in r.findings), realsearch.text(r)


@pytest.mark.parametrize("toy", ["push", "pull", "wakeup"])
def test_fixed_toy_clean(toy):
    r = realsearch.search(lambda: toys.TOYS[toy](fixed=True))
    assert r.baseline_clean and r.findings == [], realsearch.text(r)


def test_pd_components_conform():
    r = conformance.run_component_conformance()
    assert r["conforms"], r
    assert r["scenarios"]["early_release"]["rules"]

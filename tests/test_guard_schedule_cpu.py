"""Training-guard schedule on CPU (no kernels run): the every-N schedule, the dense window after a restart, and
the window that a loss or gradient-norm spike (or a non-finite value) opens."""
import math

from sdcguard_b200.train.guard import SDCGuard


def _guard(every=10):
    return SDCGuard(check_every=every, device="cpu")


def test_every_n_and_restart_window():
    g = _guard(10)
    assert [s for s in range(25) if g.should_check(s)] == [0, 10, 20]
    g.after_restart(100, steps=5)
    assert [s for s in range(98, 108) if g.should_check(s)] == [100, 101, 102, 103, 104]


def test_spike_and_nonfinite_open_windows():
    g = _guard(1000)
    for s in range(1, 40):
        assert not g.observe(s, loss=2.0 + 0.01 * math.sin(s), grad_norm=1.0 + 0.01 * math.cos(s))
    assert not g.should_check(41)
    assert g.observe(40, loss=9.0)                        # a spike far above the robust spread
    assert g.should_check(41) and g.should_check(90) and not g.should_check(91)
    assert g.anomalies[-1]["checked_through"] == 90
    assert g.observe(95, grad_norm=float("nan"))          # non-finite: always a window
    assert g.should_check(96)
    assert not g.observe(200, loss=None)

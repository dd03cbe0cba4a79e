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


# ------------------------------------------------------------------ Hugging Face callback (event order of a step)
class _State:
    def __init__(self, step):
        self.global_step = step


class _Control:
    should_training_stop = False


def test_hf_callback_reads_results_before_the_optimizer_step():
    from sdcguard_b200.train.hf import SDCGuardCallback
    from sdcguard_b200.utils.events import SDCEvent
    g = _guard(2)
    cb = SDCGuardCallback(g, stop_on_alert=True)
    ctl = _Control()
    cb.on_step_begin(None, _State(0), ctl)
    assert g.active                                        # step 0 is scheduled: window open
    g.events.append(SDCEvent(detector="checksum", step=0, detail={"layer": "fc", "phase": "dw"}))
    cb.on_pre_optimizer_step(None, _State(0), ctl)
    assert not g.active and g.steps_checked == 1           # closed and read before the weights change
    assert ctl.should_training_stop                        # the alert stops training after this step
    cb.on_step_end(None, _State(1), ctl)
    assert g.steps_checked == 1                            # nothing left to close
    cb.on_step_begin(None, _State(1), _Control())
    assert not g.active                                    # step 1 is not scheduled


def test_hf_callback_spike_checks_the_very_next_step():
    from sdcguard_b200.train.hf import SDCGuardCallback
    g = _guard(1000)
    cb = SDCGuardCallback(g)
    for step in range(1, 40):                              # the Trainer logs after counting the step
        cb.on_log(None, _State(step + 1), _Control(), logs={"loss": 2.0 + 0.01 * math.sin(step)})
    cb.on_log(None, _State(41), _Control(), logs={"loss": 50.0})    # step 40 spiked
    cb.on_step_begin(None, _State(41), _Control())
    assert g.active                                        # global_step 41 is the next step: checked
    cb.on_train_end(None, _State(41), _Control())
    assert not g.active


def test_evidence_files_load_without_unpickling_code(tmp_path):
    import torch
    from sdcguard_b200.tools import casefile
    from sdcguard_b200.utils.events import load_evidence
    x = torch.randn(4, 64).bfloat16()
    w = torch.randn(128, 64).bfloat16()
    y = (x.float() @ w.float().t()).bfloat16()
    case = casefile.capture(x, w, y, row=1, block=0, note="unit")
    path = str(tmp_path / "case.pt")
    h = casefile.save(case, path)
    back = load_evidence(path)
    assert casefile.sha256(back) == h and back["row"] == 1 and back["x_row"].device.type == "cpu"
    assert not casefile.recheck(back)["output_wrong"]

    class Evil:
        def __reduce__(self):
            return (print, ("code ran",))
    torch.save({"x": Evil()}, str(tmp_path / "evil.pt"))
    import pickle
    try:
        load_evidence(str(tmp_path / "evil.pt"))
        raise AssertionError("a file holding an arbitrary object loaded")
    except pickle.UnpicklingError:
        pass

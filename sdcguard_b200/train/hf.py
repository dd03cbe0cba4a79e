"""Hugging Face Trainer callback: runs the training guard around every training step (forward and backward of
the protected linear layers are checked on the guard's schedule) and reads the results at the step's end.

    guard = SDCGuard(check_every=10)
    trainer = Trainer(model=guard.protect(model), ..., callbacks=[SDCGuardCallback(guard)])

Reference: `SDCGuardCallback` (src/sdcguard/hf.py:33).
"""
from __future__ import annotations

from transformers import TrainerCallback

from .guard import SDCGuard


class SDCGuardCallback(TrainerCallback):
    def __init__(self, guard: SDCGuard, stop_on_alert: bool = False):
        self.guard = guard
        self.stop_on_alert = stop_on_alert
        self._ctx = None

    def on_step_begin(self, args, state, control, **kw):
        step = state.global_step
        self._ctx = self.guard.at_step(step, force=self.guard.should_check(step))   # schedule and windows
        self._ctx.__enter__()

    def on_log(self, args, state, control, logs=None, **kw):
        """Loss and gradient-norm spikes in the trainer's logs open a checked window (SDCGuard.observe)."""
        if logs:
            self.guard.observe(state.global_step, loss=logs.get("loss"), grad_norm=logs.get("grad_norm"))
        return control

    def on_step_end(self, args, state, control, **kw):
        if self._ctx is not None:
            n0 = len(self.guard.events)
            self._ctx.__exit__(None, None, None)
            self._ctx = None
            if self.stop_on_alert and len(self.guard.events) > n0:
                control.should_training_stop = True
        return control

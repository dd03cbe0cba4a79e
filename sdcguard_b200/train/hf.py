"""Hugging Face Trainer callback: runs the training guard around the training steps it schedules and reads the
results back before the optimizer applies the step's gradients.

    guard = SDCGuard(check_every=10)
    trainer = Trainer(model=model, ..., callbacks=[SDCGuardCallback(guard, stop_on_alert=True)])

Event order inside one Trainer step, and what the callback does at each:

  on_step_begin          a checked window opens when `guard.should_check(step)` (every N-th step, a window after a
                         restart, a window after a loss / grad-norm spike); a window left open by a step that never
                         reached the optimizer is closed first
  forward + backward     every protected linear layer's forward, dX and dW GEMMs are checked while the window is open
  on_pre_optimizer_step  the window closes and its results are read: a corrupted gradient is reported before the
                         weights change, and with stop_on_alert the Trainer stops after this step
  on_step_end            closes a window the optimizer hook did not (a step without an optimizer step)
  on_log                 the logged loss and grad norm feed `guard.observe`; the Trainer has already counted the
                         step when it logs, so the logged step is `global_step - 1` and a spike's window starts at
                         the next step `on_step_begin` sees
  on_train_end           closes anything still open

The model is protected at `on_train_begin` when the guard has no layers yet. Needs transformers with the
`on_pre_optimizer_step` event (4.46 or newer).

Reference: `SDCGuardCallback` (src/sdcguard/hf.py:33): the same hooks, closing before the optimizer step.
"""
from __future__ import annotations

import logging
from typing import Optional

from transformers import TrainerCallback

from .guard import SDCGuard

log = logging.getLogger("sdcguard")


class SDCGuardCallback(TrainerCallback):
    def __init__(self, guard: Optional[SDCGuard] = None, stop_on_alert: bool = False, check_every: int = 20):
        self.guard = guard if guard is not None else SDCGuard(check_every=check_every)
        self.stop_on_alert = stop_on_alert
        self._window = None                # the open `at_step` context of the current step, if any
        self._reported = 0                 # guard.events already handed to the log

    # -------------------------------------------------------------------------------- Trainer events
    def on_train_begin(self, args, state, control, model=None, **kw):
        if model is not None and not self.guard.modules:
            self.guard.protect(model)
        return control

    def on_step_begin(self, args, state, control, **kw):
        self._finish(control)
        step = state.global_step
        if self.guard.should_check(step):
            self._window = self.guard.at_step(step, force=True)
            self._window.__enter__()
        return control

    def on_pre_optimizer_step(self, args, state, control, **kw):
        self._finish(control)
        return control

    def on_step_end(self, args, state, control, **kw):
        self._finish(control)
        return control

    def on_train_end(self, args, state, control, **kw):
        self._finish(control)
        return control

    def on_log(self, args, state, control, logs=None, **kw):
        if logs:
            self.guard.observe(state.global_step - 1, loss=logs.get("loss"), grad_norm=logs.get("grad_norm"))
            logs["sdcguard/steps_checked"] = self.guard.steps_checked
            logs["sdcguard/alerts"] = len(self.guard.events)
        return control

    # -------------------------------------------------------------------------------- internals
    def _finish(self, control) -> None:
        """Close the open window (its exit reads the step's results), log alerts not yet logged, and ask the
        Trainer to stop when one came in and stop_on_alert is set."""
        win, self._window = self._window, None
        if win is not None:
            win.__exit__(None, None, None)
        fresh = self.guard.events[self._reported:]
        self._reported = len(self.guard.events)
        for ev in fresh:
            log.warning("sdcguard: check failed at training step %s: %s", ev.step, ev.detail)
        if fresh and self.stop_on_alert:
            control.should_training_stop = True

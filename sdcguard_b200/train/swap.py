"""How the training guard takes over a linear layer: the layer's class is swapped for a subclass whose forward asks
the guard state stored on the layer, and falls back to the original forward when there is none.

Replacing the module object (the obvious way) breaks three things a training job relies on: a copy of the model
(copy.deepcopy, torch.optim.swa_utils.AveragedModel, an EMA shadow) would share the guard, the state table and
the checksum caches of the original; torch.save(model) would pickle the guard and need this package to load; and
code that holds a reference to the original layer (another module's attribute, a hook, an optimizer's parameter
groups built by module) would keep the unchecked one. With a class swap the layer object, its parameters and its
state_dict stay the same, and:

  * copy.deepcopy and pickling produce plain layers of the original class without the guard's attributes (a copy
    is a separate model, unchecked until protected itself), so a model saved while checked loads anywhere;
  * a shallow copy (nn.DataParallel replicas) keeps the subclass and the guard and computes with its own weights,
    since the forward is a method and reads the weights of the layer it is called on;
  * `isinstance(layer, nn.Linear)` holds; the subclass keeps the original's name, so the model prints the same.

This is the mechanism torch.nn.utils.parametrize uses to change a module's behaviour in place.

Reference: src/sdcguard/_swap.py:29-73 (`guarded_class`, `take_over`, `give_back`).
"""
from __future__ import annotations

import copyreg
import threading

import torch

STATE = "_sdcguard_state"        # the per-layer guard state, in the instance __dict__
_SUBCLASSES: dict = {}
_LOCK = threading.Lock()


def _reconstruct_plain(base, state):
    obj = base.__new__(base)
    obj.__dict__.update(state)
    return obj


def checked_class(base: type) -> type:
    """The one subclass of `base` whose forward goes through the stored guard state."""
    with _LOCK:
        sub = _SUBCLASSES.get(base)
        if sub is not None:
            return sub

        def forward(self, input):  # noqa: A002  (nn.Linear's argument name: layer(input=x) keeps working)
            st = self.__dict__.get(STATE)
            if st is None:
                return base.forward(self, input)
            return st.forward(self, input)

        def __reduce_ex__(self, protocol):
            # copies and pickles: a plain object of the original class, the guard's attributes left out
            target = base if type(self) is sub else type(self)
            state = {k: v for k, v in self.__dict__.items() if k != STATE}
            return copyreg._reconstructor, (target, object, None), state

        sub = type(base.__name__, (base,), {"forward": forward, "__reduce_ex__": __reduce_ex__,
                                            "_sdcguard_base": base, "__module__": base.__module__,
                                            "__qualname__": base.__qualname__, "__doc__": base.__doc__})
        _SUBCLASSES[base] = sub
        return sub


def is_checked(mod: torch.nn.Module) -> bool:
    return type(mod) in _SUBCLASSES.values() and STATE in mod.__dict__


def take_over(mod: torch.nn.Module, state) -> None:
    """Route mod's forward through state.forward(mod, input)."""
    if type(mod) not in _SUBCLASSES.values():
        mod.__class__ = checked_class(type(mod))
    mod.__dict__[STATE] = state


def give_back(mod: torch.nn.Module) -> None:
    """Undo take_over: the original class and none of the guard's attributes."""
    base = getattr(type(mod), "_sdcguard_base", None)
    if base is not None and type(mod) in _SUBCLASSES.values():
        mod.__class__ = base
    mod.__dict__.pop(STATE, None)


def state_of(mod: torch.nn.Module):
    return mod.__dict__.get(STATE)

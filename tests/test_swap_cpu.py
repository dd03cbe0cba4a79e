"""The training guard's class swap: the protected layer stays the same object with the same parameters and
state_dict, copies and pickles are plain layers of the original class, and release() gives the class back."""
import copy
import io
import pickle

import torch

from sdcguard_b200.train import swap
from sdcguard_b200.train.guard import SDCGuard


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.ReLU(), torch.nn.Linear(32, 8))


def test_protect_keeps_objects_and_copies_are_plain():
    m = _model()
    first = m[0]
    keys = list(m.state_dict())
    params = [id(p) for p in m.parameters()]
    g = SDCGuard(check_every=1, device="cpu")
    g.protect(m)
    assert m[0] is first and swap.is_checked(m[0]) and isinstance(m[0], torch.nn.Linear)
    assert type(m[0]) is not torch.nn.Linear and type(m[0]).__name__ == "Linear"
    assert list(m.state_dict()) == keys and [id(p) for p in m.parameters()] == params
    assert len(g.modules) == 2 and [s.name for s in g.modules] == ["0", "2"]
    x = torch.randn(4, 16)
    ref = _model()(x)
    with g.on_step(0):
        y = m(x)                      # CPU: counted as unchecked, computed by F.linear
    assert torch.equal(y, ref) and g.unchecked == 2
    # copies: plain layers of the original class, unchecked, with their own weights
    c = copy.deepcopy(m)
    assert type(c[0]) is torch.nn.Linear and not swap.is_checked(c[0])
    assert c[0].weight is not m[0].weight and torch.equal(c[0].weight, m[0].weight)
    buf = io.BytesIO()
    torch.save(m, buf)
    buf.seek(0)
    loaded = torch.load(buf, weights_only=False)
    assert type(loaded[2]) is torch.nn.Linear and torch.equal(loaded(x), ref)
    p = pickle.loads(pickle.dumps(m[2]))
    assert type(p) is torch.nn.Linear
    # protecting twice does not double the layers; release gives the class back
    g.protect(m)
    assert len(g.modules) == 2
    g.release(m)
    assert type(m[0]) is torch.nn.Linear and not swap.is_checked(m[0]) and torch.equal(m(x), ref)


def test_shallow_copy_keeps_guard_with_own_weights():
    m = _model()
    g = SDCGuard(check_every=1, device="cpu")
    g.protect(m)
    r = m[0]._replicate_for_data_parallel()     # how nn.DataParallel makes its replicas: a shallow __dict__ copy
    assert swap.is_checked(r) and r is not m[0]
    r.weight = torch.nn.Parameter(torch.zeros(32, 16))     # replicate() then gives the replica its own weights
    r.bias = torch.nn.Parameter(torch.zeros(32))
    with g.on_step(0):
        assert torch.equal(r(torch.ones(2, 16)), torch.zeros(2, 32))

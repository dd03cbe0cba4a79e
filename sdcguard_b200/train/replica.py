"""Data-parallel replica check: after the optimizer step every data-parallel replica must hold bit-identical
weights. Each rank fingerprints all its parameters (`ops.fingerprint`, combined in parameter order), the ranks
exchange the three numbers and vote; the dissenting rank is the suspect.

Reference: `weight_fingerprint` and `check_replicas` (src/sdcguard/replica.py:36-76).
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch
import torch.distributed as dist

from ..ops.fingerprint import fingerprint
from ..utils.events import SDCEvent, device_identity, gather_identities, job_rank, suspect_event
from .canary import majority

MASK = (1 << 64) - 1


def weight_fingerprint(params: Iterable[torch.Tensor], seed: int = 0) -> tuple[int, int, int]:
    """(sum F0, position-mixed sum F1, parameter count) over the parameters, in order."""
    ps = [p.detach().contiguous() for p in params]
    if not ps:
        return 0, 0, 0
    by_dev: dict = {}
    for i, p in enumerate(ps):
        by_dev.setdefault(p.device, []).append(i)
    fps: list = [None] * len(ps)
    for dev, idx in by_dev.items():
        out = fingerprint([ps[i] for i in idx], seed).cpu().tolist()
        for i, v in zip(idx, out):
            fps[i] = v
    a = b = 0
    for i, (f0, f1) in enumerate(fps):
        a = (a + (f0 & MASK)) & MASK
        b = (b + ((f1 & MASK) * (2 * i + 1))) & MASK          # odd multipliers keep it a bijection per slot
    return a, b, len(ps)


def check_replicas(params: Iterable[torch.Tensor], group=None, step: Optional[int] = None) -> list[SDCEvent]:
    """Collective; the same event list on every rank."""
    fp = weight_fingerprint(params)
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rows: list = [None] * world
    if world > 1:
        dist.all_gather_object(rows, fp, group=group)
    else:
        rows = [fp]
    top, bad = majority([tuple(r) for r in rows])
    if not bad:
        return []
    ids = gather_identities(group) if world > 1 else [device_identity()]
    me = dist.get_rank(group) if world > 1 else 0
    return [suspect_event("replica", step, bad, ids, me, {"no_majority": top is None},
                          to_job_rank=lambda r: job_rank(group, r))]

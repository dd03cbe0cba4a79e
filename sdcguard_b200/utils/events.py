"""Alert events and their log: the record every detector emits (schema of src/sdcguard/events.py:44-87 kept so
tooling that reads the reference's JSONL alert logs reads these too), device identity for pulling the bad GPU,
and the rollback-checkpoint rule (src/sdcguard/events.py:90-103)."""
from __future__ import annotations

import json
import logging
import os
import socket
import time
from dataclasses import asdict, dataclass, field
from typing import Optional

log = logging.getLogger("sdcguard")


def load_evidence(path: str) -> dict:
    """Read an evidence or case file (`.pt`) that may come from another node: tensors land on the CPU (a file saved
    on cuda:N loads on a host with fewer GPUs) and only plain data is unpickled (tensors, dicts, lists, strings,
    numbers), so a crafted file cannot run code. Callers move the tensors to their device themselves."""
    import torch
    return torch.load(path, map_location="cpu", weights_only=True)


def plain(obj):
    """`obj` as plain JSON-able data (dicts, lists, strings, numbers), for evidence files read by `load_evidence`."""
    return json.loads(json.dumps(obj, default=str))


def device_identity(device=None) -> dict:
    """Host, rank, and (for a CUDA device) name, UUID, PCI bus id and physical index of the GPU. The fields follow
    the reference's identity record (src/sdcguard/events.py:14-41), which names the GPU to pull by UUID and bus."""
    import torch
    info: dict = {"host": socket.gethostname(), "rank": None, "device": None, "gpu_uuid": None}
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            info["rank"] = dist.get_rank()
    except Exception:  # noqa: BLE001
        pass
    if device is None:
        return info
    dev = torch.device(device)
    info["device"] = str(dev)
    if dev.type != "cuda":
        return info
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    try:
        props = torch.cuda.get_device_properties(idx)
        info["gpu_name"] = props.name
        uuid = str(getattr(props, "uuid", "") or "")
        if uuid:
            info["gpu_uuid"] = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            info["pci_bus_id"] = "%08X:%02X:%02X.0" % (getattr(props, "pci_domain_id", 0) or 0, bus,
                                                        getattr(props, "pci_device_id", 0) or 0)
    except Exception:  # noqa: BLE001  identity is best effort
        pass
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = [v.strip() for v in vis.split(",")] if vis else None
    info["gpu_index"] = ids[idx] if ids and idx < len(ids) else str(idx)
    return info


@dataclass
class SDCEvent:
    detector: str                 # "checksum", "replay", "kv_transfer", "alltoall", "canary", "replica", ...
    step: Optional[int]
    detail: dict = field(default_factory=dict)
    identity: dict = field(default_factory=dict)
    time: float = field(default_factory=time.time)

    def to_json(self) -> str:
        return json.dumps(asdict(self), default=str)


class EventLog:
    """Events in memory, optionally appended to a JSONL file. A failed write is counted, never raised."""

    def __init__(self, path: Optional[str] = None):
        self.path = path
        self.events: list[SDCEvent] = []
        self.write_errors = 0

    def add(self, ev: SDCEvent) -> None:
        self.events.append(ev)
        if not self.path:
            return
        try:
            os.makedirs(os.path.dirname(os.path.abspath(self.path)) or ".", exist_ok=True)
            with open(self.path, "a") as f:
                f.write(ev.to_json() + "\n")
        except OSError as e:
            self.write_errors += 1
            if self.write_errors == 1:
                log.warning("sdcguard: cannot append alerts to %s (%s); they stay in memory", self.path, e)

    def first_step(self) -> Optional[int]:
        steps = [e.step for e in self.events if e.step is not None]
        return min(steps) if steps else None


def rollback_checkpoint(first_alert_step: int, checkpoint_steps: list[int], check_every: int = 1,
                        windows: int = 1) -> Optional[int]:
    """Newest checkpoint no later than the last check known to have passed (first_alert_step - check_every *
    windows); None when there is none."""
    cutoff = first_alert_step - check_every * max(1, windows)
    ok = [s for s in checkpoint_steps if s <= cutoff]
    return max(ok) if ok else None


# ------------------------------------------------------------------------------------------ cross-rank suspects
IDENTITY_FIELDS = ("host", "gpu_uuid", "gpu_name", "pci_bus_id", "gpu_index")


def gather_identities(group=None, device=None) -> list:
    """Collective: every rank's `device_identity`, in the group's rank order (None entries when the exchange
    fails: the ranks are still named)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    ids: list = [None] * world
    try:
        dist.all_gather_object(ids, device_identity(device), group=group)
    except Exception:  # noqa: BLE001  identities are best effort
        ids = [None] * world
    return ids


def job_rank(group, r: int) -> int:
    """Rank r of `group` as a rank of the whole job (r itself without a group, or when it cannot be mapped)."""
    if group is None:
        return r
    import torch.distributed as dist
    try:
        return int(dist.get_global_rank(group, r))
    except Exception:  # noqa: BLE001
        return r


def suspect_event(detector: str, step, suspects: list, ids: list, my_rank: int, detail: dict,
                  to_job_rank=lambda r: r) -> SDCEvent:
    """The event of a cross-rank vote (canary outputs, replica weights), built the same on every rank from the same
    suspects (ranks of the voting group) and the gathered identities `ids`. With a clear majority (fewer suspects
    than voters) it names the suspects' GPUs and, for a single suspect, takes that GPU's identity as the event's;
    one rank, the lowest-ranked rank that agreed with the majority (rank 0 without a majority), is marked
    `reporter`, so alert hooks post one message per finding instead of one per rank. Ranks in `suspect_ranks` and
    `reported_by_rank` are the job's (`to_job_rank`); `suspect_group_ranks` keeps the group's."""
    world = len(ids)
    clear = len(suspects) < world
    reporter = min((r for r in range(world) if r not in suspects), default=0) if clear else 0
    who = [dict({"rank": to_job_rank(r)}, **{k: (ids[r] or {}).get(k) for k in IDENTITY_FIELDS}) for r in suspects]
    full = {"suspect_ranks": [to_job_rank(r) for r in suspects], "suspect_group_ranks": list(suspects),
            "world": world, "suspects": who, "reported_by_rank": to_job_rank(my_rank),
            "reporter": my_rank == reporter, "clear_majority": clear}
    full.update(detail)
    mine = ids[my_rank] if 0 <= my_rank < world and ids[my_rank] else device_identity()
    identity = dict(ids[suspects[0]]) if clear and len(suspects) == 1 and ids[suspects[0]] else dict(mine)
    return SDCEvent(detector=detector, step=step, detail=full, identity=identity)

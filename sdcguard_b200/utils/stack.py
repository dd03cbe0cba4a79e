"""Identity of what a serving process runs: model configuration hash, a digest of every weight's bit
fingerprint, library and toolkit versions, the GPU, and the checks that are on. Two processes that report the same
identity serve the same arithmetic; `compare` lists what differs.

Reference: `collect` (src/sdcguard/stack.py:117), `fingerprint` (:194), `compare` (:221); published as the
`sdcguard_stack_info` metric there and here (utils.alerts.Metrics.publish_stack).
"""
from __future__ import annotations

import hashlib
import json
import platform
from dataclasses import asdict, is_dataclass


def collect(model=None, engine=None, weight_scan=None) -> dict:
    import torch
    from .. import __version__
    out = {"sdcguard_b200": __version__, "torch": torch.__version__, "cuda": torch.version.cuda,
           "python": platform.python_version()}
    if torch.cuda.is_available():
        out["gpu"] = torch.cuda.get_device_name(0)
    if model is not None and hasattr(model, "cfg"):
        cfg = asdict(model.cfg) if is_dataclass(model.cfg) else dict(vars(model.cfg))
        out["model"] = cfg.get("name")
        out["config_sha256"] = hashlib.sha256(json.dumps(cfg, sort_keys=True, default=str).encode()).hexdigest()
        out["checked"] = bool(getattr(model, "checked", False))
    if weight_scan is not None:
        out["weights_digest"] = weight_scan.digest()
    if engine is not None:
        out["sample_every"] = getattr(engine, "sample_every", None)
        out["cuda_graph"] = getattr(engine, "cuda_graph", None)
    return out


def fingerprint(stack: dict) -> str:
    return hashlib.sha256(json.dumps(stack, sort_keys=True, default=str).encode()).hexdigest()[:16]


def compare(a: dict, b: dict) -> dict:
    keys = sorted(set(a) | set(b))
    return {k: {"a": a.get(k), "b": b.get(k)} for k in keys if a.get(k) != b.get(k)}

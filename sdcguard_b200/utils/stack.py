"""Identity of what a serving (or training) process runs: the model and its configuration, the weights' digest, the
precision and KV-cache layout, parallel sizes, the execution mode (CUDA graphs, programmatic launch), which kernels
run attention, MoE and the GEMMs and with which steering settings, which checks are on and how, the native library
build, and the toolkit, driver and GPU. Two processes that report the same identity serve the same arithmetic.

    s = collect(model, engine, weight_scan)          # a dict of strings plus its "fingerprint"
    compare(qualified, s)                            # {"same": True / False / None, "differences", "why"}

`compare` says None (unknown, never "same") when a field that ties the stack to its arithmetic is recorded on one
side only, or when neither side records the weights' digest: nothing then shows these are the weights qualified.
Per-worker fields (device, pid) are left out of what the workers of one server must agree on (`shared`). The stack
is published as the labels of the `sdcguard_stack_info` metric, which `from_metrics` reads back.

Reference: `collect` (src/sdcguard/stack.py:117), `fingerprint` (:194), `shared` (:200), `from_metrics` (:212),
`compare` (:221); the fields here describe this engine instead of vLLM's.
"""
from __future__ import annotations

import hashlib
import json
import os
import platform
import re
from dataclasses import asdict, is_dataclass
from typing import Optional

# fields that change the arithmetic or tie the stack to it: recorded on one side only means "unknown"
IDENTITY = ("model_config", "weights_digest", "precision", "library_build", "gpu")
PER_WORKER = ("device", "pid", "gpu_uuid")
STEERING_PREFIXES = ("SDCGUARD_GEMM", "SDCGUARD_PDL", "SDCGUARD_PREFILL", "SDCGUARD_SHARE", "SDCGUARD_OFFSET",
                     "SDCGUARD_NORMS", "SDCGUARD_ROPE", "SDCGUARD_ATTN", "SDCGUARD_ACT", "SDCGUARD_SPOT", "SDCGUARD_Z",
                     "SDCGUARD_SIGN_SEED", "NVIDIA_TF32_OVERRIDE", "CUBLAS", "CUBLASLT_", "TORCH_BLAS_")
NOT_STEERING = ("CUBLASLT_LOG_LEVEL", "CUBLASLT_LOG_FILE", "CUBLASLT_LOG_MASK")
_WHAT = {"model_config": "the model configuration's hash", "weights_digest": "the weights' digest",
         "precision": "the compute precision", "library_build": "the native library's build hash", "gpu": "the GPU"}


def _s(v) -> Optional[str]:
    if v is None:
        return None
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, (list, tuple)):
        return ",".join(str(x) for x in v) or None
    return str(v)


def steering_env(env=None) -> Optional[str]:
    env = os.environ if env is None else env
    kv = sorted((k, v) for k, v in env.items() if k.startswith(STEERING_PREFIXES) and k not in NOT_STEERING)
    return ",".join(f"{k}={v}" for k, v in kv) or None


def library_build() -> Optional[str]:
    """SHA-256 (first 16) of the loaded native library file: the kernels' exact build."""
    try:
        from .. import _native
        with open(_native.LIB_PATH, "rb") as f:
            return hashlib.sha256(f.read()).hexdigest()[:16]
    except OSError:
        return None


def _model_fields(model) -> dict:
    out: dict = {}
    cfg = getattr(model, "cfg", None)
    if cfg is not None:
        d = asdict(cfg) if is_dataclass(cfg) else dict(vars(cfg))
        out["model"] = d.get("name")
        out["model_config"] = hashlib.sha256(json.dumps(d, sort_keys=True, default=str).encode()).hexdigest()[:16]
    out["precision"] = getattr(model, "precision", None)
    out["checked"] = getattr(model, "checked", None)
    st = getattr(model, "settings", None)
    if st is not None and hasattr(st, "describe"):
        d = st.describe()
        out["checks"] = ",".join(f"{k}={d[k]}" for k in sorted(d) if k != "notes")
    out["tensor_parallel"] = getattr(model, "tp_size", None)
    moe = getattr(model, "moe", None)
    if moe:
        out["moe"] = f"grouped checked GEMM, {moe[0].collective}" if getattr(moe[0], "checked", False) else \
            f"PyTorch grouped GEMM, {moe[0].collective}"
        out["expert_parallel"] = getattr(moe[0], "world", None)
    return out


def _engine_fields(engine) -> dict:
    return {"cuda_graph": getattr(engine, "cuda_graph", None), "kv_page_tokens": getattr(engine, "page", None) or 16,
            "kv_cache_dtype": str(getattr(getattr(engine, "cache", None), "dtype", "")).replace("torch.", "") or None,
            "max_model_len": getattr(engine, "max_model_len", None),
            "sample_every": getattr(engine, "sample_every", None)}


def collect(model=None, engine=None, weight_scan=None, extra: Optional[dict] = None) -> dict:
    """The stack of this process (any argument may be None; fields that cannot be read are left out)."""
    import torch
    from .. import __version__
    out: dict = {"sdcguard_b200": __version__, "torch": torch.__version__, "cuda": torch.version.cuda,
                 "python": platform.python_version(), "library_build": library_build(), "env": steering_env(),
                 "pid": os.getpid(),
                 "attention": "tcgen05 paged prefill (ping-pong)" if os.environ.get("SDCGUARD_PREFILL_PINGPONG", "1")
                 != "0" else "tcgen05 paged prefill (one tile per CTA)",
                 "gemm": "checked tcgen05 GEMM, CTA pairs " + ("off" if os.environ.get("SDCGUARD_GEMM_PAIR") == "0"
                                                                 else "on"),
                 "pdl": "off" if os.environ.get("SDCGUARD_PDL") == "0" else "on"}
    if torch.cuda.is_available():
        idx = torch.cuda.current_device()
        p = torch.cuda.get_device_properties(idx)
        out.update(gpu=p.name, compute_capability=f"{p.major}.{p.minor}", device=f"cuda:{idx}",
                   sms=p.multi_processor_count)
        try:
            from .events import device_identity
            out["gpu_uuid"] = device_identity(torch.device("cuda", idx)).get("gpu_uuid")
        except Exception:  # noqa: BLE001  (best effort)
            pass
    if model is not None:
        out.update(_model_fields(model))
    if engine is not None:
        out.update(_engine_fields(engine))
    if weight_scan is not None:
        try:
            out["weights_digest"] = weight_scan.digest()
        except Exception:  # noqa: BLE001  (a digest that cannot be taken is left out)
            pass
    if extra:
        out.update(extra)
    clean = {k: _s(v) for k, v in out.items() if _s(v) not in (None, "")}
    clean["fingerprint"] = fingerprint(clean)
    return clean


def fingerprint(stack: dict) -> str:
    """Hash of every field but the per-worker ones (and the fingerprint itself)."""
    body = {k: v for k, v in stack.items() if k not in PER_WORKER and k != "fingerprint"}
    return hashlib.sha256(json.dumps(body, sort_keys=True, default=str).encode()).hexdigest()[:16]


def shared(stack: Optional[dict]) -> Optional[str]:
    """What every worker of one server must agree on: the stack without its per-worker fields."""
    if not stack:
        return None
    return json.dumps({k: v for k, v in stack.items() if k not in PER_WORKER and k != "fingerprint"},
                      sort_keys=True, default=str)


_INFO = re.compile(r'^sdcguard_stack_info\{(.*)\}\s+\S+\s*$')
_LABEL = re.compile(r'(\w+)="((?:[^"\\]|\\.)*)"')


def from_metrics(text: str) -> Optional[dict]:
    """The labels of the sdcguard_stack_info line of a metrics page, or None."""
    for line in (text or "").splitlines():
        m = _INFO.match(line.strip())
        if m:
            return {k: v.replace('\\"', '"').replace("\\\\", "\\") for k, v in _LABEL.findall(m.group(1))}
    return None


def compare(qualified: Optional[dict], live: Optional[dict]) -> dict:
    """Is `live` the stack that was qualified? same True (every field and the fingerprint agree), False (a field
    differs: listed), or None (unknown: an identity field recorded on one side only, or no weights digest on
    either side)."""
    if not qualified or not live:
        return {"same": None, "differences": [], "why": "no stack recorded" if not qualified else
                "the process publishes no stack"}
    keys = sorted((set(qualified) | set(live)) - set(PER_WORKER) - {"fingerprint"})
    one_sided = [k for k in IDENTITY if (qualified.get(k) is None) != (live.get(k) is None)]
    diffs = [f"{k}: {qualified.get(k)!r} qualified, {live.get(k)!r} now" for k in keys
             if k not in one_sided and qualified.get(k) is not None and live.get(k) is not None
             and qualified.get(k) != live.get(k)]
    diffs += [f"{k}: only {'qualified' if qualified.get(k) is not None else 'now'} records it" for k in keys
              if k not in IDENTITY and (qualified.get(k) is None) != (live.get(k) is None)]
    if diffs:
        return {"same": False, "differences": diffs, "why": "not the stack qualified: " + "; ".join(diffs)}
    unknown = [f"only one side records {_WHAT[k]}" for k in one_sided]
    if qualified.get("weights_digest") is None and live.get("weights_digest") is None:
        unknown.append("neither side records the weights' digest: nothing shows these are the weights qualified")
    if unknown:
        return {"same": None, "differences": [], "unknown": unknown,
                "why": "cannot be shown to be the stack qualified: " + "; ".join(unknown)}
    return {"same": True, "differences": [], "why": f"the stack qualified (fingerprint {fingerprint(live)})"}


def field_differences(a: dict, b: dict) -> dict:
    """Every field that differs, per-worker ones included: {field: {"a": ..., "b": ...}}."""
    return {k: {"a": a.get(k), "b": b.get(k)} for k in sorted(set(a) | set(b)) if a.get(k) != b.get(k)}

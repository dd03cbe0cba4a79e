"""Catalog of the evidence rules the offline tools emit: what each rule id states, in which section, with which
verdicts, and a shape check for findings. The catalog carries metadata only; the evaluators (config, inventory,
assessment, overhead, lifetime reports) remain the sole source of verdicts, and a well-shaped finding is not a proof
of anything.

    from sdcguard_b200.evidence import catalog
    catalog.describe("protection.kv_checksum")     # {"section", "statement", "verdicts"}
    catalog.validate_finding(finding)                # [] when the finding has the catalog's shape

Finding shape: {"id": rule id, "verdict": one of the rule's verdicts, "message": str, "basis": str, "facts": dict,
"sources": list of str}.

Reference: src/sdcguard/evidence_catalog.py:1-10 (immutable metadata, shape validation only; `catalog`, `describe`,
`validate_finding`).
"""
from __future__ import annotations

import hashlib
import json

VERDICTS = ("satisfied", "violated", "unknown", "not_applicable")

_R = {
    # static deployment contracts (evidence/config.py)
    "capacity.planned": ("config", "The declared KV page pool holds the advertised context for the declared batch "
                                   "and fits the declared device memory."),
    "capacity.startup": ("config", "The engine's saved startup line reports at least the declared KV pages."),
    "protection.gemm_abft": ("config", "Every linear layer runs on the checked GEMM (ABFT in the epilogue)."),
    "protection.replay": ("config", "Norm, attention and elementwise kernels replay a row sample of at most 1/64."),
    "protection.kv_checksum": ("config", "KV pages moved between prefill and decode are hashed on arrival and "
                                         "compared with the producer's checksums."),
    "protection.deferred_release": ("config", "A producer frees a request's pages only after its consumer answered."),
    "protection.cached_prefix": ("config", "Cached prefix pages reused by a decode worker are re-verified."),
    "deployment.peer_profile": ("config", "Every worker declares the same engine version, build and model."),
    "deployment.page_tokens_agreement": ("config", "Every worker declares the same tokens per KV page."),
    # recordings (evidence/assessment.py, evidence/inventory.py)
    "recording.coverage": ("assessment", "Every request's transferred KV was compared in full."),
    "recording.lifetime": ("assessment", "The recorded page-lifetime events break no ledger rule."),
    "recording.readiness": ("assessment", "The serving endpoint reported PROTECTED when asked."),
    "inventory.complete": ("inventory", "Each declared client request has exactly one recorded transfer."),
    # measurements (evidence/overhead.py)
    "overhead.identity": ("overhead", "Checked and unchecked runs share one configuration, GPU and build."),
    "overhead.bound": ("overhead", "The measured overhead of the checks is within the declared bound."),
    # recorded engine internals (evidence/assignment.py, evidence/forward.py)
    "assignment.exclusive": ("assignment", "No KV page was assigned to two live requests at once."),
    "forward.owned_pages": ("forward", "Every page a forward step read for a request was that request's page, "
                                       "or a prefix page shared with it."),
    "model.reference": ("model", "The model files hash to the bound reference."),
}


def catalog() -> dict:
    return {k: {"section": s, "statement": t, "verdicts": list(VERDICTS)} for k, (s, t) in sorted(_R.items())}


def catalog_hash() -> str:
    return hashlib.sha256(json.dumps(catalog(), sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def describe(rule_id: str) -> dict:
    if rule_id not in _R:
        raise KeyError(f"unknown rule {rule_id!r}")
    return catalog()[rule_id]


def finding(rule_id: str, verdict: str, message: str, basis: str, facts: dict | None = None,
            sources: list | None = None) -> dict:
    f = {"id": rule_id, "verdict": verdict, "message": message, "basis": basis, "facts": facts or {},
         "sources": list(sources or [])}
    bad = validate_finding(f)
    if bad:
        raise ValueError("; ".join(bad))
    return f


def validate_finding(f) -> list[str]:
    """Problems with a finding's shape (empty when it has the catalog's shape)."""
    if not isinstance(f, dict):
        return ["finding is not an object"]
    out = []
    if f.get("id") not in _R:
        out.append(f"unknown rule id {f.get('id')!r}")
    if f.get("verdict") not in VERDICTS:
        out.append(f"verdict {f.get('verdict')!r} is not one of {VERDICTS}")
    for k, t in (("message", str), ("basis", str), ("facts", dict), ("sources", list)):
        if not isinstance(f.get(k), t):
            out.append(f"{k} must be a {t.__name__}")
    extra = set(f) - {"id", "verdict", "message", "basis", "facts", "sources"}
    if extra:
        out.append(f"unexpected keys {sorted(extra)}")
    return out

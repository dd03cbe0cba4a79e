"""Static deployment contracts of a prefill/decode deployment of this engine, judged from the operator's declared
configuration and the engines' saved startup lines. Nothing is imported from a running engine, no server is contacted
and no device work is done.

    python -m sdcguard_b200.evidence.config DEPLOYMENT.json [--json] [--html OUT.html]
    sdcguard config-safety DEPLOYMENT.json

DEPLOYMENT.json ("sdcguard_b200.deployment.v1"):
    {"model": {"name", "layers", "kv_heads", "head_dim"}, "advertised_context_tokens": int,
     "workers": [{"id", "role": "prefill" | "decode" | "both", "version", "build", "gpu_memory_gb",
                  "kv_pages", "page_tokens", "max_num_seqs", "checked", "sample_every", "kv_checksums",
                  "release": "after_consumer_done" | "early", "verify_cached_prefix", "startup_log": path}]}

Each worker gets the capacity and protection rules, the deployment the peer rules (`evidence.catalog` states each).
A rule is "unknown" whenever its facts are missing or malformed: an absent fact is never read as a good one. The
startup log is the line `LLMEngine.startup_line()` prints (`sdcguard_b200 engine: kv_pages=... page_tokens=...`);
the declared geometry is the operator's statement, not an attestation of what ran.

Reference: src/sdcguard/config_safety.py:1-20 (`assess`, `render`), config_capacity.py:1-10 (planned and startup
capacity), config_inputs.py:1-10 (bounded read-only inputs, binding digest, `read_startup`), config_protections.py:1-10
(safeguard inventory).
"""
from __future__ import annotations

import argparse
import hashlib
import html
import json
import os
import re
import sys
from typing import Optional

from . import catalog

SCHEMA = "sdcguard_b200.deployment.v1"
RULE_SET = "sdcguard_b200.static-pd-contracts.v1"
SCOPE = ("declared configuration and saved startup lines only; a satisfied rule covers its named contract, not "
         "request isolation, build authenticity or the engines' current state")
MAX_BYTES = 1 << 20
MAX_WORKERS = 256
KV_MEMORY_FRACTION = 0.9          # of device memory that the KV pool may take in a plan (weights, activations: rest)
STARTUP = re.compile(r"sdcguard_b200 engine: (.*)$", re.M)


def _sha(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _read_bounded(path: str, limit: int = MAX_BYTES) -> bytes:
    with open(path, "rb") as f:
        raw = f.read(limit + 1)
    if len(raw) > limit:
        raise ValueError(f"{path}: larger than {limit} bytes")
    return raw


def load_deployment(path: str) -> tuple[dict, dict]:
    """(document, provenance): the parsed declaration and the digests that bind it (file bytes, canonical form)."""
    raw = _read_bounded(path)
    doc = json.loads(raw)
    if not isinstance(doc, dict) or doc.get("schema") != SCHEMA:
        raise ValueError(f"{path}: not a {SCHEMA} document")
    ws = doc.get("workers")
    if not isinstance(ws, list) or not ws or len(ws) > MAX_WORKERS:
        raise ValueError(f"{path}: workers must be a non-empty list of at most {MAX_WORKERS}")
    ids = [w.get("id") for w in ws if isinstance(w, dict)]
    if len(ids) != len(ws) or len(set(ids)) != len(ids) or not all(isinstance(i, str) and i for i in ids):
        raise ValueError(f"{path}: every worker needs a unique string id")
    return doc, {"file_sha256": hashlib.sha256(raw).hexdigest(), "binding": _sha(doc),
                 "base": os.path.dirname(os.path.abspath(path))}


def read_startup(worker: dict, base: str) -> dict:
    """The facts of the worker's saved startup line, or {"error": why}."""
    p = worker.get("startup_log")
    if not isinstance(p, str) or not p:
        return {"error": "no startup log declared"}
    path = p if os.path.isabs(p) else os.path.join(base, p)
    try:
        text = _read_bounded(path).decode("utf-8", "replace")
    except (OSError, ValueError) as e:
        return {"error": f"startup log unreadable: {e}"}
    lines = STARTUP.findall(text)
    if len(lines) != 1:
        return {"error": f"startup log holds {len(lines)} engine lines (want exactly 1)"}
    facts = {}
    for kv in lines[0].split():
        if "=" in kv:
            k, v = kv.split("=", 1)
            facts[k] = v
    return {"facts": facts, "sha256": hashlib.sha256(text.encode()).hexdigest()}


def _int(v) -> Optional[int]:
    return v if type(v) is int and v >= 0 else None


def _f(rule, verdict, message, basis, facts=None) -> dict:
    return catalog.finding(rule, verdict, message, basis, facts or {})


def kv_page_bytes(model: dict, page_tokens: int) -> Optional[int]:
    vals = [_int(model.get(k)) for k in ("layers", "kv_heads", "head_dim")]
    if None in vals or not page_tokens:
        return None
    layers, kvh, hd = vals
    return layers * 2 * kvh * page_tokens * hd * 2          # K and V, bf16


def capacity(worker: dict, model: dict, context: Optional[int], startup: dict) -> list[dict]:
    out = []
    pages, pt, seqs = _int(worker.get("kv_pages")), _int(worker.get("page_tokens")), _int(worker.get("max_num_seqs"))
    mem = worker.get("gpu_memory_gb")
    pb = kv_page_bytes(model, pt or 0)
    if None in (pages, pt, seqs, pb, _int(context)) or not isinstance(mem, (int, float)) or mem <= 0:
        out.append(_f("capacity.planned", "unknown", "Pages, page size, batch, context, memory or model geometry "
                      "is missing or malformed.", "missing evidence"))
    else:
        need = seqs * -(-context // pt) + 1                  # page 0 is the engine's reserved zero page
        pool = pages * pb
        budget = mem * 1e9 * KV_MEMORY_FRACTION
        ok = pages >= need and pool <= budget
        out.append(_f("capacity.planned", "satisfied" if ok else "violated",
                      "The pool holds the advertised context for the declared batch and fits memory." if ok else
                      ("The pool is smaller than the advertised context for the declared batch." if pages < need else
                       "The pool does not fit the declared device memory."),
                      "declared geometry", {"pages": pages, "pages_needed": need, "pool_bytes": pool,
                                            "budget_bytes": int(budget)}))
    if "error" in startup:
        out.append(_f("capacity.startup", "unknown", startup["error"], "startup evidence unavailable"))
    else:
        got = startup["facts"]
        try:
            sp, spt = int(got.get("kv_pages", "")), int(got.get("page_tokens", ""))
        except ValueError:
            out.append(_f("capacity.startup", "unknown", "The startup line has no integer kv_pages/page_tokens.",
                          "malformed startup evidence"))
        else:
            ok = pages is not None and sp >= pages and spt == pt
            out.append(_f("capacity.startup", "satisfied" if ok else "violated",
                          "The saved startup line reports the declared pool." if ok else
                          "The saved startup line reports fewer pages or another page size than declared.",
                          "saved startup line", {"startup_kv_pages": sp, "startup_page_tokens": spt,
                                                 "declared_kv_pages": pages, "log_sha256": startup["sha256"]}))
    return out


def protections(worker: dict) -> list[dict]:
    out = []
    role = worker.get("role")
    pd_role = role in ("prefill", "decode")

    def boolean(rule, key, good_msg, bad_msg, applies=True, want=True):
        v = worker.get(key)
        if not applies:
            out.append(_f(rule, "not_applicable", "The worker moves no KV between roles.", "declared role"))
        elif type(v) is not bool:
            out.append(_f(rule, "unknown", f"{key} is not declared as a boolean.", "missing evidence"))
        else:
            out.append(_f(rule, "satisfied" if v == want else "violated", good_msg if v == want else bad_msg,
                          "declared configuration", {key: v}))

    boolean("protection.gemm_abft", "checked", "Linear layers run on the checked GEMM.",
            "The engine runs unchecked (checked=false).")
    se = _int(worker.get("sample_every"))
    if se is None or se == 0:
        out.append(_f("protection.replay", "unknown", "sample_every is not a positive integer.", "missing evidence"))
    else:
        ok = se <= 64 and worker.get("checked") is True
        out.append(_f("protection.replay", "satisfied" if ok else "violated",
                      "Replay checks sample at least one row in 64." if ok else
                      "Replay checks are off or sample fewer than one row in 64.", "declared configuration",
                      {"sample_every": se}))
    boolean("protection.kv_checksum", "kv_checksums", "Transferred KV pages are hashed and compared.",
            "KV pages move unverified.", applies=pd_role)
    rel = worker.get("release")
    if role != "prefill":
        out.append(_f("protection.deferred_release", "not_applicable", "Only prefill workers release sent pages.",
                      "declared role"))
    elif rel not in ("after_consumer_done", "early"):
        out.append(_f("protection.deferred_release", "unknown", "release is not declared.", "missing evidence"))
    else:
        ok = rel == "after_consumer_done"
        out.append(_f("protection.deferred_release", "satisfied" if ok else "violated",
                      "Pages are freed after the consumer's answer." if ok else
                      "Pages may be freed while the consumer still reads them (stale reads).",
                      "declared configuration", {"release": rel}))
    boolean("protection.cached_prefix", "verify_cached_prefix", "Cached prefix pages are re-verified on reuse.",
            "Cached prefix pages are reused without re-verification.", applies=role in ("decode", "both"))
    return out


def peers(workers: list) -> list[dict]:
    ident = {(w.get("version"), w.get("build")) for w in workers}
    missing = [w["id"] for w in workers if not w.get("version") or not w.get("build")]
    if missing:
        prof = _f("deployment.peer_profile", "unknown", "Workers without version or build: " + ", ".join(missing),
                  "missing evidence")
    else:
        one = len(ident) == 1
        prof = _f("deployment.peer_profile", "satisfied" if one else "violated",
                  "Every worker declares the same version and build." if one else
                  "Workers declare different versions or builds.", "declared peer profile",
                  {"profiles": sorted(str(i) for i in ident)})
    pts = [w.get("page_tokens") for w in workers]
    if any(_int(p) is None for p in pts):
        pt = _f("deployment.page_tokens_agreement", "unknown", "A worker declares no page size.", "missing evidence")
    else:
        pt = _f("deployment.page_tokens_agreement", "satisfied" if len(set(pts)) == 1 else "violated",
                "Every worker uses the same page size." if len(set(pts)) == 1 else
                "Page sizes differ: pulled pages would be misread.", "declared configuration", {"page_tokens": pts})
    return [prof, pt]


def assess(document: dict, provenance: dict) -> dict:
    model = document.get("model") if isinstance(document.get("model"), dict) else {}
    ctx = document.get("advertised_context_tokens")
    workers = []
    for w in document["workers"]:
        rules = capacity(w, model, ctx, read_startup(w, provenance.get("base", ".")))
        rules += protections(w)
        workers.append({"id": w["id"], "role": w.get("role"), "rules": rules})
    dep = peers(document["workers"])
    allr = [r for w in workers for r in w["rules"]] + dep
    if any(r["verdict"] == "violated" for r in allr):
        verdict = "FAIL"
    elif all(r["verdict"] in ("satisfied", "not_applicable") for r in allr):
        verdict = "PASS"
    else:
        verdict = "HOLD"
    return {"schema": "sdcguard_b200.config-assessment.v1", "rule_set": RULE_SET, "scope": SCOPE,
            "catalog_sha256": catalog.catalog_hash(), "provenance": {k: v for k, v in provenance.items() if k != "base"},
            "workers": workers, "deployment": dep, "verdict": verdict}


def render(a: dict) -> str:
    lines = [f"deployment contracts: {a['verdict']}", f"scope: {a['scope']}"]
    for w in a["workers"]:
        lines.append(f"worker {w['id']} ({w['role']}):")
        lines += [f"  {r['verdict']:<15} {r['id']}: {r['message']}" for r in w["rules"]]
    lines.append("deployment:")
    lines += [f"  {r['verdict']:<15} {r['id']}: {r['message']}" for r in a["deployment"]]
    return "\n".join(lines)


def render_html(a: dict) -> str:
    rows = []
    for w in a["workers"]:
        for r in w["rules"]:
            rows.append((w["id"], r))
    rows += [("deployment", r) for r in a["deployment"]]
    body = "".join(f"<tr><td>{html.escape(str(w))}</td><td>{html.escape(r['id'])}</td><td>{html.escape(r['verdict'])}"
                   f"</td><td>{html.escape(r['message'])}</td></tr>" for w, r in rows)
    return (f"<html><body><h1>Deployment contracts: {html.escape(a['verdict'])}</h1><p>{html.escape(a['scope'])}</p>"
            f"<table border=1><tr><th>worker</th><th>rule</th><th>verdict</th><th>message</th></tr>{body}</table>"
            f"</body></html>")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard config-safety", description="static deployment contracts")
    ap.add_argument("deployment")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--html")
    a = ap.parse_args(argv)
    try:
        doc, prov = load_deployment(a.deployment)
    except (OSError, ValueError) as e:
        print(f"config-safety: {e}", file=sys.stderr)
        return 2
    res = assess(doc, prov)
    if a.html:
        with open(a.html, "w") as f:
            f.write(render_html(res))
    print(json.dumps(res, indent=1) if a.json else render(res))
    return {"PASS": 0, "HOLD": 1, "FAIL": 3}[res["verdict"]]


if __name__ == "__main__":
    raise SystemExit(main())

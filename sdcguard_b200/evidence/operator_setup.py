"""Setup files for an operator and an offline preflight of the inputs they supplied.

    python -m sdcguard_b200.evidence.operator_setup export OUT_DIR          # templates + checksums
    python -m sdcguard_b200.evidence.operator_setup preflight DEPLOYMENT.json [--model-ref REF.json --model-dir DIR]
    python -m sdcguard_b200.evidence.operator_setup verify OUT_DIR            # the exported files are unchanged
    sdcguard operator-setup ...

export writes a deployment template (`deployment.template.json`, the `evidence.config` schema with one prefill and one
decode worker at this package's defaults), a client-inventory template, the recording environment, and
`SETUP_MANIFEST.json` with the SHA-256 of each file and of this package's sources. preflight checks what the operator
filled in, without starting anything: the deployment parses and binds, its startup logs are readable and name this
engine, the static contracts do not fail, and, when given, the model directory still matches its reference.

Reference: src/sdcguard/operator_setup.py:1-10 (`export_setup`, `preflight`, `verify_output`, `render`).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os

from . import config, inventory, overhead

TEMPLATE = {
    "schema": config.SCHEMA,
    "model": {"name": "Qwen3-0.6B", "layers": 28, "kv_heads": 8, "head_dim": 128},
    "advertised_context_tokens": 4096,
    "workers": [
        {"id": "prefill0", "role": "prefill", "version": "", "build": "", "gpu_memory_gb": 180, "kv_pages": 66000,
         "page_tokens": 16, "max_num_seqs": 256, "checked": True, "sample_every": 64, "kv_checksums": True,
         "release": "after_consumer_done", "startup_log": "prefill0.log"},
        {"id": "decode0", "role": "decode", "version": "", "build": "", "gpu_memory_gb": 180, "kv_pages": 66000,
         "page_tokens": 16, "max_num_seqs": 256, "checked": True, "sample_every": 64, "kv_checksums": True,
         "verify_cached_prefix": True, "startup_log": "decode0.log"},
    ],
}


def _sha_file(p: str) -> str:
    with open(p, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def export_setup(out: str) -> dict:
    from .. import __version__
    os.makedirs(out, exist_ok=True)
    t = json.loads(json.dumps(TEMPLATE))
    for w in t["workers"]:
        w["version"] = __version__
    files = {
        "deployment.template.json": t,
        "client_inventory.template.json": {"schema": inventory.SCHEMA, "workload": "declared-batch", "requests": []},
        "recording.env.json": {"SDCGUARD_SIGN_SEED": "1", "MASTER_ADDR": "127.0.0.1"},
    }
    man = {"schema": "sdcguard_b200.setup-manifest.v1", "package_version": __version__,
           "package_sha256": overhead.package_digest(), "files": {}}
    for name, doc in files.items():
        p = os.path.join(out, name)
        with open(p, "w") as f:
            json.dump(doc, f, indent=1, sort_keys=True)
        man["files"][name] = _sha_file(p)
    with open(os.path.join(out, "SETUP_MANIFEST.json"), "w") as f:
        json.dump(man, f, indent=1, sort_keys=True)
    return man


def verify_output(out: str) -> list[str]:
    try:
        with open(os.path.join(out, "SETUP_MANIFEST.json")) as f:
            man = json.load(f)
    except (OSError, ValueError) as e:
        return [f"manifest unreadable: {e}"]
    bad = []
    for name, sha in man.get("files", {}).items():
        p = os.path.join(out, name)
        if not os.path.isfile(p):
            bad.append(f"{name}: missing")
        elif _sha_file(p) != sha:
            bad.append(f"{name}: changed since export")
    if man.get("package_sha256") != overhead.package_digest():
        bad.append("exported by another version of this package")
    return bad


def preflight(deployment: str, model_ref: str | None = None, model_dir: str | None = None) -> dict:
    checks = []
    try:
        doc, prov = config.load_deployment(deployment)
        checks.append(("deployment parses and binds", True, prov["binding"][:16]))
    except (OSError, ValueError) as e:
        return {"ok": False, "checks": [("deployment parses and binds", False, str(e))]}
    for w in doc["workers"]:
        st = config.read_startup(w, prov["base"])
        checks.append((f"startup log of {w['id']}", "error" not in st, st.get("error", "one engine line")))
    a = config.assess(doc, prov)
    checks.append(("static contracts do not fail", a["verdict"] != "FAIL", a["verdict"]))
    if model_ref and model_dir:
        from . import model_reference
        with open(model_ref) as f:
            r = model_reference.observe(json.load(f), model_dir)
        checks.append(("model files match their reference", r["match"], r["findings"][0]["message"]))
    return {"ok": all(c[1] for c in checks), "checks": checks}


def render(r: dict) -> str:
    return "\n".join([f"{'ok  ' if c[1] else 'FAIL'} {c[0]}: {c[2]}" for c in r["checks"]]
                     + ["preflight " + ("passed" if r["ok"] else "failed")])


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard operator-setup")
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("export")
    e.add_argument("out")
    p = sub.add_parser("preflight")
    p.add_argument("deployment")
    p.add_argument("--model-ref")
    p.add_argument("--model-dir")
    v = sub.add_parser("verify")
    v.add_argument("out")
    a = ap.parse_args(argv)
    if a.cmd == "export":
        m = export_setup(a.out)
        print(f"exported {len(m['files'])} files to {a.out}")
        return 0
    if a.cmd == "verify":
        bad = verify_output(a.out)
        print("setup files verified" if not bad else "\n".join("FAIL " + b for b in bad))
        return 0 if not bad else 1
    r = preflight(a.deployment, a.model_ref, a.model_dir)
    print(render(r))
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())

"""Signed GPU correctness certificates from a screen report (Ed25519).

    python -m sdcguard_b200.tools.certify keygen --out fleet              # fleet.key (secret), fleet.pub (share)
    python -m sdcguard_b200.tools.certify sign screen_out/screen.json --key fleet.key [--ops screen_ops.json]
    python -m sdcguard_b200.tools.certify verify screen_out/certificate.json --pubkey fleet.pub

A certificate records which GPU was tested (name, UUID, serial, PCI slot, VBIOS, driver from the screen's telemetry),
the workload (screen size, seed, tokens, checks, versions), the verdict (PASS only when every round of the workload
screen and every operator test passed), the SHA-256 of every evidence file, when it was issued and until when it is
meant to be valid. The canonical form (sorted-key compact JSON without the signature) is signed with Ed25519. A valid
signature shows the certificate is unchanged since the key's holder issued it; whom to trust is the reader's choice.
`verify` also re-hashes the evidence files next to the certificate and checks the validity window.

Reference: src/sdcguard/certify.py:1-20 (fields, trust statement, keygen :51, make :151, verify :249).
"""
from __future__ import annotations

import argparse
import base64
import datetime as dt
import hashlib
import json
import os
from typing import Optional

FORMAT = "sdcguard-b200-certificate/1"


def _crypto():
    from cryptography.hazmat.primitives import serialization
    from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PrivateKey, Ed25519PublicKey
    return serialization, Ed25519PrivateKey, Ed25519PublicKey


def key_id(pub) -> str:
    ser, _, _ = _crypto()
    raw = pub.public_bytes(ser.Encoding.Raw, ser.PublicFormat.Raw)
    return hashlib.sha256(raw).hexdigest()[:16]


def keygen(prefix: str) -> tuple[str, str]:
    ser, Priv, _ = _crypto()
    k = Priv.generate()
    priv = k.private_bytes(ser.Encoding.PEM, ser.PrivateFormat.PKCS8, ser.NoEncryption())
    pub = k.public_key().public_bytes(ser.Encoding.PEM, ser.PublicFormat.SubjectPublicKeyInfo)
    kp, pp = prefix + ".key", prefix + ".pub"
    fd = os.open(kp, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
    with os.fdopen(fd, "wb") as f:
        f.write(priv)
    with open(pp, "wb") as f:
        f.write(pub)
    return kp, pp


def canonical(cert: dict) -> bytes:
    body = {k: v for k, v in cert.items() if k != "signature"}
    return json.dumps(body, sort_keys=True, separators=(",", ":"), default=str).encode()


def _sha256(path: str) -> Optional[str]:
    try:
        h = hashlib.sha256()
        with open(path, "rb") as f:
            for chunk in iter(lambda: f.read(1 << 20), b""):
                h.update(chunk)
        return h.hexdigest()
    except OSError:
        return None


def make(screen: dict, ops: Optional[dict] = None, issuer: str = "", valid_days: float = 30.0,
         now: Optional[dt.datetime] = None, base_dir: str = ".") -> dict:
    now = now or dt.datetime.now(dt.timezone.utc)
    tel = screen.get("telemetry_before") or {}
    evidence = {}
    for r in screen.get("rounds", []):
        p = r.get("evidence")
        if p:
            evidence[os.path.basename(p)] = _sha256(p if os.path.isabs(p) else os.path.join(base_dir, p)) or \
                _sha256(p)
    ops_ok = ops is None or ops.get("verdict") == "pass"
    verdict = "PASS" if screen.get("verdict") == "PASS" and ops_ok else "FAIL"
    import torch
    return {"format": FORMAT, "issuer": issuer, "issued": now.isoformat(),
            "valid_until": (now + dt.timedelta(days=valid_days)).isoformat(),
            "gpu": {"name": screen.get("gpu") or tel.get("name"), "uuid": tel.get("uuid"), "serial": tel.get("serial"),
                    "pci": tel.get("pci.bus_id"), "vbios": tel.get("vbios_version"),
                    "driver": tel.get("driver_version"), "ecc_mode": tel.get("ecc.mode.current")},
            "workload": {"screen_size": screen.get("size"), "seed": screen.get("seed"), "tokens": screen.get("tokens"),
                         "checks": screen.get("checks"), "rounds": len(screen.get("rounds", [])),
                         "operator_tests": sorted((ops or {}).get("tests", {})), "torch": torch.__version__,
                         "sdcguard_b200": _version()},
            "result": {"verdict": verdict, "screen": screen.get("verdict"),
                       "operator_screen": None if ops is None else ops.get("verdict"),
                       "failed_rounds": screen.get("failed_rounds", []),
                       "failed_operator_tests": sorted(k for k, v in (ops or {}).get("tests", {}).items()
                                                       if v.get("verdict") != "pass"),
                       "worst_clean_z": screen.get("worst_clean_z")},
            "evidence_sha256": evidence}


def _version() -> str:
    try:
        from importlib.metadata import version
        return version("sdcguard_b200")
    except Exception:  # noqa: BLE001  (in-tree, not installed)
        return "in-tree"


def sign(cert: dict, key_path: str) -> dict:
    ser, _, _ = _crypto()
    with open(key_path, "rb") as f:
        key = ser.load_pem_private_key(f.read(), password=None)
    cert = dict(cert)
    cert["key_id"] = key_id(key.public_key())
    cert["signature"] = base64.b64encode(key.sign(canonical(cert))).decode()
    return cert


def verify(path: str, pubkey_path: Optional[str] = None, now: Optional[dt.datetime] = None) -> dict:
    """{valid, problems}: signature (when a public key is given), format, validity window, evidence hashes."""
    with open(path) as f:
        cert = json.load(f)
    problems = []
    if cert.get("format") != FORMAT:
        problems.append("unknown format")
    if pubkey_path:
        ser, _, _ = _crypto()
        with open(pubkey_path, "rb") as f:
            pub = ser.load_pem_public_key(f.read())
        if cert.get("key_id") != key_id(pub):
            problems.append("signed with another key")
        try:
            pub.verify(base64.b64decode(cert.get("signature", "")), canonical(cert))
        except Exception:  # noqa: BLE001  (InvalidSignature and malformed input alike)
            problems.append("bad signature")
    now = now or dt.datetime.now(dt.timezone.utc)
    try:
        if now > dt.datetime.fromisoformat(cert["valid_until"]):
            problems.append("expired")
        if now < dt.datetime.fromisoformat(cert["issued"]):
            problems.append("issued in the future")
    except (KeyError, ValueError):
        problems.append("unreadable validity window")
    d = os.path.dirname(os.path.abspath(path))
    for name, h in cert.get("evidence_sha256", {}).items():
        got = _sha256(os.path.join(d, name))
        if got is None:
            problems.append(f"evidence missing: {name}")
        elif got != h:
            problems.append(f"evidence changed: {name}")
    return {"valid": not problems, "problems": problems, "verdict": cert.get("result", {}).get("verdict"),
            "gpu": cert.get("gpu")}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.certify")
    sub = ap.add_subparsers(dest="cmd", required=True)
    k = sub.add_parser("keygen")
    k.add_argument("--out", required=True)
    s = sub.add_parser("sign")
    s.add_argument("screen")
    s.add_argument("--ops")
    s.add_argument("--key")
    s.add_argument("--issuer", default="")
    s.add_argument("--days", type=float, default=30.0)
    v = sub.add_parser("verify")
    v.add_argument("certificate")
    v.add_argument("--pubkey")
    a = ap.parse_args(argv)
    if a.cmd == "keygen":
        print(json.dumps(dict(zip(("private", "public"), keygen(a.out)))))
        return 0
    if a.cmd == "sign":
        with open(a.screen) as f:
            screen = json.load(f)
        ops = None
        if a.ops:
            with open(a.ops) as f:
                ops = json.load(f)
        cert = make(screen, ops, a.issuer, a.days, base_dir=os.path.dirname(os.path.abspath(a.screen)))
        if a.key:
            cert = sign(cert, a.key)
        out = os.path.join(os.path.dirname(os.path.abspath(a.screen)), "certificate.json")
        with open(out, "w") as f:
            json.dump(cert, f, indent=1)
        print(json.dumps({"certificate": out, "verdict": cert["result"]["verdict"], "signed": "signature" in cert}))
        return 0 if cert["result"]["verdict"] == "PASS" else 1
    r = verify(a.certificate, a.pubkey)
    print(json.dumps(r))
    return 0 if r["valid"] else 1


if __name__ == "__main__":
    raise SystemExit(main())

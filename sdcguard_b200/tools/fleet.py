"""Fleet view: every GPU's latest screen, operator screen and certificate, as one HTML page, a JSON table and a
quarantine list.

    python -m sdcguard_b200.tools.fleet collect /shared/screens --out fleet_out [--pubkey fleet.pub] [--days 30]

Each directory below the roots that holds a `screen.json`, `screen_ops.json` or `certificate.json` is one result of
one GPU (keyed by its UUID, else its serial, else the directory). Per GPU the newest result within the window counts:

  quarantine   a FAIL (the workload screen, an operator test, or a certificate's verdict), or a certificate whose
               signature or evidence does not verify
  stale        the newest result is older than the window
  ok           passed within the window

`fleet_out/` gets `fleet.json` (rows), `fleet.html` (a sortable table, worst first), `quarantine.txt` (one UUID or
serial per line, for a scheduler's drain list) and, per quarantined GPU, a zip of its result files for an RMA case.

Reference: src/sdcguard/fleet.py (`collect` :260, `write` :430, RMA zip `_rma_zip` :366).
"""
from __future__ import annotations

import argparse
import html
import json
import os
import time
import zipfile
from typing import Iterable, Optional

FILES = ("screen.json", "screen_ops.json", "certificate.json")
RANK = {"quarantine": 0, "stale": 1, "ok": 2}


def _load(p: str) -> Optional[dict]:
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def _row(d: str, pubkey: Optional[str], now: float, window_s: float) -> Optional[dict]:
    docs = {n: _load(os.path.join(d, n)) for n in FILES if os.path.exists(os.path.join(d, n))}
    if not docs:
        return None
    screen, ops, cert = docs.get("screen.json"), docs.get("screen_ops.json"), docs.get("certificate.json")
    tel = (screen or ops or {}).get("telemetry_before") or {}
    gpu = (cert or {}).get("gpu") or {}
    key = tel.get("uuid") or gpu.get("uuid") or tel.get("serial") or gpu.get("serial") or d
    reasons = []
    if any(v is None for v in docs.values()):
        reasons.append("unreadable result file")
    if screen and screen.get("verdict") != "PASS":
        reasons.append(f"workload screen {screen.get('verdict')} (rounds {screen.get('failed_rounds')})")
    if ops and ops.get("verdict") != "pass":
        bad = [k for k, v in ops.get("tests", {}).items() if v.get("verdict") != "pass"]
        reasons.append(f"operator screen {ops.get('verdict')} {bad}")
    if cert:
        from .certify import verify
        v = verify(os.path.join(d, "certificate.json"), pubkey)
        if cert.get("result", {}).get("verdict") != "PASS":
            reasons.append("certificate verdict FAIL")
        if not v["valid"] and not (v["problems"] == ["expired"]):
            reasons.append(f"certificate does not verify: {v['problems']}")
    mtime = max(os.path.getmtime(os.path.join(d, n)) for n in docs)
    status = "quarantine" if reasons else ("stale" if now - mtime > window_s else "ok")
    return {"gpu": key, "name": tel.get("name") or gpu.get("name") or (screen or {}).get("gpu"),
            "pci": tel.get("pci.bus_id") or gpu.get("pci"), "dir": d, "time": mtime, "status": status,
            "reasons": reasons, "files": sorted(docs)}


def collect(roots: Iterable[str], window_days: float = 30.0, pubkey: Optional[str] = None,
            now: Optional[float] = None) -> list[dict]:
    now = now or time.time()
    newest: dict = {}
    for root in roots:
        for d, _, files in os.walk(root):
            if not any(f in FILES for f in files):
                continue
            r = _row(d, pubkey, now, window_days * 86400)
            if r and (r["gpu"] not in newest or r["time"] > newest[r["gpu"]]["time"]):
                newest[r["gpu"]] = r
    return sorted(newest.values(), key=lambda r: (RANK[r["status"]], r["gpu"]))


def write(rows: list[dict], out_dir: str) -> dict:
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "fleet.json"), "w") as f:
        json.dump(rows, f, indent=1)
    q = [r for r in rows if r["status"] == "quarantine"]
    with open(os.path.join(out_dir, "quarantine.txt"), "w") as f:
        f.write("".join(r["gpu"] + "\n" for r in q))
    zips = []
    for r in q:
        name = os.path.join(out_dir, "rma_" + "".join(c if c.isalnum() or c in "-_" else "_" for c in r["gpu"])[:80]
                            + ".zip")
        with zipfile.ZipFile(name, "w", zipfile.ZIP_DEFLATED) as z:
            for fn in os.listdir(r["dir"]):
                p = os.path.join(r["dir"], fn)
                if os.path.isfile(p) and os.path.getsize(p) < (256 << 20):
                    z.write(p, fn)
        zips.append(name)
    cells = "".join(
        f"<tr class='{r['status']}'><td>{html.escape(r['status'])}</td><td>{html.escape(str(r['gpu']))}</td>"
        f"<td>{html.escape(str(r['name']))}</td><td>{html.escape(str(r['pci']))}</td>"
        f"<td>{time.strftime('%Y-%m-%d %H:%M', time.gmtime(r['time']))}</td>"
        f"<td>{html.escape('; '.join(r['reasons']))}</td></tr>" for r in rows)
    page = ("<!doctype html><meta charset='utf-8'><title>GPU fleet</title><style>td{padding:2px 8px}"
            ".quarantine{background:#fbb}.stale{background:#ffd}.ok{background:#dfd}</style>"
            f"<h1>GPU fleet: {len(rows)} GPUs, {len(q)} quarantined</h1><table><tr><th>status</th><th>GPU</th>"
            f"<th>model</th><th>PCI</th><th>last result (UTC)</th><th>why</th></tr>{cells}</table>")
    with open(os.path.join(out_dir, "fleet.html"), "w") as f:
        f.write(page)
    return {"gpus": len(rows), "quarantined": len(q), "stale": sum(r["status"] == "stale" for r in rows),
            "rma_zips": zips}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.fleet")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("collect")
    c.add_argument("roots", nargs="+")
    c.add_argument("--out", required=True)
    c.add_argument("--pubkey")
    c.add_argument("--days", type=float, default=30.0)
    a = ap.parse_args(argv)
    s = write(collect(a.roots, a.days, a.pubkey), a.out)
    print(json.dumps(s))
    return 1 if s["quarantined"] else 0


if __name__ == "__main__":
    raise SystemExit(main())

"""Results board: shared `check` cards aggregated by GPU model and provider, with an output-fingerprint reference.

    python -m sdcguard_b200.tools.board --dir results/ --out board_out

Reads every `*.json` card below the directories, keeps the valid ones and writes:

  index.html      totals, a table per GPU model (runs, distinct GPUs, PASS / FAIL, median checked and library TFLOPS,
                  copy bandwidth, fingerprint agreement) and per provider, and the FAIL cards
  results.json    every accepted card
  reference.json  per exact setup (GPU model, GEMM size, seed, CUDA version), how many distinct GPUs gave each output
                  fingerprint: the checked GEMM is deterministic, so a healthy GPU matches the majority, and `check`
                  can compare a new card against it
  rejected.json   cards that failed validation, with the reason

Validation: schema, digest of the contents, result word, plausible numbers (finite, in range), consistency (a PASS
card has no wrong results), at least a minute of checking. Cards are self-reported; hardware ids are hashed.

Reference: src/sdcguard/board.py:1-20 (outputs and acceptance rules), `validate` :195, `aggregate` :270.
"""
from __future__ import annotations

import argparse
import html
import json
import math
import os
import statistics
from typing import Optional

from .check import SCHEMA, card_digest

MIN_MINUTES = 1.0


def _num(v, lo=0.0, hi=1e9) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v) and lo <= v <= hi


def validate(c: dict) -> Optional[str]:
    """None if the card is acceptable, else the reason."""
    if not isinstance(c, dict) or c.get("schema") != SCHEMA:
        return "not a check card"
    if c.get("digest") != card_digest(c):
        return "digest does not match the contents"
    if c.get("result") not in ("PASS", "FAIL"):
        return "unknown result"
    sp, ck = c.get("speed") or {}, c.get("checked") or {}
    for k in ("checked_tflops", "cublas_tflops", "d2d_gbs"):
        if not _num(sp.get(k), 0, 1e5):
            return f"implausible speed.{k}"
    for k in ("gemm_checks", "copies_verified", "wrong"):
        if not _num(ck.get(k), 0, 1e15):
            return f"implausible checked.{k}"
    if c["result"] == "PASS" and ck.get("wrong"):
        return "PASS card with wrong results"
    if c["result"] == "FAIL" and not ck.get("wrong"):
        return "FAIL card without wrong results"
    if not _num(c.get("minutes"), MIN_MINUTES, 1e6):
        return f"checked for less than {MIN_MINUTES} minute"
    if not (c.get("gpu") or {}).get("name"):
        return "no GPU model"
    return None


def load(dirs: list[str]) -> tuple[list, list]:
    ok, bad = [], []
    for d in dirs:
        for root, _, files in os.walk(d):
            for fn in sorted(files):
                if not fn.endswith(".json"):
                    continue
                p = os.path.join(root, fn)
                try:
                    with open(p) as f:
                        c = json.load(f)
                except (OSError, ValueError) as e:
                    bad.append({"file": p, "reason": f"unreadable: {e}"})
                    continue
                why = validate(c)
                if why:
                    bad.append({"file": p, "reason": why})
                else:
                    ok.append({**c, "_file": p})
    return ok, bad


def _med(v):
    v = [x for x in v if _num(x, 0, 1e9)]
    return round(statistics.median(v), 1) if v else None


def aggregate(cards: list[dict]) -> dict:
    models: dict = {}
    providers: dict = {}
    fps: dict = {}
    for c in cards:
        name = c["gpu"]["name"]
        gid = c["gpu"].get("id_hash") or c["digest"]
        m = models.setdefault(name, {"runs": 0, "gpus": set(), "PASS": 0, "FAIL": 0, "tflops": [], "lib": [],
                                     "bw": []})
        m["runs"] += 1
        m["gpus"].add(gid)
        m[c["result"]] += 1
        m["tflops"].append(c["speed"]["checked_tflops"])
        m["lib"].append(c["speed"]["cublas_tflops"])
        m["bw"].append(c["speed"]["d2d_gbs"])
        f = c.get("fingerprint") or {}
        if f.get("key") and f.get("output"):
            fps.setdefault(f["key"], {}).setdefault(f["output"], set()).add(gid)
        p = providers.setdefault(c.get("provider") or "not stated", {"runs": 0, "PASS": 0, "FAIL": 0})
        p["runs"] += 1
        p[c["result"]] += 1
    out_models = {}
    for name, m in models.items():
        keys = [k for k in fps if k.startswith(name + "|")]
        agree = sum(max(len(g) for g in fps[k].values()) for k in keys)
        total = sum(sum(len(g) for g in fps[k].values()) for k in keys)
        out_models[name] = {"runs": m["runs"], "gpus": len(m["gpus"]), "PASS": m["PASS"], "FAIL": m["FAIL"],
                            "median_checked_tflops": _med(m["tflops"]), "median_library_tflops": _med(m["lib"]),
                            "median_d2d_gbs": _med(m["bw"]), "fingerprint_agreement": [agree, total]}
    return {"totals": {"cards": len(cards), "gpus": len({c["gpu"].get("id_hash") or c["digest"] for c in cards}),
                       "PASS": sum(c["result"] == "PASS" for c in cards),
                       "FAIL": sum(c["result"] == "FAIL" for c in cards), "models": len(models)},
            "models": out_models, "providers": providers,
            "reference": {k: {o: len(g) for o, g in outs.items()} for k, outs in fps.items()}}


def build(dirs: list[str], out: str) -> dict:
    cards, rejected = load(dirs)
    agg = aggregate(cards)
    os.makedirs(out, exist_ok=True)
    with open(os.path.join(out, "results.json"), "w") as f:
        json.dump([{k: v for k, v in c.items() if k != "_file"} for c in cards], f, indent=1)
    with open(os.path.join(out, "reference.json"), "w") as f:
        json.dump({"schema": "sdcguard-b200-board-reference/1", "fingerprints": agg["reference"]}, f, indent=1)
    with open(os.path.join(out, "rejected.json"), "w") as f:
        json.dump(rejected, f, indent=1)
    e = html.escape
    rows = "".join(f"<tr><td>{e(n)}</td><td>{m['runs']}</td><td>{m['gpus']}</td><td>{m['PASS']}</td><td>{m['FAIL']}"
                   f"</td><td>{m['median_checked_tflops']}</td><td>{m['median_library_tflops']}</td>"
                   f"<td>{m['median_d2d_gbs']}</td><td>{m['fingerprint_agreement'][0]}/"
                   f"{m['fingerprint_agreement'][1]}</td></tr>" for n, m in sorted(agg["models"].items()))
    prov = "".join(f"<tr><td>{e(p)}</td><td>{v['runs']}</td><td>{v['PASS']}</td><td>{v['FAIL']}</td></tr>"
                   for p, v in sorted(agg["providers"].items()))
    fails = "".join(f"<li>{e(c['gpu']['name'])} {e(str(c['gpu'].get('id_hash')))}: {c['checked']['wrong']} wrong "
                    f"({e(os.path.basename(c['_file']))})</li>" for c in cards if c["result"] == "FAIL")
    t = agg["totals"]
    page = (f"<!doctype html><meta charset='utf-8'><title>GPU check board</title><h1>GPU check board</h1>"
            f"<p>{t['cards']} cards, {t['gpus']} GPUs, {t['models']} models: {t['PASS']} PASS, {t['FAIL']} FAIL</p>"
            "<h2>By GPU model</h2><table><tr><th>model</th><th>runs</th><th>GPUs</th><th>PASS</th><th>FAIL</th>"
            "<th>checked TFLOPS</th><th>library TFLOPS</th><th>D2D GB/s</th><th>fingerprint agreement</th></tr>"
            f"{rows}</table><h2>By provider</h2><table><tr><th>provider</th><th>runs</th><th>PASS</th><th>FAIL</th>"
            f"</tr>{prov}</table><h2>FAIL cards</h2><ul>{fails}</ul>")
    with open(os.path.join(out, "index.html"), "w") as f:
        f.write(page)
    return {"accepted": len(cards), "rejected": len(rejected), **t}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.tools.board")
    ap.add_argument("--dir", nargs="+", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    print(json.dumps(build(a.dir, a.out)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

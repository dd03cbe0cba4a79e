"""python -m sdcguard_b200.lifetime explore --model pd-abort:buggy [--budget 3]
   python -m sdcguard_b200.lifetime explore --all
   python -m sdcguard_b200.lifetime check events.jsonl
   python -m sdcguard_b200.lifetime realsearch --toy push|pull|wakeup [--fixed]   (model-free search of real code)
   python -m sdcguard_b200.lifetime conformance [--json]                          (pd.py components, CPU mocks)"""
from __future__ import annotations

import argparse
import json
import sys

from . import adapter
from .explore import explore
from .models import MODELS, make


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.lifetime")
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("explore")
    e.add_argument("--model")
    e.add_argument("--all", action="store_true")
    e.add_argument("--budget", type=int, default=3)
    c = sub.add_parser("check")
    c.add_argument("events")
    rs = sub.add_parser("realsearch")
    rs.add_argument("--toy", required=True, choices=("push", "pull", "wakeup"))
    rs.add_argument("--fixed", action="store_true")
    rs.add_argument("--json", action="store_true")
    cf = sub.add_parser("conformance")
    cf.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    if a.cmd == "realsearch":
        from . import realsearch, toys
        r = realsearch.search(lambda: toys.TOYS[a.toy](fixed=a.fixed))
        print(json.dumps(r.as_dict(), indent=1) if a.json else realsearch.text(r))
        return 1 if r.findings else 0
    if a.cmd == "conformance":
        from . import conformance
        return conformance.main(["--json"] if a.json else [])
    if a.cmd == "check":
        r = adapter.check(adapter.load(a.events))
        print(json.dumps(r, indent=1))
        return 1 if r["violations"] else 0
    names = [f"{k}:{v}" for k, cls in MODELS.items() for v in cls.VARIANTS] if a.all else [a.model]
    out = [explore(make(n), a.budget).as_dict() for n in names]
    print(json.dumps(out if a.all else out[0], indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Conformance of this package's own prefill/decode components to the lifetime rules, run on the CPU with mocks.

    python -m sdcguard_b200.lifetime conformance [--json]

The components under test are the real functions of `serve/pd.py` (`produce`, `consume`, `release_producer`) and its
`PrefixCache`, unchanged. What they drive is mocked on the CPU: an engine with the real `BlockAllocator` and a small
bf16 KV cache whose prefill writes a deterministic function of the prompt into each page, and the two transfer
kernels replaced by CPU versions with the same contract (`page_checksum_reference` for the checksums; a page copy that
hashes on arrival and compares for the pull). No GPU, network or subprocess is used.

Scenarios (each a sequence of component calls; the recorded lifetime events are replayed through the ledger):
  ordered            produce -> consume -> release_producer (the order `pd.run_single_process` and `pd_mp` use)
  prefix_reuse       two rounds with shared prefixes, so the second round reuses cached prefix pages
  early_release      release_producer before consume, then a new prefill reuses the freed pages: a misuse the
                     rules must catch (a pull names a producer allocation that is no longer current)
The result says, per scenario, the ledger's violations and whether they match the expectation (none for the first
two, at least one for the third). A satisfied result covers these component functions under these mocks, not the
GPU kernels or a deployment.

Reference: src/sdcguard/lifetime/component_conformance.py:1-20 (pinned component functions run with controlled CPU
mocks; the allocation / read / done and release paths; a satisfied result is not a physical-write attestation).
"""
from __future__ import annotations

import contextlib
import json
import sys
from dataclasses import dataclass

import torch

from . import adapter

PAGE = 16


@dataclass
class _Cfg:
    vocab: int = 1000
    name: str = "mock"


class MockEngine:
    """The engine surface pd.py uses: device, cfg, alloc, cache, prefill, decode_from."""

    def __init__(self, num_blocks: int = 64):
        from ..serve.engine import BlockAllocator
        self.device = torch.device("cpu")
        self.cfg = _Cfg()
        self.alloc = BlockAllocator(num_blocks)
        self.cache = torch.zeros(2, num_blocks, 2, 1, PAGE, 8, dtype=torch.bfloat16)

    def prefill(self, prompts, plens, pages, out) -> None:
        for i, (n, pg) in enumerate(zip(plens, pages)):
            for b, p in enumerate(pg):
                toks = prompts[i, b * PAGE:min(n, (b + 1) * PAGE)].float()
                self.cache[:, p].zero_()
                self.cache[:, p, :, :, :toks.numel(), :] = (toks.view(1, 1, 1, -1, 1) % 97).to(torch.bfloat16)
            out[i, 0] = int(prompts[i, n - 1]) % self.cfg.vocab

    def decode_from(self, plens, pages, out_tokens, max_new_tokens) -> None:
        for i in range(out_tokens.shape[0]):
            out_tokens[i, 1:] = out_tokens[i, 0]


@contextlib.contextmanager
def cpu_transfers():
    """Replace the two transfer kernels in pd's namespace by CPU versions with the same contract."""
    from ..ops import kv_transfer as real
    from ..serve import pd

    def page_checksums(cache, pages, seed=real.DEFAULT_SEED, out=None):
        v = [real.page_checksum_reference(cache, int(p), seed) for p in pages.tolist()]
        return torch.tensor([x - (1 << 64) if x >= (1 << 63) else x for x in v], dtype=torch.int64)

    def pull_pages(src, dst, sp, dp, want, seed=real.DEFAULT_SEED, state_row=None, acc=None):
        got, res = [], []
        for s, d, w in zip(sp.tolist(), dp.tolist(), want.tolist()):
            dst[:, d] = src[:, s]
            h = real.page_checksum_reference(dst, d, seed)
            got.append(h - (1 << 64) if h >= (1 << 63) else h)
            res.append(1 if (h & 0xFFFFFFFFFFFFFFFF) == (w & 0xFFFFFFFFFFFFFFFF) else 2)
        return torch.tensor(got, dtype=torch.int64), torch.tensor(res, dtype=torch.int32)

    saved = (pd.kvx.page_checksums, pd.kvx.pull_pages)
    pd.kvx.page_checksums, pd.kvx.pull_pages = page_checksums, pull_pages
    try:
        yield
    finally:
        pd.kvx.page_checksums, pd.kvx.pull_pages = saved


def _requests(round_: int, n: int = 4, prefix: int = 40):
    g = torch.Generator().manual_seed(11)
    pre = torch.randint(0, 1000, (prefix,), generator=g).tolist()
    return [(f"r{round_}-{i}", pre + torch.randint(0, 1000, (5 + 3 * i,), generator=g).tolist()) for i in range(n)]


def _scenario(name: str) -> list[dict]:
    from ..serve import pd
    prod, cons = MockEngine(), MockEngine()
    sink = adapter.EventSink()
    rec, prefix = pd.Recorder(), pd.PrefixCache()
    rounds = 2 if name == "prefix_reuse" else 1
    for r in range(rounds):
        ts = pd.produce(prod, _requests(r), sink=sink)
        if name == "early_release":
            pd.release_producer(prod, ts, sink=sink)
            pd.produce(prod, _requests(9), sink=sink)          # the freed pages go to new requests
        pd.consume(cons, ts, prod.cache, prefix, rec, 4, sink=sink)
        if name != "early_release":
            pd.release_producer(prod, ts, sink=sink)
    return sink.events


SCENARIOS = {"ordered": False, "prefix_reuse": False, "early_release": True}     # name -> violations expected


def run_component_conformance() -> dict:
    out = {"schema": "sdcguard_b200.component-conformance.v1", "scenarios": {}, "scope":
           "serve/pd.py component functions with CPU mocks of the engine and the transfer kernels"}
    with cpu_transfers():
        for name, expect in SCENARIOS.items():
            ev = _scenario(name)
            r = adapter.check(ev)
            rules = sorted({v["rule"] for v in r["violations"]})
            out["scenarios"][name] = {"events": r["events"], "rules": rules, "expected_violations": expect,
                                      "conforms": bool(rules) == expect,
                                      "first": r["violations"][0]["message"] if r["violations"] else None}
    out["conforms"] = all(s["conforms"] for s in out["scenarios"].values())
    return out


def main(argv=None) -> int:
    r = run_component_conformance()
    if argv and "--json" in argv:
        print(json.dumps(r, indent=1))
    else:
        for n, s in r["scenarios"].items():
            print(f"{'ok  ' if s['conforms'] else 'FAIL'} {n}: {s['events']} events, rules {s['rules'] or 'none'}"
                  + (f" ({s['first']})" if s["first"] else ""))
    return 0 if r["conforms"] else 1


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1:]))

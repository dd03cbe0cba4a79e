"""KV lifetime: the ledger's four rules, the explorer on the protocol models (buggy variants break their rule with the
fewest delays, fixed variants break none), and the adapter on recorded event streams."""
import pytest

from sdcguard_b200.lifetime import adapter
from sdcguard_b200.lifetime.explore import explore
from sdcguard_b200.lifetime.ledger import Ledger
from sdcguard_b200.lifetime.models import make

EXPECT = {
    "pd-abort:buggy": {"R2"}, "pd-abort:fixed": set(), "pd-abort:release-timeout": {"R2"},
    "pd-lease:buggy": {"R1", "R2"}, "pd-lease:fixed": set(),
    "pd-notify:buggy": {"R4"}, "pd-notify:fixed": set(),
    "offload-load:buggy": {"R3"}, "offload-load:fixed": set(),
}


@pytest.mark.parametrize("name", sorted(EXPECT))
def test_explorer_finds_exactly_the_buggy_orderings(name):
    r = explore(make(name), budget=4)
    assert {f.rule for f in r.findings} == EXPECT[name], [f.as_dict() for f in r.findings]
    assert not r.coverage["bounds_hit"]
    for f in r.findings:
        assert f.trace and any("VIOLATION" in t for t in f.trace)
        assert f.delays <= 4


def test_findings_need_their_departures():
    r = explore(make("pd-abort:buggy"), budget=3)
    f = r.findings[0]
    assert f.delays == 2 and any("timeout" in d[1] for d in f.departures)


def test_ledger_rules_directly():
    led = Ledger()
    h1 = led.alloc(("d", 0), "a")
    led.submit("w", "write", "p", dst=h1, payload=("a", 1, "kv"))
    led.free(h1)
    h2 = led.alloc(("d", 0), "b")                        # R2: w still outstanding
    led.submit("w2", "write", "p", dst=h1)               # R1: h1 is stale
    led.complete("w", h2)                                 # R4: w never named h2
    led.consume(h2, "b")                                  # R3: not ready / written by w? (w completed) -> not ready
    assert [v.rule for v in led.violations] == ["R2", "R1", "R4", "R3"]


def _good_stream():
    s = adapter.EventSink()
    for p in (0, 1):
        s.alloc("prefill", p, "r1")
        s.local_write("prefill", p, "r1")
    for p in (5, 6):
        s.alloc("decode", p, "r1")
    s.transfer("read", "pull", ("prefill", 0), ("decode", 5))
    s.transfer("read", "pull", ("prefill", 1), ("decode", 6))
    s.consume("decode", 5, "r1")
    s.consume("decode", 6, "r1")
    s.share("decode", 5, "r2")                           # a cached prefix page reused by r2
    s.consume("decode", 5, "r2")
    s.free("prefill", 0)
    s.free("prefill", 1)
    return s


def test_adapter_on_recorded_streams(tmp_path):
    s = _good_stream()
    assert adapter.check(s.events)["violations"] == []
    bad = adapter.EventSink(str(tmp_path / "ev.jsonl"))
    bad.alloc("prefill", 0, "r1")
    bad.local_write("prefill", 0, "r1")
    bad.free("prefill", 0)                               # producer released before the pull
    bad.alloc("prefill", 0, "r9")
    bad.local_write("prefill", 0, "r9")
    bad.alloc("decode", 3, "r1")
    bad.transfer("read", "pull", ("prefill", 0), ("decode", 3))            # reads the reused page
    bad.consume("decode", 3, "r1")
    bad.alloc("decode", 4, "r1")
    bad.transfer("read", "pull", ("prefill", 0), ("decode", 4), src_gen=1)  # names r1's old allocation
    bad.close()
    r = adapter.check(adapter.load(str(tmp_path / "ev.jsonl")))
    assert [v["rule"] for v in r["violations"]] == ["R3", "R1"], r  # r1 received r9's data; a stale handle
    s2 = adapter.EventSink()
    s2.alloc("decode", 1, "a")
    s2.consume("decode", 1, "b")
    assert adapter.check(s2.events)["violations"][0]["rule"] == "R3"

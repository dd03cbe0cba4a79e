"""Server probes against fakes (no GPU): readiness verdicts from metrics, isolation and consistency against a
deterministic fake model, throughput bookkeeping, and the stack-change decision."""
import os
import threading
import time

import pytest

from sdcguard_b200.tools import _client, consistency, decide, isolation, perf, ready


def _next(ctx):
    return (sum(ctx) * 31 + len(ctx)) % 1000


def fake_complete(base, prompt, n):
    ctx, out = list(prompt), []
    for _ in range(n):
        t = _next(ctx)
        out.append(t)
        ctx.append(t)
    return out


def fake_score(base, prompt, k):
    """Teacher-forced scores of the fake model: at each position its next token first (margin 3 nats)."""
    vals, ids = [], []
    for p in range(len(prompt)):
        t = _next(list(prompt[: p + 1]))
        ids.append([t] + [(t + j) % 1000 for j in range(1, k)])
        vals.append([-0.1] + [-3.1 - j for j in range(1, k)])
    return {"top_logprobs": vals, "top_ids": ids}


def _text(checks, tokens, alarms=0, protected=1, ops=10, ops_checked=10, polls=3, started="1", line=6.0,
          confirmed=None, alerts=None, layers=8, ratio=1.0, uuid="u", precision="bf16", share=1.0, spot="true",
          z=6.0, longest=64, scan=None, fp8=None):
    t = (f"sdcguard_protected {protected}\nsdcguard_checks_total {checks}\nsdcguard_alarms_total {alarms}\n"
         f"sdcguard_ops_total {ops}\nsdcguard_ops_checked {ops_checked}\nsdcguard_alarm_line {line}\n"
         f"sdcguard_polls_total {polls}\nsdcguard_generated_tokens_total {tokens}\n"
         f"sdcguard_layers_checked {layers}\nsdcguard_layers_unchecked 0\nsdcguard_weights_checked_ratio {ratio}\n"
         f"sdcguard_longest_prompt_tokens {longest}\n"
         f'sdcguard_worker_info{{gpu="B200",uuid="{uuid}",pid="7",started="{started}"}} 1\n'
         f'sdcguard_stack_info{{model="tiny",precision="{precision}",weights_digest="abc",version="0.2"}} 1\n'
         f'sdcguard_protection_info{{share="{share}",offset="0",norms="true",rope="true",attn="true",act="true",'
         f'spot="{spot}",z="{z}",weight_scan="{"true" if scan else "false"}"}} 1\n')
    if confirmed is not None:
        t += f"sdcguard_confirmed_alerts_total {confirmed}\n"
    t += f"sdcguard_alerts_total {alerts if alerts is not None else alarms}\n"
    if scan is not None:
        t += "".join(f"sdcguard_weight_scan_{k} {v}\n" for k, v in scan.items())
    if fp8 is not None:
        t += f"sdcguard_fp8_layers_checked 8\nsdcguard_fp8_calls_judged_total {fp8[0]}\n" \
             f"sdcguard_fp8_findings_total {fp8[1]}\n"
    return t


def _metrics(*a, **k):
    return _client.parse_metrics(_text(*a, **k))


def test_ready_verdicts():
    assert ready.judge(_metrics(10, 5), _metrics(20, 9))["verdict"] == "PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(10, 5))["verdict"] == "IDLE"
    assert ready.judge(_metrics(10, 5), _metrics(10, 9))["verdict"] == "NOT PROTECTED"      # tokens, no checks
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, alarms=1))["verdict"] == "FAULT FOUND"
    # an alarm whose own evidence cleared it is a note, unless --strict-alerts
    r = ready.judge(_metrics(10, 5), _metrics(20, 9, alarms=1, confirmed=0))
    assert r["verdict"] == "PROTECTED" and r["notes"]
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, alarms=1, confirmed=0),
                       strict_alerts=True)["verdict"] == "FAULT FOUND"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, protected=0))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, line=1000))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, started="2"))["verdict"] == "INCONCLUSIVE"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, ops_checked=8))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(0, 0, polls=0), _metrics(0, 0, polls=0))["verdict"] == "INCONCLUSIVE"
    assert ready.judge(None, _metrics(1, 1))["verdict"] == "NOT PROTECTED"
    # requirements
    assert ready.judge(_metrics(10, 5), _metrics(20, 9), layers=9)["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, ratio=0.25), min_weights=0.5)["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9), gpus=["v"])["verdict"] == "NOT PROTECTED"
    # two workers: both must move; on one GPU each; same layer count
    two = [_metrics(10, 5, uuid="a"), _metrics(10, 5, uuid="b")]
    assert ready.judge(two, [_metrics(20, 9, uuid="a"), _metrics(20, 9, uuid="b")])["verdict"] == "PROTECTED"
    assert ready.judge(two, [_metrics(20, 9, uuid="a"), _metrics(10, 9, uuid="b")])["verdict"] == "NOT PROTECTED"
    assert ready.judge(two, [_metrics(20, 9, uuid="a"), _metrics(20, 9, uuid="a")])["verdict"] == "NOT PROTECTED"
    assert ready.judge(two, [_metrics(20, 9, uuid="a"), _metrics(20, 9, uuid="b", layers=4)])["verdict"] == \
        "NOT PROTECTED"


def _decision(**over):
    d = decide.decide(None, quality={"verdict": "PASS", "mean_kl": 0.0, "top1_agreement": 1.0},
                      alerts=[], metrics=[_text(50, 9)])
    d.update(over)
    return d


def test_ready_qualified():
    d = _decision()
    assert d["decision"] == "ACCEPT", d["why"]
    assert ready.qualified([_metrics(20, 9)], d) == {"verdict": None, "notes": []}
    q = ready.qualified([_metrics(20, 9, precision="fp8")], d)
    assert q["verdict"] == "NOT THE QUALIFIED STACK" and "precision" in q["why"][0]
    assert ready.qualified([_metrics(20, 9)], dict(d, decision="REJECT"))["verdict"] == "NOT QUALIFIED"
    # weaker checks than qualified
    q = ready.qualified([_metrics(20, 9, share=0.5, spot="false")], d)
    assert q["verdict"] == "NOT PROTECTED" and any("spot" in w for w in q["why"]) and \
        any("share" in w for w in q["why"])
    assert ready.qualified([_metrics(20, 9, z=8.0)], d, max_z=10)["verdict"] == "NOT PROTECTED"
    # age: a decision older than the limit is inconclusive
    old = dict(d, created_unix=d["created_unix"] - 10 * 86400)
    assert ready.qualified([_metrics(20, 9)], old, max_age_days=5)["verdict"] == "INCONCLUSIVE"
    # served beyond the tested conditions: a note, or INCONCLUSIVE when strict
    t = dict(d, tested={"longest_prompt": 32})
    assert ready.qualified([_metrics(20, 9)], t)["notes"]
    assert ready.qualified([_metrics(20, 9)], t, strict_conditions=True)["verdict"] == "INCONCLUSIVE"
    r = ready.check(["a"], decision=dict(d, decision="REJECT"), window=0,
                    scrape=lambda u, it=iter([_metrics(10, 5), _metrics(20, 9)]): next(it))
    assert r["verdict"] == "NOT QUALIFIED" and ready.EXIT.get(r["verdict"], 1) == 1


def fake_cancel(base, prompt, n):
    return True


def test_isolation_consistency_perf_on_fake_model():
    assert isolation.run("x", probes=2, primers=3, complete=fake_complete, cancel=fake_cancel)["verdict"] == \
        "NO LEAK SEEN"
    # no stream could be dropped (no server at "x"): the cancellation probe judges nothing
    r = isolation.run("x", probes=1, primers=2, complete=fake_complete)
    assert r["verdict"] == "INCONCLUSIVE" and r["cancellation"]["dropped_mid_flight"] == 0
    assert consistency.run("x", probes=2, complete=fake_complete, score=fake_score)["verdict"] == "CONSISTENT"

    def wrong_decode(base, prompt, n):     # decode goes wrong after 3 tokens, while prefill paths are right
        out = fake_complete(base, prompt, n)
        return out[:3] + [(t + 7) % 1000 for t in out[3:]] if n > 1 else out
    r = consistency.run("x", probes=1, cuts=(), complete=wrong_decode, score=fake_score)
    assert r["verdict"] == "INCONSISTENT" and r["logprob_mismatches"][0]["generated_index"] == 3

    def tied_score(base, prompt, k):       # a near tie at every position: reported, never counted
        d = fake_score(base, prompt, k)
        d["top_logprobs"] = [[-0.1, -0.2] + v[2:] for v in d["top_logprobs"]]
        return d
    r = consistency.run("x", probes=1, cuts=(), complete=wrong_decode, score=tied_score)
    assert r["verdict"] == "CONSISTENT" and r["near_ties"] > 0 and not r["logprob_mismatches"]
    calls = [0]

    def flaky(base, prompt, n):          # the 3rd call (the batched one) differs: a batch-dependent server
        calls[0] += 1
        out = fake_complete(base, prompt, n)
        return [out[0] + 1] + out[1:] if calls[0] == 3 else out

    calls[0] = -100                          # (the concurrency probe's batched call comes after the primer probe)

    def batch_dependent(base, prompt, n):    # the probe's answer changes when other requests share its batch
        out = fake_complete(base, prompt, n)
        batched = threading.current_thread() is not threading.main_thread()     # sent beside other requests
        return [out[0] + 1] + out[1:] if batched and len(prompt) == 24 else out
    assert isolation.run("x", probes=1, primers=2, complete=batch_dependent)["verdict"] == "LEAK"

    state = {"last": None}

    def remembers(base, prompt, n):          # the answer depends on the previous request: a stale buffer
        out = fake_complete(base, prompt, n)
        prev, state["last"] = state["last"], prompt
        return [(out[0] + len(prev or [])) % 1000] + out[1:] if len(prompt) == 24 else out
    assert isolation.run("x", probes=1, primers=3, complete=remembers)["verdict"] == "LEAK"
    del flaky

    def bad_prefill(base, prompt, n):
        out = fake_complete(base, prompt, n)
        return [(out[0] + 1) % 1000] if n == 1 else out

    r = consistency.run("x", probes=1, complete=bad_prefill, score=None)
    assert r["verdict"] == "INCONSISTENT" and len(r["mismatches"]) == 4


def fake_stream(base, prompt, n):
    """A streamed request of the fake model: 10 ms to the first token, then 2 ms per token."""
    return {"ttft_s": 0.010, "gaps_s": [0.002] * (n - 1), "latency_s": 0.010 + 0.002 * (n - 1), "tokens": n,
            "chunks": n, "done": True}


def _perf(scale=1.0, spread=0.0, rounds=3, fail=False):
    k = [0]

    def req(base, prompt, n):
        k[0] += 1
        if fail and k[0] == 5:
            raise perf.RequestFailed("HTTP 500", {})
        r = fake_stream(base, prompt, n)
        time.sleep(0.0005)
        return r
    m = perf.measure("x", perf.default_load(8, lo=4, hi=8), concurrency=2, max_tokens=4, rounds=rounds, warmup=1,
                     request=req, info=lambda u: {"model": "tiny", "stack": None, "checks_on": True})
    for i, r in enumerate(m["rounds"]):          # make throughput deterministic: scale, with a chosen spread
        r["output_tokens_per_s"] = 100.0 * scale * (1.0 + spread * (i - 1))
    vals = [r["output_tokens_per_s"] for r in m["rounds"]]
    m["median"]["output_tokens_per_s"] = sorted(vals)[len(vals) // 2]
    m["spread"]["output_tokens_per_s"] = (max(vals) - min(vals)) / m["median"]["output_tokens_per_s"]
    return m


def test_perf_measure_and_compare():
    m = _perf()
    assert m["complete"] and len(m["rounds"]) == 3 and m["rounds"][0]["completed"] == 8
    assert abs(m["median"]["ttft_p50_ms"] - 10.0) < 1e-6 and abs(m["median"]["itl_p99_ms"] - 2.0) < 1e-6
    assert perf.percentile([1, 2, 3, 4], 0.5) == 2.5 and perf.percentile([], 0.5) is None
    base = _perf()
    assert perf.compare(base, _perf(1.10))["verdict"] == "FASTER"
    assert perf.compare(base, _perf(1.01))["verdict"] == "SAME"
    assert perf.compare(base, _perf(0.90))["verdict"] == "SLOWER"
    assert perf.compare(base, _perf(1.10, spread=0.1))["verdict"] == "SAME"          # inside twice the spread
    bad = _perf(fail=True)
    assert not bad["complete"] and perf.compare(base, bad)["verdict"] == "INCONCLUSIVE"
    other = _perf()
    other["load"] = dict(other["load"], max_tokens=5)
    assert not perf.compare(base, other)["comparable"]


def _alert(det, **detail):
    return {"detector": det, "step": 3, "detail": detail}


def test_decide_sections():
    ok_q = {"verdict": "PASS", "mean_kl": 1e-5, "top1_agreement": 1.0}
    full = dict(quality=ok_q, alerts=[], metrics=[_text(50, 9)], perf_before=_perf(), perf_after=_perf(0.98),
                isolation_run={"verdict": "NO LEAK SEEN", "why": []},
                consistency_run={"verdict": "CONSISTENT"})
    d = decide.decide(None, **full)
    assert d["decision"] == "ACCEPT", d["why"]
    assert d["arithmetic"]["verdict"] == "NO FAULT OBSERVED" and d["performance"]["verdict"] == "MEETS"
    assert d["weights"]["verdict"] == "NO CHANGE SEEN" and d["quantization"]["verdict"] == "UNMEASURED"
    # a slower candidate misses a required gain only when performance is required
    slow = dict(full, perf_after=_perf(0.5))
    assert decide.decide(None, **slow)["decision"] == "ACCEPT"
    d = decide.decide({"performance": {"required": True}}, **slow)
    assert d["decision"] == "REJECT" and d["performance"]["verdict"] == "MISSES"
    # arithmetic: a confirmed wrong output is a fault; an unconfirmed alarm leaves it undecided
    d = decide.decide(None, **dict(full, alerts=[_alert("checksum", layer="L0.qkv", recheck={"verdict":
                                                                                             "output_wrong"})],
                                   metrics=[_text(50, 9, alarms=1)]))
    assert d["decision"] == "REJECT" and d["arithmetic"]["verdict"] == "FAULT"
    d = decide.decide(None, **dict(full, alerts=[_alert("checksum", layer="L0.qkv")],
                                   metrics=[_text(50, 9, alarms=1)]))
    assert d["decision"] == "NOT DECIDED" and d["arithmetic"]["verdict"] == "INCONCLUSIVE"
    d = decide.decide(None, **dict(full, alerts=[_alert("checksum", layer="L0", recheck={"verdict":
                                                                                         "not_reproduced"})],
                                   metrics=[_text(50, 9, alarms=1)]))
    assert d["arithmetic"]["verdict"] == "NO FAULT OBSERVED" and d["arithmetic"]["notes"]
    # the alerts must be the ones counted; the weight share must reach the policy's
    d = decide.decide(None, **dict(full, metrics=[_text(50, 9, alarms=2)]))
    assert d["arithmetic"]["verdict"] == "INCONCLUSIVE"
    d = decide.decide(None, **dict(full, metrics=[_text(50, 9, ratio=0.25)]))
    assert d["arithmetic"]["verdict"] == "INCONCLUSIVE"
    assert decide.decide({"arithmetic": {"min_weights_checked": 0.2}},
                         **dict(full, metrics=[_text(50, 9, ratio=0.25)]))["decision"] == "ACCEPT"
    assert decide.decide(None, **dict(full, metrics=[_text(0, 9)]))["arithmetic"]["verdict"] == "INCONCLUSIVE"
    # other sources: kept gate cases and the kernel test
    d = decide.decide(None, quality=ok_q, gate={"cases": {"c1": {"verdict": "REGRESSED", "why": "wrong"}}})
    assert d["arithmetic"]["verdict"] == "FAULT"
    d = decide.decide(None, quality=ok_q, gate={"cases": {"c1": {"verdict": "PASSED"}}})
    assert d["decision"] == "ACCEPT"
    kt = {"calls": [{"call": "k | 64x64x64", "verdict": "PASSED", "runs": 3}], "counts": {"PASSED": 1}}
    assert decide.decide(None, quality=ok_q, kernel_test=kt)["decision"] == "ACCEPT"
    kt_bad = {"calls": [{"call": "k", "verdict": "WRONG", "runs": 3, "runs_wrong": 1}]}
    assert decide.decide(None, quality=ok_q, kernel_test=kt_bad)["arithmetic"]["verdict"] == "FAULT"
    assert decide.decide(None, quality=ok_q, kernel_test={"calls": [{"call": "k", "verdict": "NOT RUN"}]}
                         )["decision"] == "NOT DECIDED"
    # weights: a scan finding rejects; a complete scan verifies
    d = decide.decide(None, **dict(full, alerts=[_alert("weights", weight="layers.0.qkv")],
                                   metrics=[_text(50, 9, alarms=0, alerts=1)]))
    assert d["decision"] == "REJECT" and d["weights"]["verdict"] == "CHANGED"
    scan = {"entries": 40, "passes_total": 2, "never_compared": 0, "changed": 0, "left_out": 0,
            "oldest_age_seconds": 3.5}
    d = decide.decide(None, **dict(full, metrics=[_text(50, 9, scan=scan)]))
    assert d["weights"]["verdict"] == "VERIFIED" and d["decision"] == "ACCEPT"
    d = decide.decide(None, **dict(full, metrics=[_text(50, 9, scan=dict(scan, never_compared=3))]))
    assert d["weights"]["verdict"] == "NO CHANGE SEEN"
    # quantization
    assert decide.decide(None, **dict(full, metrics=[_text(50, 9, fp8=(20, 0))]))["quantization"]["verdict"] == \
        "RIGHT"
    d = decide.decide(None, **dict(full, alerts=[_alert("quantization", layer="L1.o.quant")],
                                   metrics=[_text(50, 9, alerts=1, fp8=(20, 1))]))
    assert d["quantization"]["verdict"] == "WRONG" and d["decision"] == "REJECT"
    # approximation and its policy
    assert decide.decide(None, **dict(full, quality=None))["decision"] == "NOT DECIDED"
    warn = dict(ok_q, verdict="WARN")
    assert decide.decide(None, **dict(full, quality=warn))["approximation"]["verdict"] == "OUTSIDE"
    assert decide.decide({"quality": {"accept_warn": True}}, **dict(full, quality=warn))["decision"] == "ACCEPT"
    assert decide.decide({"quality": {"min_top1": 1.01}}, **full)["approximation"]["verdict"] == "OUTSIDE"
    # isolation and consistency
    assert decide.decide(None, **dict(full, isolation_run={"verdict": "LEAK", "why": ["x"]}))["decision"] == \
        "REJECT"
    assert decide.decide({"isolation": {"required": True}}, **dict(full, isolation_run=None))["decision"] == \
        "NOT DECIDED"
    inc = {"verdict": "INCONSISTENT", "mismatches": [1], "largest_gap": 2.0, "probe_set": {"p": 1}}
    assert decide.decide(None, **dict(full, consistency_run=inc))["decision"] == "REJECT"
    same = dict(inc, largest_gap=1.8)
    assert decide.decide(None, **dict(full, consistency_run=inc, consistency_baseline=same))["decision"] == "ACCEPT"
    # unknown policy keys fail loudly; the text rendering names every section
    with pytest.raises(ValueError):
        decide.policy_with_defaults({"performance": {"speed": 1}})
    text = decide.render(decide.decide(None, **full))
    assert text.startswith("DECISION: ACCEPT") and "4b. Consistency" in text and "5. Scope" in text
    # still_applies against a stack record
    d = decide.decide(None, **full)
    st = d["scope"]["stacks"]["candidate"]
    assert decide.still_applies(d, st)["applies"] is True
    assert decide.still_applies(d, dict(st, precision="fp8"))["applies"] is False


def test_consistency_judge_against():
    base = {"verdict": "CONSISTENT", "largest_gap": 0.1, "probe_set": {"a": 1}}
    bad = {"verdict": "INCONSISTENT", "largest_gap": 3.0, "mismatches": [{}], "probe_set": {"a": 1}}
    assert consistency.judge_against(bad, base)["verdict"] == "INCONSISTENT"
    assert consistency.judge_against(bad, dict(bad, largest_gap=2.8))["verdict"] == "CONSISTENT"
    assert consistency.judge_against(bad, dict(bad, largest_gap=1.0))["verdict"] == "INCONSISTENT"
    assert consistency.judge_against(bad, dict(base, probe_set={"a": 2}))["verdict"] == "INCONCLUSIVE"
    assert consistency.judge_against({"verdict": "INCONCLUSIVE"})["verdict"] == "INCONCLUSIVE"


def test_qualify_helpers(tmp_path):
    from sdcguard_b200.tools import qualify
    assert qualify._pairs(["fp8=--precision fp8", "--unchecked"]) == [("fp8", "--precision fp8"),
                                                                      ("candidate2", "--unchecked")]
    with pytest.raises(ValueError):
        qualify._pairs(["a=x", "a=y"])
    (tmp_path / "report.txt").write_text("old")
    (tmp_path / "runs").mkdir()
    moved = qualify.set_aside_earlier(str(tmp_path))
    assert moved and os.path.exists(os.path.join(moved, "report.txt")) and not (tmp_path / "runs").exists()
    assert qualify.set_aside_earlier(str(tmp_path)) is None
    d = _decision()
    text = qualify.report([("fp8", d)])
    assert "fp8" in text and "ACCEPT" in text


def test_isolation_cancellation_probe():
    """Answers that change while requests of the same prompt heads are dropped mid-flight are a LEAK; solo answers
    that do not repeat make the probe inconclusive."""
    dropped = threading.Event()

    def cancel(base, prompt, n):
        dropped.set()
        return True

    def stale_after_drop(base, prompt, n):      # a dropped request's pages handed to a live one too early
        out = fake_complete(base, prompt, n)
        if threading.current_thread() is not threading.main_thread() and len(prompt) == 104:
            dropped.wait(2.0)
            return [(out[0] + 1) % 1000] + out[1:]
        return out
    r = isolation.cancel_probe("x", complete=stale_after_drop, cancel=cancel)
    assert r["verdict"] == "LEAK" and len(r["changed_under_load"]) == r["requests"] == 16, r
    assert r["dropped_mid_flight"] == r["cancelled"] == 8
    assert isolation.run("x", probes=1, primers=2, complete=stale_after_drop, cancel=cancel)["verdict"] == "LEAK"
    calls = {"n": 0}

    def noisy(base, prompt, n):                 # solo answers that do not repeat
        calls["n"] += 1
        out = fake_complete(base, prompt, n)
        return [(out[0] + calls["n"]) % 1000] + out[1:] if len(prompt) == 104 else out
    r = isolation.cancel_probe("x", complete=noisy, cancel=cancel)
    assert r["verdict"] == "INCONCLUSIVE" and r["controls_disagree"], r
    assert isolation.cancel_probe("x", complete=fake_complete, cancel=cancel)["verdict"] == "NO LEAK SEEN"


def test_consistency_prefix_cache_probe():
    """The cached answer must equal the cold one where two cold answers agree and the hit counter shows the cache
    read; without a counter the probe is not applicable and takes no part in the verdict."""
    cache, hits = set(), [0.0]

    def salted(bad):
        def complete(base, prompt, n, salt):
            key = (salt, tuple(prompt[:256]))
            cached = key in cache
            cache.add(key)
            if cached:
                hits[0] += 256
            out = fake_complete(base, prompt, n)
            return [(out[0] + 1) % 1000] + out[1:] if bad and cached else out
        return complete
    r = consistency.prefix_probe("x", complete_salted=salted(False), hits=lambda b: hits[0])
    assert r["verdict"] == "CONSISTENT" and all(c["cache_hit"] for c in r["cases"]), r
    r = consistency.prefix_probe("x", complete_salted=salted(True), hits=lambda b: hits[0])
    assert r["verdict"] == "INCONSISTENT" and r["cases"][0]["cached_first_difference"] == 0, r
    # a counter that does not move: no cache hit shown, nothing judged
    r = consistency.prefix_probe("x", complete_salted=salted(True), hits=lambda b: 0.0)
    assert r["verdict"] == "INCONCLUSIVE", r
    assert consistency.prefix_probe("x", complete_salted=salted(True), hits=lambda b: None)["verdict"] == \
        "NOT_APPLICABLE"
    full = consistency.run("x", probes=1, complete=fake_complete, score=fake_score, complete_salted=salted(True),
                           hits=lambda b: hits[0])
    assert full["verdict"] == "INCONSISTENT" and full["decode_verdict"] == "CONSISTENT"
    j = consistency.judge_against(full, dict(full, verdict="INCONSISTENT"))
    assert j["verdict"] == "INCONSISTENT" and j["why"][0].startswith("prefix cache")

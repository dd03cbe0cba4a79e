"""Server probes against fakes (no GPU): readiness verdicts from metrics, isolation and consistency against a
deterministic fake model, throughput bookkeeping, and the stack-change decision."""
import threading

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


def _metrics(checks, tokens, alarms=0, protected=1, ops=10, ops_checked=10, polls=3, started="1", line=6.0):
    return _client.parse_metrics(
        f"sdcguard_protected {protected}\nsdcguard_checks_total {checks}\nsdcguard_alarms_total {alarms}\n"
        f"sdcguard_ops_total {ops}\nsdcguard_ops_checked {ops_checked}\nsdcguard_alarm_line {line}\n"
        f"sdcguard_polls_total {polls}\nsdcguard_generated_tokens_total {tokens}\n"
        f'sdcguard_worker_info{{gpu="B200",uuid="u",pid="7",started="{started}"}} 1\n'
        f'sdcguard_stack_info{{model="tiny",precision="bf16",weights_digest="abc"}} 1\n')


def test_ready_verdicts():
    assert ready.judge(_metrics(10, 5), _metrics(20, 9))["verdict"] == "PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(10, 5))["verdict"] == "IDLE"
    assert ready.judge(_metrics(10, 5), _metrics(10, 9))["verdict"] == "NOT PROTECTED"      # tokens, no checks
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, alarms=1))["verdict"] == "FAULT FOUND"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, protected=0))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, line=1000))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, started="2"))["verdict"] == "NOT PROTECTED"
    assert ready.judge(_metrics(10, 5), _metrics(20, 9, ops_checked=8))["verdict"] == "NOT PROTECTED"
    assert ready.judge(None, _metrics(1, 1))["verdict"] == "NOT PROTECTED"
    dec = {"decision": "ACCEPT", "candidate_stack": {"model": "tiny", "precision": "fp8", "weights_digest": "abc"}}
    q = ready.qualified(_metrics(1, 1), dec)
    assert q["verdict"] == "NOT THE QUALIFIED STACK" and "precision" in q["why"][0]


def test_isolation_consistency_perf_on_fake_model():
    assert isolation.run("x", probes=2, primers=3, complete=fake_complete)["verdict"] == "NO LEAK SEEN"
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
    p = perf.run("x", clients=2, prompt=8, tokens=4, seconds=0.2, max_requests=10, complete=fake_complete)
    assert p["requests"] == 10 and p["errors"] == 0 and p["latency_ms"]["p50"] is not None


def _result(tps=100.0, alarms=0, iso="NO LEAK SEEN", cons="CONSISTENT", readyv="PROTECTED", checks=50):
    text = (f"sdcguard_protected 1\nsdcguard_checks_total {checks}\nsdcguard_alarms_total {alarms}\n"
            "sdcguard_ops_total 4\nsdcguard_ops_checked 4\n")
    return {"ready": {"verdict": readyv}, "perf": {"total_tokens_per_s": tps, "errors": 0},
            "isolation": {"verdict": iso, "probes": []}, "consistency": {"verdict": cons, "checks": 4},
            "metrics": text, "stack": {"model": "tiny"}}


def test_decide_sections():
    assert decide.decide(_result(), _result(95.0))["decision"] == "ACCEPT"
    d = decide.decide(_result(), _result(50.0))
    assert d["decision"] == "REJECT" and d["failed"] == ["performance"]
    assert decide.decide(_result(), _result(50.0), {"waive": ["performance"]})["decision"] == "ACCEPT"
    assert decide.decide(_result(), _result(alarms=2))["decision"] == "REJECT"
    assert decide.decide(_result(), _result(checks=0))["decision"] == "INCONCLUSIVE"
    assert decide.decide(_result(), _result(iso="LEAK"))["failed"] == ["isolation"]


def test_perf_measure_and_compare():
    m = perf.measure("x", rounds=3, warmup=0.05, clients=2, prompt=8, tokens=4, seconds=0.1, complete=fake_complete)
    assert len(m["rounds"]) == 3 and m["errors"] == 0 and m["spread"] is not None
    base = {"total_tokens_per_s": 100.0, "errors": 0, "spread": 0.01, "rounds": [1, 2],
            "latency_ms": {"p50": 10.0}}
    assert perf.compare(base, dict(base, total_tokens_per_s=110.0))["verdict"] == "FASTER"
    assert perf.compare(base, dict(base, total_tokens_per_s=101.0))["verdict"] == "SAME"
    assert perf.compare(base, dict(base, total_tokens_per_s=90.0))["verdict"] == "SLOWER"
    noisy = dict(base, spread=0.2)
    assert perf.compare(base, dict(noisy, total_tokens_per_s=110.0))["verdict"] == "SAME"
    assert perf.compare(base, dict(base, errors=1))["verdict"] == "INCONCLUSIVE"

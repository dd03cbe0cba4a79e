"""Prefill/decode disaggregation with checksummed KV transfer, and its coverage recording.

A producer engine prefills requests into its paged KV cache and publishes, per request, the page list, the first
generated token and a 64-bit checksum of every prompt page (`ops.kv_transfer.page_checksums`). A consumer engine
keeps a prefix cache of full 16-token pages; for each request it reuses the pages of the longest cached prefix,
pulls the rest straight from the producer GPU's memory with the hashing copy kernel (`ops.kv_transfer.pull_pages`),
compares every received page with the producer's checksum, then decodes.

Reused prefix pages are the gap the reference found in vLLM's KV checksum (src/sdcguard/kv_checksum_observer.py:33,
`CACHED_PREFIX_REASON`): they were checked once, when they first arrived, not for this request. Here
`verify_cached_prefix=True` closes it: the consumer re-hashes the reused pages and compares them with this
request's producer checksums, so the whole prompt is compared.

The run is recorded per request in the observer schema the gate reads (`sdcguard.checksum-observer.v1`
`recv_plan` and `verification` records, same fields), plus prefill-cache accounting and, when enabled, a
`cached_prefix_verification` record. `sdcguard_b200.coverage.own.gate` judges such a recording.

Placement: in one process (producer and consumer on the same GPU, or two GPUs of one process) or, for the 4+4
configuration, one process per GPU: prefill ranks 0..P-1 and decode ranks P..2P-1; each decode rank maps its
producer's cache through CUDA IPC (`torch.multiprocessing` reductions) and only this library's copy kernel reads it.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import time
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

from ..coverage import evidence as ev
from ..coverage import observer as obs
from ..ops import kv_transfer as kvx
from .engine import PAGE, LLMEngine

SOURCE_PROFILE = "sdcguard-b200-pd-kvpage.v1"
CALL_PATH = list(obs.CALL_PATH)


def _fingerprint(vals: Sequence[int]) -> int:
    """64-bit fingerprint of a checksum array (both sides compute it over the same uint64 values)."""
    h = hashlib.sha256(b"".join((v & 0xFFFFFFFFFFFFFFFF).to_bytes(8, "little") for v in vals)).digest()
    return int.from_bytes(h[:8], "little")


@dataclass
class Transfer:
    """What the producer publishes for one request."""
    request_id: str
    prompt_tokens: int
    token_ids: list
    pages: list              # producer page ids covering the prompt
    checksums: list          # uint64 per page
    first_token: int
    page_gens: Optional[list] = None   # lifetime generation of each producer page (when recorded)
    pool: str = "prefill"              # lifetime pool name of the producer's pages


@dataclass
class Recorder:
    """Records in the observer schema, in order, with one sequence counter."""
    records: list = field(default_factory=list)
    cache_records: list = field(default_factory=list)
    prefix_verifications: list = field(default_factory=list)
    seq: int = 0

    def _next(self) -> int:
        self.seq += 1
        return self.seq

    def _plan_fields(self, n, local, sent_count, start, fp, plan_seq) -> dict:
        group = {"attention_chunk_size": None, "block_count": sent_count - start, "block_size": PAGE,
                 "compare_called": False, "consumer_reports": [], "group_id": 0, "native_group_result": None,
                 "non_causal": False, "sent_block_size": PAGE, "sent_count": sent_count, "sent_dtype": "uint64",
                 "sent_fingerprint": fp, "sent_shape": [sent_count], "sent_start": 0, "sliding_window": None,
                 "spec_fields_recorded": True, "spec_source_supported": True, "spec_type": "FullAttentionSpec",
                 "start": start}
        return {"configured_group_count": 1, "configured_group_ids": [0], "expected_group_ids": [0],
                "expected_num_tokens": n, "expected_tp_size": 1, "groups": [group], "native_tp_size": 1,
                "num_local_computed_tokens": local, "num_tokens": n, "num_workers": 1,
                "parallel": {"dcp": 1, "dp": 1, "pcp": 1, "pp": 1, "tp": 1}, "plan_sequence": plan_seq,
                "planned_group_count": 1, "producer_payload_present": True, "source_supported": True,
                "speculative_disabled": True}

    def transfer(self, rid: str, n: int, local: int, sent: Sequence[int], mismatched: Sequence[int]) -> dict:
        """recv_plan + verification of one request; `mismatched` are chunk positions whose checksum differed."""
        total = len(sent)
        start = local // PAGE
        fp = _fingerprint(sent)
        plan_seq = self._next()
        plan = {"coverage": "unknown", "kind": "recv_plan", "native_result": "scheduled", "plan_sequence": plan_seq,
                "reason": "native_checksum_receive_scheduled", "request_id": rid, "sequence": self._next(),
                "load_plan": dict(self._plan_fields(n, local, total, start, fp, plan_seq), worker_ranks=[],
                                  worker_report_count=0)}
        update = self._next()
        proof = dict(self._plan_fields(n, local, total, start, fp, plan_seq), call_path=CALL_PATH, metadata_stable=True,
                     worker_ranks=[[0, 0]], worker_report_count=1)
        g = proof["groups"][0]
        g.update(compare_called=True, native_group_error=None, native_group_result=sorted(mismatched),
                 consumer_reports=[{"fingerprint": fp, "group_start": start, "pp_rank": 0, "record_pp_rank": 0,
                                    "record_tp_rank": 0, "replica_keys": [[1, 0]], "skipped": False, "tp_rank": 0,
                                    "value_dtype": "uint64", "value_shape": [total - start, 1]}])
        ok = not mismatched
        ver = {"kind": "verification", "request_id": rid, "origin_update_sequence": update, "native_return": ok,
               "groups": [{"group_id": 0, "native_result": "passed" if ok else "mismatch", "reason": None,
                           "returned_positions": sorted(mismatched)}],
               "proof": proof, "recording_complete": True, "recording_issue": None, "unverified_reasons": [],
               "engine_exception": None, "sequence": self._next()}
        d = obs.classify_verification(ver)
        for k in ("native_result", "coverage", "expected_units", "compared_units", "missing_units", "reason", "reasons",
                  "token_coverage"):
            ver[k] = d[k]
        self.records += [plan, ver]
        return ver

    def cache(self, role: str, rid: str, n: int, local_cached: int, external: int, output_tokens: int,
              prompt_sha256: str) -> None:
        self.cache_records.append({"request_id": rid, "role": role, "prompt_tokens": n, "prompt_sha256": prompt_sha256,
                                   "output_tokens": output_tokens, "preemptions": 0, "status": "FINISHED_LENGTH_CAPPED",
                                   "stats": {"num_prompt_tokens": n, "num_computed_tokens": n - local_cached - external,
                                             "num_cached_tokens": local_cached + external,
                                             "num_local_cached_tokens": local_cached,
                                             "num_external_cached_tokens": external}})

    def prefix_verified(self, rid: str, chunks: Sequence[int], mismatched: Sequence[int]) -> None:
        self.prefix_verifications.append({"kind": "cached_prefix_verification", "request_id": rid,
                                          "compared_units": [f"group:0:chunk:{c}" for c in chunks],
                                          "mismatched_units": [f"group:0:chunk:{c}" for c in mismatched],
                                          "native_result": "passed" if not mismatched else "mismatch"})


class PrefixCache:
    """Consumer-side prefix cache of full pages keyed by the token ids up to the end of the page."""

    def __init__(self):
        self.pages: dict[bytes, int] = {}
        self.owned: set[int] = set()       # pages held by the cache (never released with a request)

    @staticmethod
    def key(tokens: Sequence[int], upto: int) -> bytes:
        return hashlib.sha256(json.dumps(list(tokens[:upto])).encode()).digest()

    def lookup(self, tokens: Sequence[int]) -> list[int]:
        out = []
        for b in range(len(tokens) // PAGE):
            p = self.pages.get(self.key(tokens, (b + 1) * PAGE))
            if p is None:
                break
            out.append(p)
        # a request must transfer at least its last chunk (the consumer recomputes nothing)
        if out and len(out) * PAGE >= len(tokens):
            out.pop()
        return out

    def insert(self, tokens: Sequence[int], pages: Sequence[int]) -> None:
        for b in range(len(tokens) // PAGE):
            k = self.key(tokens, (b + 1) * PAGE)
            if k not in self.pages:
                self.pages[k] = pages[b]
                self.owned.add(pages[b])


def produce(engine: LLMEngine, requests: list[tuple[str, list]], seed: int = kvx.DEFAULT_SEED,
            sink=None, pool: str = "prefill") -> list[Transfer]:
    """Prefill on the producer; pages stay allocated until `release_producer`. sink: optional
    `lifetime.adapter.EventSink` that records the page lifetimes (pool "prefill")."""
    dev = engine.device
    plens = [len(t) for _, t in requests]
    maxlen = max(plens)
    vocab = engine.cfg.vocab
    if any(x < 0 or x >= vocab for _, t in requests for x in t):
        raise ValueError(f"token ids must lie in [0, {vocab})")
    prompts = torch.zeros(len(requests), maxlen, dtype=torch.long)
    for i, (_, t) in enumerate(requests):
        prompts[i, :len(t)] = torch.tensor(t)
    pages = [engine.alloc.alloc(-(-n // PAGE)) for n in plens]
    out = torch.zeros(len(requests), 1, dtype=torch.long, device=dev)
    engine.prefill(prompts.to(dev), plens, pages, out)
    gens = None
    if sink is not None:
        gens = []
        for (rid, _), pg, n in zip(requests, pages, plens):
            for p in pg:
                sink.alloc(pool, p, rid)
            sink.forward("prefill", rid, pool, pg, 0, n - 1)
            for p in pg:
                sink.local_write(pool, p, rid)
            gens.append([sink.gen[(pool, p)] for p in pg])
    flat = torch.tensor([p for pg in pages for p in pg], dtype=torch.int32, device=dev)
    sums = kvx.page_checksums(engine.cache, flat, seed).cpu().tolist()
    first = out[:, 0].cpu().tolist()
    res, o = [], 0
    for i, (rid, toks) in enumerate(requests):
        k = len(pages[i])
        res.append(Transfer(rid, plens[i], list(toks), pages[i], [s & 0xFFFFFFFFFFFFFFFF for s in sums[o:o + k]],
                            int(first[i]), None if gens is None else gens[i], pool))
        o += k
    return res


def release_producer(engine: LLMEngine, transfers: Sequence[Transfer], sink=None) -> None:
    for t in transfers:
        engine.alloc.release(t.pages)
        if sink is not None:
            for p in t.pages:
                sink.free(t.pool, p)


def consume(engine: LLMEngine, transfers: Sequence[Transfer], src_cache: torch.Tensor, prefix: PrefixCache,
            rec: Recorder, max_new_tokens: int, *, verify_cached_prefix: bool = False, seed: int = kvx.DEFAULT_SEED,
            corrupt: Optional[dict] = None, sink=None, stats: Optional[dict] = None) -> torch.Tensor:
    """Receive every request's KV pages (reusing cached prefix pages), check them, decode. Returns generated ids
    (N, max_new_tokens) on the host. `corrupt` = {request index: page index} flips one bit in that producer page
    before the pull (fault injection: the pulled page then mismatches its checksum); only for a producer cache in
    this process (a peer's memory is read by the copy kernel alone). `stats`, when given, accumulates the pulls'
    device time ("pull_ms", CUDA events around each pull launch) and the bytes they moved ("pull_bytes")."""
    dev = engine.device
    N = len(transfers)
    page_bytes = engine.cache[:, 0].numel() * engine.cache.element_size()     # one page over every layer
    local_pages, owned = [], []
    for i, t in enumerate(transfers):
        cached = prefix.lookup(t.token_ids)
        need = -(-(t.prompt_tokens + max_new_tokens) // PAGE) - len(cached)
        fresh = engine.alloc.alloc(need)
        owned.append(fresh)
        local_pages.append(cached + fresh)
        c = len(cached)
        if sink is not None:
            for p in fresh:
                sink.alloc("decode", p, t.request_id)
            for p in cached:
                sink.share("decode", p, t.request_id)
        total = len(t.pages)
        src = torch.tensor(t.pages[c:], dtype=torch.int32, device=dev)
        dst = torch.tensor(fresh[:total - c], dtype=torch.int32, device=dev)
        want = torch.tensor([v - (1 << 64) if v >= (1 << 63) else v for v in t.checksums[c:]], dtype=torch.int64,
                            device=dev)
        if corrupt and i in corrupt:
            pg = t.pages[corrupt[i]]
            flip_bit_in_page(src_cache, pg)
        if stats is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        _, res = kvx.pull_pages(src_cache, engine.cache, src, dst, want, seed)
        if stats is not None:
            e1.record()
        res = res.cpu().tolist()                   # waits for the pull
        if stats is not None:
            stats["pull_ms"] = stats.get("pull_ms", 0.0) + e0.elapsed_time(e1)
            stats["pull_bytes"] = stats.get("pull_bytes", 0) + src.numel() * page_bytes
            stats["pulls"] = stats.get("pulls", 0) + 1
        if sink is not None:
            for j, (sp, dp) in enumerate(zip(t.pages[c:], fresh[:total - c])):
                sink.transfer("read", "decode-pull", (t.pool, sp), ("decode", dp),
                              src_gen=t.page_gens[c + j] if t.page_gens else None)
        mism = [c + j for j, r in enumerate(res) if r != 1]
        rec.transfer(t.request_id, t.prompt_tokens, c * PAGE, t.checksums, mism)
        if verify_cached_prefix and c:
            got = kvx.page_checksums(engine.cache, torch.tensor(cached, dtype=torch.int32, device=dev), seed)
            got = [x & 0xFFFFFFFFFFFFFFFF for x in got.cpu().tolist()]
            bad = [j for j in range(c) if got[j] != t.checksums[j]]
            rec.prefix_verified(t.request_id, list(range(c)), bad)
        digest = ev.digest(ev.json_bytes(t.token_ids))
        rec.cache("decode", t.request_id, t.prompt_tokens, c * PAGE, t.prompt_tokens - c * PAGE, max_new_tokens, digest)
        if not mism:
            prefix.insert(t.token_ids, local_pages[-1][:t.prompt_tokens // PAGE])
    out = torch.zeros(N, max_new_tokens, dtype=torch.long, device=dev)
    out[:, 0] = torch.tensor([t.first_token for t in transfers], device=dev)
    if sink is not None:
        for t, pg in zip(transfers, local_pages):
            for p in pg[:len(t.pages)]:
                sink.consume("decode", p, t.request_id)
            sink.forward("decode", t.request_id, "decode", pg, t.prompt_tokens, t.prompt_tokens + max_new_tokens - 2)
    engine.decode_from([t.prompt_tokens for t in transfers], local_pages, out, max_new_tokens)
    host = out.cpu()
    for pg in owned:
        engine.alloc.release([p for p in pg if p not in prefix.owned])
        if sink is not None:
            for p in pg:
                if p not in prefix.owned:
                    sink.free("decode", p)
    return host


def flip_bit_in_page(cache: torch.Tensor, page: int, layer: int = 0, word: int = 3, bit: int = 5) -> None:
    """Flip one bit of one page (fault injection for tests: done with a torch op on a LOCAL tensor only)."""
    v = cache[layer, page].view(torch.int16).view(-1)
    v[word] ^= (1 << bit)


# ------------------------------------------------------------------------------------------ workload + recording
def pd_workload(groups: int = 8, per_group: int = 20, prefix_len: int = 1400, seed: int = 7, vocab: int = 151936):
    """Config 3: requests in groups sharing a random prefix, each with a unique suffix of 16-64 tokens."""
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for gi in range(groups):
        pre = torch.randint(0, vocab, (prefix_len,), generator=g).tolist()
        for r in range(per_group):
            suf = torch.randint(0, vocab, (int(torch.randint(16, 65, (1,), generator=g)),), generator=g).tolist()
            reqs.append((f"pd-{gi}-{r}", pre + suf))
    return reqs


def write_recording(out_dir: str, rec: Recorder, requests: list, meta: dict) -> None:
    os.makedirs(out_dir, exist_ok=True)
    plan = {**meta, "schema": "sdcguard_b200.pd-request-plan.v1", "engine": "sdcguard_b200",
            "source_profile": SOURCE_PROFILE,
            "requests": [{"request_id": rid, "prompt_tokens": len(t), "prompt_sha256": ev.digest(ev.json_bytes(t))}
                         for rid, t in requests]}
    snap = {"schema": obs.SCHEMA, "profile": SOURCE_PROFILE, "closed": True, "records": rec.records,
            "health": {"complete": True, "budget_exhausted": False, "errors": 0, "dropped_records": 0}}
    files = {"REQUEST_PLAN.json": plan, "OBSERVER.json": snap,
             "CACHE.json": {"schema": obs.CACHE_SCHEMA, "records": rec.cache_records},
             "CACHED_PREFIX_VERIFICATION.json": {"schema": "sdcguard_b200.cached-prefix-verification.v1",
                                                 "records": rec.prefix_verifications}}
    digests = {}
    for name, value in files.items():
        raw = ev.json_bytes(value)
        with open(os.path.join(out_dir, name), "wb") as f:
            f.write(raw)
        digests[name] = ev.digest(raw)
    with open(os.path.join(out_dir, "RESULT.json"), "wb") as f:
        f.write(ev.json_bytes({"schema": "sdcguard_b200.pd-result.v1", "files_sha256": digests, **meta}))


def run_single_process(out_dir: Optional[str], *, checked: bool = True, verify_cached_prefix: bool = False,
                       groups: int = 8, per_group: int = 20, new_tokens: int = 32, corrupt: Optional[dict] = None,
                       model_cfg=None, producer_device="cuda:0", consumer_device=None, sink=None) -> dict:
    """Producer and consumer engines in this process (same GPU, or two GPUs of this process)."""
    from ..models.decoder import QWEN3_0_6B
    cfg = model_cfg or QWEN3_0_6B
    consumer_device = consumer_device or producer_device
    reqs = pd_workload(groups, per_group, vocab=cfg.vocab)
    pages_needed = sum(-(-(len(t) + new_tokens) // PAGE) for _, t in reqs) + 64
    same = consumer_device == producer_device
    # one engine serving both roles holds the producer's and the consumer's copies of every page
    prod = LLMEngine(cfg, device=producer_device, checked=checked, num_blocks=pages_needed * (2 if same else 1),
                     max_num_seqs=len(reqs))
    cons = prod if same else LLMEngine(cfg, device=consumer_device, checked=checked,
                                                                     num_blocks=pages_needed, max_num_seqs=len(reqs),
                                                                     model=None)
    rec, prefix = Recorder(), PrefixCache()
    t0 = time.perf_counter()
    transfers = produce(prod, reqs, sink=sink)
    for t in transfers:
        rec.cache("prefill", t.request_id, t.prompt_tokens, 0, 0, 1, ev.digest(ev.json_bytes(t.token_ids)))
    out = consume(cons, transfers, prod.cache, prefix, rec, new_tokens, verify_cached_prefix=verify_cached_prefix,
                  corrupt=corrupt, sink=sink)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    release_producer(prod, transfers, sink=sink)
    meta = {"num_requests": len(reqs), "groups": groups, "new_tokens": new_tokens, "verify_cached_prefix": verify_cached_prefix,
            "wall_s": round(wall, 3)}
    if out_dir:
        write_recording(out_dir, rec, reqs, meta)
    return {"recorder": rec, "tokens": out, "meta": meta}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="sdcguard pd-record", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("out")
    ap.add_argument("--verify-cached-prefix", action="store_true")
    ap.add_argument("--groups", type=int, default=8)
    ap.add_argument("--per-group", type=int, default=20)
    ap.add_argument("--new-tokens", type=int, default=32)
    a = ap.parse_args(argv)
    r = run_single_process(a.out, verify_cached_prefix=a.verify_cached_prefix, groups=a.groups,
                           per_group=a.per_group, new_tokens=a.new_tokens)
    print(json.dumps(r["meta"]))
    return 0

"""Disaggregated prefill/decode across processes: P prefill ranks and D decode ranks, one process per GPU (torchrun),
KV pages pulled from the producer's GPU memory by the consumer's checksumming copy kernel over NVLink.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m sdcguard_b200.serve.pd_mp --prefill 4 --out rec/

Every rank allocates its KV cache from the symmetric heap (CUDA IPC), so a decode rank can map its producer's cache.
Requests are dealt round-robin to the prefill ranks; prefill rank p hands its requests to decode rank P + p mod D.
A producer prefills its requests, computes each page's checksum, waits for its kernels, and sends the request table
(ids, token ids, pages, checksums, first tokens) to its consumer over torch.distributed (control plane). The consumer
maps the producer's cache, pulls the pages with `kv_transfer.pull_pages` (peer loads, hashed on arrival and compared),
reuses cached prefix pages (optionally re-verified), decodes, and answers "done", after which the producer frees the
pages. Each decode rank writes its own recording (`OUT/decode<c>/`, the same files the single-process path writes),
which `sdcguard gate` judges, and its page-lifetime events (`OUT/decode<c>/lifetime.jsonl`).

Timing: the device time of the whole exchange on every rank (CUDA events, after a barrier), max over ranks.

Reference: the reference observes vLLM's NIXL transfer and its checksums (src/sdcguard/kv_checksum_observer.py); the
P/D layout on 4 + 4 GPUs is the plan's configuration.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from ..lifetime.adapter import EventSink
from ..models.decoder import CONFIGS
from ..parallel.symm import SymmetricHeap, _wrap
from . import pd
from .engine import PAGE, LLMEngine


def _max(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


NVLINK_GBS = 770.0          # measured peer copy on this pool's B200s, GB/s per direction per GPU


def _gate(d: str) -> dict:
    """The coverage gate's verdict on one decode rank's recording (`sdcguard gate D --require checksum`)."""
    from ..coverage import gate
    try:
        ans = gate.inspect(d, ["checksum"])
    except (ValueError, OSError, KeyError, TypeError, AttributeError) as e:
        return {"decision": "HOLD", "error": f"{type(e).__name__}: {str(e)[:200]}"}
    reasons = sorted({x for r in ans.get("requests", []) for x in r.get("reasons", [])} | set(ans.get("hold_reasons", [])))
    return {"decision": ans.get("decision"), "selected_requests": ans.get("selected_requests"),
            "passed_requests": ans.get("passed_requests"), "reasons": reasons[:8]}


def _pull_summary(rows: list) -> dict:
    """Bytes and device time of the decode ranks' KV pulls; bandwidth per decode rank as a fraction of NVLink."""
    per = [r["pull_bytes"] / (r["pull_ms"] * 1e6) for r in rows if r["pull_ms"] > 0]
    return {"bytes": sum(r["pull_bytes"] for r in rows), "launches": sum(r["pulls"] for r in rows),
            "device_ms_max": max((r["pull_ms"] for r in rows), default=0.0),
            "gbs_per_decode_rank": [round(x, 1) for x in per],
            "fraction_of_nvlink": round(min(per) / NVLINK_GBS, 3) if per else None,
            "nvlink_gbs": NVLINK_GBS, "timing": "CUDA events around each pull launch on the decode rank"}


def run(args) -> dict:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=args.pg_timeout))
    P = args.prefill
    D = world - P
    if P < 1 or D < 1:
        raise SystemExit("need at least one prefill and one decode rank")
    cfg = CONFIGS[args.model]
    reqs = pd.pd_workload(args.groups, args.per_group, vocab=cfg.vocab)
    mine = [r for i, r in enumerate(reqs) if i % P == rank] if rank < P else []
    pages_all = sum(-(-(len(t) + args.new_tokens) // PAGE) for _, t in reqs) + 64
    blocks = pages_all if rank >= P else sum(-(-len(t) // PAGE) for _, t in reqs) + 64
    blocks = max(blocks, pages_all)      # symmetric: every rank the same shape
    heap = SymmetricHeap(device=dev)
    shape = [cfg.layers, blocks, 2, cfg.kv_heads, PAGE, cfg.head_dim]
    buf = heap.alloc(shape, torch.bfloat16)
    buf.local.zero_()
    eng = LLMEngine(cfg, device=dev, checked=not args.unchecked, max_num_seqs=max(1, len(reqs)),
                    max_prefill_tokens=16384, cache=buf.local, max_model_len=2048 + args.new_tokens)
    sink = EventSink()
    rec = pd.Recorder()
    out_tokens = None
    rec_dir = None
    torch.cuda.synchronize(dev)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    if rank < P:
        transfers = pd.produce(eng, mine, sink=sink, pool=f"prefill{rank}")
        if args.corrupt_page is not None and transfers and rank == 0:
            pd.flip_bit_in_page(eng.cache, transfers[0].pages[args.corrupt_page % len(transfers[0].pages)])
        torch.cuda.synchronize(dev)        # every page written before the consumer reads it
        dst = P + rank % D
        dist.send_object_list([[t.__dict__ for t in transfers], list(sink.events)], dst=dst)
        ack = [None]
        dist.recv_object_list(ack, src=dst)
        pd.release_producer(eng, transfers, sink=sink)
    else:
        c = rank - P
        prefix = pd.PrefixCache()
        pull = {}
        outs = []
        served = []
        for p in range(P):
            if p % D != c:
                continue
            box = [None, None]
            dist.recv_object_list(box, src=p)
            transfers = [pd.Transfer(**d) for d in box[0]]
            sink.ingest(box[1])                # the producer's page allocations precede the pulls
            src_view = _wrap(buf.addr[p], shape, torch.bfloat16, dev)
            outs.append(pd.consume(eng, transfers, src_view, prefix, rec, args.new_tokens,
                                   verify_cached_prefix=args.verify_cached_prefix, sink=sink, stats=pull))
            served += [(t.request_id, t.token_ids) for t in transfers]
            dist.send_object_list(["done"], dst=p)
        out_tokens = torch.cat(outs) if outs else None
        if args.out:
            d = os.path.join(args.out, f"decode{c}")
            pd.write_recording(d, rec, served, {"num_requests": len(served), "prefill_ranks": P, "decode_ranks": D,
                                                "verify_cached_prefix": args.verify_cached_prefix})
            with open(os.path.join(d, "lifetime.jsonl"), "w") as f:
                f.writelines(json.dumps(e) + "\n" for e in sink.events)
            rec_dir = d
    b.record()
    torch.cuda.synchronize(dev)
    dev_ms = _max(a.elapsed_time(b), dev)
    wall_ms = _max((time.perf_counter() - t0) * 1e3, dev)
    from ..lifetime import adapter
    viol = len(adapter.check(sink.events)["violations"])
    tot_viol = int(_max(float(viol), dev))
    mism = sum(1 for r in rec.records if r.get("kind") == "verification" and r.get("native_result") == "mismatch")
    tot_mism = int(_max(float(mism), dev))
    tokens = sum(len(t) + args.new_tokens for _, t in reqs)
    # per decode rank: the KV pulls' bytes and device time, and the gate's verdict on its recording
    mine_row = None
    if rank >= P:
        mine_row = {"rank": rank, "pull_bytes": pull.get("pull_bytes", 0), "pull_ms": round(pull.get("pull_ms", 0.0), 3),
                    "pulls": pull.get("pulls", 0), "gate": _gate(rec_dir) if rec_dir else None}
    rows = [None] * world
    dist.all_gather_object(rows, mine_row)
    rows = [r for r in rows if r is not None]
    res = {"world": world, "prefill_ranks": P, "decode_ranks": D, "requests": len(reqs), "device_ms": round(dev_ms, 2),
           "wall_ms": round(wall_ms, 2), "tokens_per_s": round(tokens / (dev_ms / 1e3), 1),
           "lifetime_violations": tot_viol, "ranks_with_mismatch": tot_mism, "model": cfg.name,
           "checked": not args.unchecked, "kv_pull": _pull_summary(rows),
           "gate": [dict(r["gate"], decode_rank=r["rank"]) for r in rows if r.get("gate")] or None}
    dist.barrier()
    del eng
    heap.close()
    return res if rank == 0 else {}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sdcguard_b200.serve.pd_mp")
    ap.add_argument("--prefill", type=int, default=4)
    ap.add_argument("--model", default="Qwen3-0.6B")
    ap.add_argument("--groups", type=int, default=8)
    ap.add_argument("--per-group", type=int, default=20)
    ap.add_argument("--new-tokens", type=int, default=32)
    ap.add_argument("--out")
    ap.add_argument("--verify-cached-prefix", action="store_true")
    ap.add_argument("--unchecked", action="store_true")
    ap.add_argument("--corrupt-page", type=int, default=None, help="flip a bit in a producer page (rank 0)")
    ap.add_argument("--pg-timeout", type=int, default=120)
    a = ap.parse_args(argv)
    r = run(a)
    if r:
        print(json.dumps(r), flush=True)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

"""Recorded-engine source profiles: the two pinned checksum-capable vLLM revisions whose recordings the coverage
gate accepts, with the file hashes their recorders were bound to.

`data/checksum-builds.json` is the reference's pin table (src/sdcguard/case_data/checksum-builds.json) kept byte
for byte: recordings name those revisions and hashes, so the table must be the same to validate them. Profiles
for this package's own engine (sdcguard_b200.serve) are in `own_profile()`.
"""
from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

BASELINE = "29d2f4e03740acb14439ce22d24b06d8095d17d3"
CANDIDATE = "1a0c6954a9d881c81f85fc1a6cbf51c76f3fcba8"
REVISIONS = (BASELINE, CANDIDATE)

OBSERVER_PROFILE = "vllm-checksum-62211-full-load-tp1-pp1.v1"
CLIENT_PROFILE = "vllm-checksum-62211-client-join.v1"
BINDING_PROFILE = "vllm-checksum-62211-request-id.v1"


@lru_cache(maxsize=1)
def _table() -> dict:
    return json.loads((Path(__file__).with_name("data") / "checksum-builds.json").read_bytes())


def supported(revision) -> bool:
    return type(revision) is str and revision in REVISIONS


def get(revision: str = BASELINE) -> dict:
    if not supported(revision):
        raise ValueError("unsupported checksum engine revision")
    v = _table()[revision]
    if v["revision"] != revision:
        raise ValueError("checksum profile identity differs")
    return v


def startup_supported(value, revision) -> bool:
    """The candidate revision adds a scheduler branch that a recording must show unused."""
    if not supported(revision) or type(value) is not dict:
        return False
    if revision == BASELINE:
        return True
    return ("hisparse_host_num_blocks" in value and value["hisparse_host_num_blocks"] is None
            and value.get("defer_async_loads") is False)


def observer_source(revision: str = BASELINE) -> dict:
    pins = get(revision)["checksum_pins"]
    return {"profile": OBSERVER_PROFILE, "revision": revision,
            "files": {name: receipt["sha256"] for name, receipt in pins["files"].items()}}


def client_source(revision: str = BASELINE) -> dict:
    return {"profile": CLIENT_PROFILE, "revision": revision, "api_request_id_files": get(revision)["binding_files"],
            "checksum_profile": observer_source(revision)}


def cache_source(revision: str = BASELINE) -> dict:
    p = get(revision)
    return {"profile": p["prefix_profile"], "revision": revision, "files": p["prefix_files"]}


def own_profile() -> dict:
    """Identity this package's serving engine writes into its own recordings (sdcguard_b200.serve.pd)."""
    from .. import __version__
    return {"engine": "sdcguard_b200", "version": __version__, "kv_page_tokens": 16,
            "checksum": "kvpage-fmix64-v1"}

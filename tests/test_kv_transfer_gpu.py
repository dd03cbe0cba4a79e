"""Checksummed KV-page transfer on the GPU: checksums equal the NumPy definition, pulled pages equal their source,
a flipped bit in a source page is detected at its page, and an end-to-end prefill/decode run is judged by the gate
(HOLD for reused prefix pages, PASS once they are re-verified)."""
import contextlib
import io

import pytest
import torch

from sdcguard_b200.ops import kv_transfer as kvx

pytestmark = pytest.mark.gpu


def _cache(blocks=24, layers=3, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(layers, blocks, 2, 2, 16, 128, device="cuda", generator=g)).bfloat16()


def test_page_checksums_match_reference():
    c = _cache()
    pages = torch.tensor([0, 5, 23], dtype=torch.int32, device="cuda")
    got = [x & 0xFFFFFFFFFFFFFFFF for x in kvx.page_checksums(c, pages).tolist()]
    want = [kvx.page_checksum_reference(c, p) for p in (0, 5, 23)]
    assert got == want


def test_pull_copies_and_flags_flipped_page():
    src, dst = _cache(seed=1), torch.zeros(3, 24, 2, 2, 16, 128, device="cuda", dtype=torch.bfloat16)
    sp = torch.tensor([3, 4, 9, 10], dtype=torch.int32, device="cuda")
    dp = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    want = kvx.page_checksums(src, sp)
    st = torch.zeros(4, dtype=torch.int64, device="cuda")
    got, res = kvx.pull_pages(src, dst, sp, dp, want, state_row=st)
    torch.cuda.synchronize()
    assert res.tolist() == [1, 1, 1, 1] and torch.equal(got, want)
    assert torch.equal(dst[:, :4], src[:, [3, 4, 9, 10]])
    assert st[0].item() == 0 and st[2].item() == 1
    src.view(torch.int16)[2, 9, 1, 1, 7, 100] ^= 1 << 3        # one bit, layer 2 of page 9
    got, res = kvx.pull_pages(src, dst, sp, dp, want, state_row=st)
    torch.cuda.synchronize()
    assert res.tolist() == [1, 1, 2, 1]
    assert (st[0].item() >> 32) == 0x7F800000 and (st[0].item() & 0xFFFFFFFF) == 2


def test_pd_end_to_end_gate(tmp_path):
    from sdcguard_b200 import cli
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve import pd

    def gate(p):
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            rc = cli.main(["gate", str(p), "--require", "checksum"])
        return rc, buf.getvalue()
    r1 = pd.run_single_process(str(tmp_path / "plain"), groups=2, per_group=3, new_tokens=4, model_cfg=TINY)
    rc, out = gate(tmp_path / "plain")
    assert rc == 2 and "2 / 6 selected requests passed" in out and "cached prefix not covered by checksum" in out
    r2 = pd.run_single_process(str(tmp_path / "verified"), groups=2, per_group=3, new_tokens=4, model_cfg=TINY,
                               verify_cached_prefix=True)
    rc, out = gate(tmp_path / "verified")
    assert rc == 0 and "6 / 6 selected requests passed" in out
    assert torch.equal(r1["tokens"], r2["tokens"])
    r3 = pd.run_single_process(str(tmp_path / "bad"), groups=2, per_group=3, new_tokens=4, model_cfg=TINY,
                               verify_cached_prefix=True, corrupt={4: 88})
    rc, out = gate(tmp_path / "bad")
    assert rc == 2 and "native_checksum_mismatch" in out


def test_pd_page_lifetimes_obey_the_ledger_rules():
    """The P/D path's recorded page lifetimes (producer pages, pulls, shared prefix pages, consumes, frees) replayed
    through the lifetime ledger: no rule broken."""
    from sdcguard_b200.lifetime import adapter
    from sdcguard_b200.models.decoder import TINY
    from sdcguard_b200.serve import pd
    sink = adapter.EventSink()
    pd.run_single_process(None, groups=2, per_group=3, new_tokens=4, model_cfg=TINY, sink=sink)
    r = adapter.check(sink.events)
    kinds = {e["ev"] for e in sink.events}
    assert {"alloc", "submit", "complete", "consume", "share", "free"} <= kinds, kinds
    assert r["violations"] == [], r["violations"][:3]

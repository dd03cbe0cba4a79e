"""The fingerprint kernel against its NumPy restatement, on buffers of odd sizes and alignments; the weight scan
on GPU weights."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fingerprint_kernel_matches_host():
    from sdcguard_b200.ops.fingerprint import fingerprint, fingerprint_host
    g = torch.Generator().manual_seed(0)
    base = torch.randint(0, 256, (3 * 1024 * 1024 + 13,), dtype=torch.uint8, generator=g)
    dev = base.cuda()
    ts = [dev, dev[1:1000], dev[16:16 + 4096], dev[:7], torch.randn(1000, 333, device="cuda").bfloat16()]
    got = fingerprint(ts, seed=5).cpu().tolist()
    for t, (a, b) in zip(ts, got):
        ha, hb = fingerprint_host(t.cpu(), seed=5)
        assert (a & (2 ** 64 - 1), b & (2 ** 64 - 1)) == (ha, hb)


def test_weight_scan_on_gpu_weights():
    from sdcguard_b200.serve.weights import WeightScan
    from sdcguard_b200.utils.inject import flip_bit_
    ws = [torch.randn(512, 256, device="cuda").bfloat16() for _ in range(4)]
    scan = WeightScan([(f"w{i}", w) for i, w in enumerate(ws)], keep_host_copy=True)
    assert scan.full() == []
    flip_bit_(ws[2], 1000, 14)
    ev = scan.full()
    assert len(ev) == 1 and ev[0].detail["weight"] == "w2" and ev[0].detail["repaired"]
    assert scan.full() == []

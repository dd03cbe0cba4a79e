"""CPU: the chunked weight init of the tensor-parallel decoder builds the same global model at every TP size
(rank shards of TP=2 reassemble TP=1's weights in the column/row-parallel layouts)."""
import torch

from sdcguard_b200.models.decoder import TINY
from sdcguard_b200.models.tp_decoder import TPDecoder


def _m(rank, world):
    return TPDecoder(TINY, None, rank, world, "cpu", checked=False, collective="nccl", max_rows=64, seed=7)


def test_tp2_shards_reassemble_tp1():
    full, r0, r1 = _m(0, 1), _m(0, 2), _m(1, 2)
    d, qh = 128, TINY.heads // 2
    for i in range(TINY.layers):
        f, a, b = full.layers[i], r0.layers[i], r1.layers[i]
        nq_l = qh
        # qkv: [q of rank 0, q of rank 1 | k0, k1 | v0, v1]
        q = torch.cat([a.qkv[:nq_l * d], b.qkv[:nq_l * d]])
        k = torch.cat([a.qkv[nq_l * d:(nq_l + 1) * d], b.qkv[nq_l * d:(nq_l + 1) * d]])
        v = torch.cat([a.qkv[(nq_l + 1) * d:], b.qkv[(nq_l + 1) * d:]])
        assert torch.equal(f.qkv, torch.cat([q, k, v]))
        assert torch.equal(f.o, torch.cat([a.o, b.o], dim=1))
        ih = TINY.intermediate // 2
        g = torch.cat([a.gate_up[:ih], b.gate_up[:ih]])
        u = torch.cat([a.gate_up[ih:], b.gate_up[ih:]])
        assert torch.equal(f.gate_up, torch.cat([g, u]))
        assert torch.equal(f.down, torch.cat([a.down, b.down], dim=1))
    assert torch.equal(full.lm_head, torch.cat([r0.lm_head, r1.lm_head]))
    assert torch.equal(full.embed, r0.embed) and torch.equal(full.embed, r1.embed)

"""ABFT numerics shared by every checked GEMM path: the sign pattern of the signed checksum, the checksum rows
of a weight matrix, the fp32-accumulator noise model, the encoding of scores into the per-layer state row, and
plain-PyTorch reference implementations used as test oracles and as the CPU path.

The identity (reference: src/sdcguard/checksum.py:1-54): for C = A @ W^T (+ bias) and every block of 128
consecutive output columns b,

    sum_{j in b} C[i, j]        = A[i, :] . (sum_{j in b} W[j, :])          (+ sum_{j in b} bias[j])
    sum_{j in b} s_j C[i, j]    = A[i, :] . (sum_{j in b} s_j W[j, :])      (+ sum_{j in b} s_j bias[j])

with fixed pseudo-random signs s_j = +-1, so errors that cancel in the plain sum still show in the signed one.

Noise model of a check made on the fp32 accumulator (reference: checksum.py:536-560, `_acc_zscores`):

    den = u * (c1 sqrt(k) ||a_i||_2 W_b  +  (c2 sqrt(k) + c3 k / nfma + sqrt(128)) ||C_ib||_2)  + abs_floor

where W_b is the largest of ||W_b||_F and the 2-norms of the plain and signed block sums (the expected side is
itself an fp32 tensor-core accumulation of A against those sums), u = 2^-24. z = |expected - actual| / den;
the plain sum must also exceed the same bound with ||C_ib||_1 in place of ||C_ib||_2 (errors that line up).
An alarm is z > 6. Non-finite outputs are corruption when the inputs cannot produce them
(sqrt(k) ||a_i||_2 max|W_b| + max|bias| < 1e18), otherwise the block is not judged.

The checksum rows of W: six bf16 rows per block, the plain block sum split into three bf16 parts whose sum
carries about 24 significant bits (hi = bf16(v), mid = bf16(v - hi), lo = bf16(v - hi - mid)), then the
signed block sum the same way (reference: checksum.py:160 `_split3`). The GEMM kernels compute A @ Wc^T as
extra output tiles and add the parts in fp32.
"""
from __future__ import annotations

import math
import os
import struct
from dataclasses import dataclass
from typing import Optional

import torch

BLOCK = 128
CS_ROWS = 6
ACC_UNIT = 2.0 ** -24
ABS_FLOOR = 1e-20
Z_ALARM = 6.0
BIG = 1e18

# Coefficients of the fp32-accumulator model on B200 tcgen05 (bf16 inputs, fp32 accumulation). Chosen from the
# rounding argument (an fp32 running sum loses up to one ulp per step; the standard deviation is about 0.58 ulp)
# with margin, then checked against clean runs on B200 (tools/calibrate.py). C3 covers the tensor cores'
# truncating accumulation: each step of NFMA products drops bits toward zero, and when the partial sums keep one
# sign (structured activations, a softmax gradient against position-correlated features) those errors add up
# linearly in K instead of as a random walk. Without it, GPT-2 training's LM-head dW GEMM (K = 16384 tokens) scored
# up to z = 8 on clean data; with C3 = 1 the term is k / 16 ulps of the block's output norm.
C1 = 1.0
C2 = 1.0
C3 = 1.0
NFMA = 16

# State row of one checked layer (same layout as src/sdcguard/serve.py:55-65):
#   0: (bits of worst z << 32) | flat index of that checksum  (flat = (row * nb + block) * 2 + signed)
#   1: (bits of worst z << 32) | bits of its noise
#   2: checks executed (kernel launches)
#   3: checksums that could not be judged
STATE_COLS = 4
COL_CHECKS, COL_UNJUDGED = 2, 3


def _seed_from_env() -> int:
    s = os.environ.get("SDCGUARD_SIGN_SEED")
    return int(s) if s else int.from_bytes(os.urandom(4), "little")


_SIGN_SEED = _seed_from_env()


def sign_mask(seed: Optional[int] = None) -> tuple[int, int, int, int]:
    """Four 32-bit words: bit j (word j // 32) set means column j of every block counts with sign -1.
    A splitmix64 stream of the seed, so every process (or replica) can pick its own pattern."""
    x = (_SIGN_SEED if seed is None else int(seed)) & 0xFFFFFFFFFFFFFFFF
    words = []
    for _ in range(2):
        x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = x
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        z ^= z >> 31
        words += [z & 0xFFFFFFFF, z >> 32]
    return tuple(words)  # type: ignore[return-value]


def sign_vector(mask: tuple[int, int, int, int], dtype=torch.float64, device="cpu") -> torch.Tensor:
    bits = [((mask[j // 32] >> (j % 32)) & 1) for j in range(BLOCK)]
    return torch.tensor([-1.0 if b else 1.0 for b in bits], dtype=dtype, device=device)


def split3(v: torch.Tensor) -> torch.Tensor:
    """(..., k) float64 -> (..., 3, k) bf16 parts hi, mid, lo with hi + mid + lo ~ v to ~2^-24 relative."""
    hi = v.to(torch.bfloat16)
    r = v - hi.double()
    mid = r.to(torch.bfloat16)
    lo = (r - mid.double()).to(torch.bfloat16)
    return torch.stack([hi, mid, lo], dim=-2)


@dataclass
class WeightChecksums:
    """Per-layer static data of a checked linear layer y = x @ W^T + b (computed once at load)."""
    n: int
    k: int
    nb: int
    wc: torch.Tensor        # (6 nb, k) bf16 checksum rows
    wstat: torch.Tensor     # (nb, 4) fp32: ||W_b||_F, ||plain||_2, ||signed||_2, max|W_b|
    bsum: Optional[torch.Tensor]   # (nb, 2) fp32 plain/signed block sums of the bias
    bias_max: float
    mask: tuple


def weight_checksums(weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     mask: Optional[tuple] = None) -> WeightChecksums:
    """Checksum rows and block statistics of W (n, k), in float64 on W's device."""
    mask = mask or sign_mask()
    n, k = weight.shape
    nb = -(-n // BLOCK)
    w64 = torch.zeros(nb * BLOCK, k, dtype=torch.float64, device=weight.device)
    w64[:n] = weight.detach().double()
    blocks = w64.view(nb, BLOCK, k)
    s = sign_vector(mask, device=weight.device)
    plain = blocks.sum(1)
    signed = (blocks * s.view(1, BLOCK, 1)).sum(1)
    wc = torch.cat([split3(plain), split3(signed)], dim=1).reshape(nb * CS_ROWS, k).contiguous()
    wstat = torch.stack([
        torch.linalg.vector_norm(blocks, dim=(1, 2)),
        torch.linalg.vector_norm(plain, dim=1),
        torch.linalg.vector_norm(signed, dim=1),
        blocks.abs().amax(dim=(1, 2)),
    ], dim=1).float().contiguous()
    bsum, bias_max = None, 0.0
    if bias is not None:
        b64 = torch.zeros(nb * BLOCK, dtype=torch.float64, device=weight.device)
        b64[:n] = bias.detach().double()
        bb = b64.view(nb, BLOCK)
        bsum = torch.stack([bb.sum(1), (bb * s.view(1, BLOCK)).sum(1)], dim=1).float().contiguous()
        bias_max = float(bias.detach().abs().max()) if n else 0.0
    return WeightChecksums(n=n, k=k, nb=nb, wc=wc, wstat=wstat, bsum=bsum, bias_max=bias_max, mask=mask)


def coefficients(k: int, c1: float = C1, c2: float = C2, c3: float = C3, nfma: int = NFMA) -> tuple[float, float]:
    """(prod_coef, out_coef) of the noise model for inner dimension k."""
    sk = math.sqrt(k)
    prod = c1 * sk * ACC_UNIT
    out = (c2 * sk + (c3 * k / nfma if nfma else 0.0) + math.sqrt(BLOCK)) * ACC_UNIT
    return prod, out


def block_stats(acc: torch.Tensor, mask: tuple) -> torch.Tensor:
    """(m, n) fp32 accumulator -> (m, nb, 4) float64: plain, signed, sum of squares, sum of |c|."""
    m, n = acc.shape
    nb = -(-n // BLOCK)
    c = torch.zeros(m, nb * BLOCK, dtype=torch.float64, device=acc.device)
    c[:, :n] = acc.double()
    c = c.view(m, nb, BLOCK)
    s = sign_vector(mask, device=acc.device).view(1, 1, BLOCK)
    return torch.stack([c.sum(-1), (c * s).sum(-1), (c * c).sum(-1), c.abs().sum(-1)], dim=-1)


def expected_sums(x: torch.Tensor, cs: WeightChecksums) -> torch.Tensor:
    """(m, nb, 2) float64 expected plain and signed sums, from the bf16 checksum rows (as the kernel sees them)."""
    e = x.double() @ cs.wc.double().t()                      # (m, 6 nb)
    e = e.view(x.shape[0], cs.nb, 2, 3).sum(-1)
    if cs.bsum is not None:
        e = e + cs.bsum.double().view(1, cs.nb, 2)
    return e


def zscores(x: torch.Tensor, cs: WeightChecksums, stats: torch.Tensor, expected: torch.Tensor,
            z_alarm: float = Z_ALARM, c1: float = C1, c2: float = C2, c3: float = C3) -> torch.Tensor:
    """(m, nb, 2) scores (plain, signed) under the model above; inf = corruption, -1 = not judged.
    The same formula the kernels evaluate on the device."""
    prod_coef, out_coef = coefficients(cs.k, c1, c2, c3)
    xn = torch.linalg.vector_norm(x.double(), dim=1).view(-1, 1)
    wmax = cs.wstat[:, :3].double().amax(1).view(1, -1)
    prod = prod_coef * xn * wmax
    den = stats[..., 2].sqrt() * out_coef + prod + ABS_FLOOR
    worst = stats[..., 3] * out_coef + prod + ABS_FLOOR
    dp = (expected[..., 0] - stats[..., 0]).abs()
    ds = (expected[..., 1] - stats[..., 1]).abs()
    zp = torch.minimum(dp / den, dp / worst * z_alarm)
    zs = ds / den
    z = torch.stack([zp, zs], dim=-1)
    fin_act = torch.isfinite(stats).all(-1, keepdim=True)
    fin_exp = torch.isfinite(expected).all(-1, keepdim=True)
    bound = math.sqrt(cs.k) * xn * cs.wstat[:, 3].double().view(1, -1) + cs.bias_max
    bad = (~fin_act) & fin_exp
    z = torch.where(bad & (bound < BIG).unsqueeze(-1), torch.full_like(z, math.inf), z)
    z = torch.where((bad & ~(bound < BIG).unsqueeze(-1)) | ~fin_exp, torch.full_like(z, -1.0), z)
    return z


def reference_check(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                    cs: Optional[WeightChecksums] = None, acc: Optional[torch.Tensor] = None) -> dict:
    """Plain-PyTorch check of y = x @ W^T + b computed in fp32 (or of a given fp32 accumulator `acc`).
    Returns worst score, its location and the per-block scores."""
    cs = cs or weight_checksums(weight, bias)
    if acc is None:
        acc = x.float() @ weight.float().t()
        if bias is not None:
            acc = acc + bias.float()
    st = block_stats(acc, cs.mask)
    ex = expected_sums(x, cs)
    z = zscores(x, cs, st, ex)
    flat = int(torch.argmax(z.reshape(-1)))
    worst = float(z.reshape(-1)[flat])
    row, rem = divmod(flat, cs.nb * 2)
    block, which = divmod(rem, 2)
    return {"z": worst, "row": row, "block": block, "signed": bool(which), "scores": z,
            "unjudged": int((z < 0).sum())}


def decode_state_row(row) -> dict:
    """Decode one state row (4 int64) into worst z, location, noise and counts."""
    k0, k1, checks, unj = (int(v) & 0xFFFFFFFFFFFFFFFF for v in row)
    zbits = k0 >> 32
    z = struct.unpack("<f", struct.pack("<I", zbits))[0] if k0 else 0.0
    flat = k0 & 0xFFFFFFFF
    noise = struct.unpack("<f", struct.pack("<I", k1 & 0xFFFFFFFF))[0] if k1 else 0.0
    return {"z": z, "flat": flat, "noise": noise, "checks": checks, "unjudged": unj}


def locate(flat: int, nb: int) -> tuple[int, int, bool]:
    """flat checksum index -> (row, block, signed)."""
    row, rem = divmod(flat, nb * 2)
    block, which = divmod(rem, 2)
    return row, block, bool(which)


def product_zscores(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, mask: tuple,
                    rnd_unit: float = 0.0, judged: Optional[torch.Tensor] = None,
                    z_alarm: float = Z_ALARM, return_den: bool = False):
    """Scores of batched products c ~ a @ b made by another library (cuBLAS, CPU BLAS), in float64 torch ops:
    a (G, m, k), b (G, k, n), c (G, m, n) the product as the library returned it (already freed of any bias,
    alpha and beta). Returns (G, m, nb) scores, the larger of plain and signed; inf = corruption, -1 = not judged.

    The noise model is the accumulator model above with b's blocks in place of W's (the plain and signed block
    sums of b are formed here in float64, so the expected side adds only its own float64 rounding). When c was
    rounded to a narrower type (rnd_unit = its unit roundoff, 2^-8 for bf16), each element may differ from the
    accumulator by up to rnd_unit |c| with a sign that varies from element to element: the statistical bound grows by
    rnd_unit ||c_b||_2 and the worst-case bound of the plain sum by 1.25 rnd_unit ||c_b||_1. judged: optional (G, m, nb) bool,
    False where the inputs themselves hold non-finite values (a product block that is then not scored). With
    return_den, also the (G, m, nb) noise scale each score divides by.
    Reference: src/sdcguard/checksum.py (`matmul_zscores` on the rounded output, `matmul_zscores_acc` on the
    accumulator)."""
    G, m, k = a.shape
    n = b.shape[-1]
    nb = -(-n // BLOCK)
    pad = nb * BLOCK - n
    s = sign_vector(mask, device=a.device)
    bb = torch.nn.functional.pad(b.double(), (0, pad)).view(G, k, nb, BLOCK)
    plain = bb.sum(-1)
    signed = (bb * s).sum(-1)                                                  # (G, k, nb)
    wmax = torch.stack([bb.square().sum((1, 3)).sqrt(), torch.linalg.vector_norm(plain, dim=1),
                        torch.linalg.vector_norm(signed, dim=1)], -1).amax(-1)       # (G, nb)
    babs = bb.abs().amax((1, 3))                                               # (G, nb)
    del bb
    a64 = a.double()
    exp = torch.bmm(a64, torch.cat([plain, signed], -1)).view(G, m, 2, nb)
    cc = torch.nn.functional.pad(c.double(), (0, pad)).view(G, m, nb, BLOCK)
    sp, ssg = cc.sum(-1), (cc * s).sum(-1)
    l2, l1 = cc.square().sum(-1).sqrt(), cc.abs().sum(-1)
    fin_act = torch.isfinite(cc).all(-1)
    del cc
    prod_coef, out_coef = coefficients(k)
    xn = torch.linalg.vector_norm(a64, dim=2).unsqueeze(-1)                  # (G, m, 1)
    prod = prod_coef * xn * wmax.unsqueeze(1)
    den = l2 * (out_coef + rnd_unit) + prod + ABS_FLOOR
    worst = l1 * (out_coef + 1.25 * rnd_unit) + prod + ABS_FLOOR
    dp = (exp[:, :, 0] - sp).abs()
    ds = (exp[:, :, 1] - ssg).abs()
    z = torch.maximum(torch.minimum(dp / den, dp / worst * z_alarm), ds / den)
    fin_exp = torch.isfinite(exp).all(2)
    bound = math.sqrt(k) * xn * babs.unsqueeze(1)
    ok = torch.isfinite(a64).all(-1, keepdim=True) & torch.isfinite(babs).unsqueeze(1)
    if judged is not None:
        ok = ok & judged
    bad = ~fin_act & fin_exp & ok
    z = torch.where(bad & (bound < BIG), torch.full_like(z, math.inf), z)
    z = torch.where((bad & ~(bound < BIG)) | ~fin_exp | ~ok, torch.full_like(z, -1.0), z)
    z = torch.where(torch.isnan(z), torch.full_like(z, -1.0), z)
    return (z, den) if return_den else z

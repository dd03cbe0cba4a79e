"""Check a product another library already computed: C = beta bias + alpha (A @ B), answered at once.

    r = check_matmul(A, B, C)                  # A (m, k) or (G, m, k); B (k, n) or (G, k, n); C like A @ B
    r = check_linear(x, weight, bias, y)       # y = F.linear(x, weight, bias), any leading dimensions
    r.ok, r.max_z, r.row, r.col_block, r.noise, r.judged

The plain and +-1-signed sums of every 128-column block of every row of C are compared with the same sums computed
from A and B's block sums in float64 (`numerics.abft.product_zscores`), in units of the block's rounding noise:
the fp32-accumulator model of the checked GEMM plus the output's own rounding (bf16 2^-8, fp16 2^-11). `ok` is
False when a block's score is above the line (z, default 6) or the output holds a value its inputs cannot produce
(score inf); a block whose inputs are not finite is not judged (score -1), and `judged` is False when no block
could be. For this library's own GEMMs the check runs inside the kernel instead (`ops.gemm.checked_linear`).

Reference: src/sdcguard/checksum.py:107-122 (`CheckResult`), `check_matmul` :728, `check_linear` :763.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import abft

ROUND = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}


@dataclass
class CheckResult:
    ok: bool                        # False: looks corrupted
    max_z: float                    # worst score (inf: a value the inputs cannot produce; -1: nothing judged)
    nonfinite: bool                 # the output holds NaN or inf where the inputs are finite
    batch: Optional[int] = None     # where the worst block is (batched products)
    row: Optional[int] = None
    col_block: Optional[int] = None
    noise: Optional[float] = None   # the noise scale of that block

    @property
    def judged(self) -> bool:
        """False when no checksum could be judged (non-finite inputs, or an overflow the inputs allow)."""
        return not (math.isfinite(self.max_z) and self.max_z < 0)


def check_matmul(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
                 alpha: float = 1.0, beta: float = 1.0, z: float = abft.Z_ALARM,
                 seed: Optional[int] = None) -> Optional[CheckResult]:
    """None when C's dtype is not one the noise model knows (bf16, fp16, fp32). seed: the sign pattern of the
    signed sums (default: this process's)."""
    if C.dtype not in ROUND:
        return None
    batched = C.dim() == 3
    A3 = A if A.dim() == 3 else A.unsqueeze(0)
    B3 = B if B.dim() == 3 else B.unsqueeze(0)
    C3 = C if batched else C.unsqueeze(0)
    if C3.numel() == 0:
        return CheckResult(ok=True, max_z=0.0, nonfinite=False)
    if A3.shape[0] != C3.shape[0]:
        A3 = A3.expand(C3.shape[0], -1, -1)
    if B3.shape[0] != C3.shape[0]:
        B3 = B3.expand(C3.shape[0], -1, -1)
    c = C3.double()
    if bias is not None and beta != 0.0:
        c = c - beta * bias.double()
    if alpha != 1.0:
        if alpha == 0.0:
            raise ValueError("alpha = 0: C holds no product to check")
        c = c / alpha
    zs, den = abft.product_zscores(A3, B3, c, abft.sign_mask(seed), rnd_unit=ROUND[C.dtype] / abs(alpha),
                                   z_alarm=z, return_den=True)
    flat = int(torch.argmax(zs).item())
    mz = float(zs.view(-1)[flat])
    g, rem = divmod(flat, zs.shape[1] * zs.shape[2])
    row, blk = divmod(rem, zs.shape[2])
    nonfinite = bool(torch.isinf(zs).any())
    return CheckResult(ok=bool(math.isfinite(mz) and mz <= z), max_z=mz, nonfinite=nonfinite,
                       batch=g if batched else None, row=row, col_block=blk, noise=float(den.view(-1)[flat]))


def check_linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], y: torch.Tensor,
                 **kw) -> Optional[CheckResult]:
    """Check y = torch.nn.functional.linear(x, weight, bias) for any leading dimensions."""
    return check_matmul(x.reshape(-1, x.shape[-1]), weight.t(), y.reshape(-1, y.shape[-1]), bias, **kw)

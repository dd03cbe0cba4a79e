"""Python entry points of the checked sm_100a GEMM (`csrc/gemm_abft.cu`).

    cw = CheckedWeight(weight, bias)                 # once, at load: checksum rows + block statistics
    y = checked_linear(x, cw, state, slot)           # every call: one kernel, output + check
    StateTable.read()                                # worst score per layer, when the caller wants it

`checked_linear` needs ||x_i||_2^2 per row. Producers in this library (RMSNorm, attention, activation kernels)
emit it for free; pass it as `row_sq`. Without it a small row-norm kernel runs first.

Reference: the serving check `ServeGuard.check` (src/sdcguard/serve.py:846) and its per-layer constants
`LayerChecksums` (serve.py:140); the training-side fused GEMM `fused_mm` (src/sdcguard/fused.py:119).
"""
from __future__ import annotations

import math
import threading
from typing import Optional

import torch

from .. import _native
from ..numerics import abft

_ws_lock = threading.Lock()
_WS: dict = {}          # device index -> zero-initialised workspace tensor (uint8)
_ERR: dict = {}         # device index -> int32 error word


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device workspace of at least nbytes, zero-filled when (re)allocated. Reallocation must not happen
    while a CUDA graph is being captured: engines call `reserve_workspace` with their largest shape first.

    One workspace serves every checked GEMM of the device, so checked GEMMs of one device must not run
    concurrently on different streams (the engines and guards of this package issue them on one stream; the
    replay checks that run on side streams launch no GEMM). Its band counters return to zero at the end of every
    launch that completes; `take_errors` zeroes them after a launch whose wait ran out."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _WS.get(idx)
        if ws is None or ws.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("checked GEMM workspace too small inside CUDA graph capture: "
                                   "call reserve_workspace() with the largest shape before capturing")
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _WS[idx] = ws
        return ws


ERROR_NAMES = {0: "none", 1: "producer wait timed out", 2: "MMA wait timed out", 3: "epilogue wait timed out",
               4: "peer or band wait timed out", 5: "bad argument"}


def take_errors(device: torch.device) -> int:
    """Read and clear the device's kernel error word (first error code recorded by any launch since the last
    call; 0 = none). One device-to-host copy on the current stream, so call it where a sync is acceptable (poll
    time). When a wait ran out, a checked GEMM may have stopped in the middle of a band and left its counters
    raised: they are zeroed on the current stream, so the next launch starts from clean counters instead of
    judging against the expected sums of an unfinished launch."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    e = _ERR.get(idx)
    if e is None:
        return 0
    code = int(e.item())
    if code:
        e.zero_()
        ws = _WS.get(idx)
        if ws is not None:
            n = int(_native.lib().sdc_gemm_counter_bytes())
            ws[:n].zero_()
    return code


_CAP: dict = {}          # device index -> capture record (uint8)
_CAP_HEADER = 80         # bytes before the captured row: 6 int32, the state row's address, 12 float32


def enable_capture(device: torch.device) -> torch.Tensor:
    """Give the checked GEMMs of `device` an alarm-capture record (once per device; call before any CUDA graph is
    captured). The first alarm of any checked GEMM afterwards leaves its evidence there until `read_capture`."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _CAP.get(idx)
    if buf is None:
        lib = _native.lib()
        buf = torch.zeros(int(lib.sdc_gemm_capture_bytes()), dtype=torch.uint8, device=torch.device("cuda", idx))
        with torch.cuda.device(idx):
            _native.check(lib.sdc_gemm_set_capture(buf.data_ptr()), "gemm capture")
        _CAP[idx] = buf
    return buf


def read_capture(device: torch.device, clear: bool = True) -> Optional[dict]:
    """The captured alarm of `device` (one device-to-host copy), or None: the state slot, row and block that
    alarmed, its score, noise, the accumulator's plain / signed / squared / absolute block sums, the expected
    sums, and the input row (bf16, on the CPU). clear: free the record for the next alarm."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _CAP.get(idx)
    if buf is None:
        return None
    head = buf[:_CAP_HEADER].cpu()
    ints = head.view(torch.int32)[:6].tolist()
    if ints[0] != 1:
        return None
    state_row = int(head[24:32].view(torch.int64)[0]) & 0xFFFFFFFFFFFFFFFF
    f = head.view(torch.float32)[8:20].tolist()
    k = ints[4]
    x = buf[_CAP_HEADER:_CAP_HEADER + 2 * k].cpu().view(torch.bfloat16).clone()
    if clear:
        buf[:_CAP_HEADER].zero_()
    return {"state_row": state_row, "slot": ints[1], "row": ints[2], "block": ints[3], "k": k,
            "signed": bool(ints[5]), "z": f[0],
            "noise": f[1], "actual_plain": f[2], "actual_signed": f[3], "expected_plain": f[4],
            "expected_signed": f[5], "sum_sq": f[6], "sum_abs": f[7], "row_sq": f[8], "x_row": x}


def recheck_capture(cap: dict, cw: "CheckedWeight") -> dict:
    """Float64 recheck of a captured alarm against the layer's weights (as they are now) and the checksum rows
    built when the layer was registered. Verdicts:
      weights_changed  the current weights' block sums no longer match the registered checksum rows
      output_wrong     the accumulator's block sums are off the exact product, the expected sums are right
      expected_wrong   the expected sums (checksum tiles) are off the exact product, the accumulator is right
      both_wrong       both are off
      not_reproduced   both agree with the exact product within the noise the alarm was judged with"""
    b = cap["block"]
    c0, c1 = b * abft.BLOCK, min((b + 1) * abft.BLOCK, cw.n)
    x = cap["x_row"].double().to(cw.weight.device)
    w = cw.weight[c0:c1].double()
    signs = abft.sign_vector(cw.mask, device=w.device)[: c1 - c0]
    vals = w @ x
    if cw.bias is not None:
        vals = vals + cw.bias[c0:c1].double()
    exact = (float(vals.sum()), float((vals * signs).sum()))
    # what the registered checksum rows say the block sums are (three bf16 parts per sum)
    parts = cw.cs.wc[b * abft.CS_ROWS:(b + 1) * abft.CS_ROWS].double() @ x
    reg = (float(parts[:3].sum()), float(parts[3:].sum()))
    if cw.cs.bsum is not None:
        reg = (reg[0] + float(cw.cs.bsum[b, 0]), reg[1] + float(cw.cs.bsum[b, 1]))
    noise = max(cap["noise"], abft.ABS_FLOOR)
    line = abft.Z_ALARM * noise
    act = (cap["actual_plain"], cap["actual_signed"])
    exp = (cap["expected_plain"], cap["expected_signed"])
    off = lambda a, e: any(abs(u - v) > line for u, v in zip(a, e))     # noqa: E731
    if off(reg, exact):
        verdict = "weights_changed"
    elif off(act, exact) and off(exp, exact):
        verdict = "both_wrong"
    elif off(act, exact):
        verdict = "output_wrong"
    elif off(exp, exact):
        verdict = "expected_wrong"
    else:
        verdict = "not_reproduced"
    return {"verdict": verdict, "exact": exact, "registered_checksums": reg, "actual": act, "expected": exp,
            "line": line}


def reserve_workspace(device: torch.device, m: int, n: int) -> None:
    workspace(device, int(_native.lib().sdc_gemm_ws_bytes(m, n)))


_RESERVED_ROWS: dict = {}


def reserve_for_rows(device: torch.device, n: int, max_m: int) -> int:
    """Size the workspace for every row count 1..max_m of an n-column GEMM (split-K at small row counts can need
    more than the largest count does); returns the bytes reserved. For callers whose row count varies under CUDA
    graph capture (a serving engine's batch sizes)."""
    key = (n, max_m)
    need = _RESERVED_ROWS.get(key)
    if need is None:
        f = _native.lib().sdc_gemm_ws_bytes
        need = _RESERVED_ROWS[key] = max(int(f(m, n)) for m in range(1, max_m + 1))
    workspace(device, need)
    return need


def error_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    e = _ERR.get(idx)
    if e is None:
        e = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[idx] = e
    return e


class StateTable:
    """Per-device int64 state rows [slots, 4], one per checked layer (layout in numerics.abft)."""

    def __init__(self, device, slots: int = 256):
        self.device = torch.device(device)
        self.state = torch.zeros(slots, abft.STATE_COLS, dtype=torch.int64, device=self.device)
        self.names: list[str] = []
        self.nbs: list[int] = []
        self.kinds: list[str] = []

    def add(self, name: str, nb: int, kind: str = "gemm") -> int:
        """kind "gemm": location = checksum index (row, block, signed); "collective": location = (row, block,
        peer) as the TP collective kernels encode it ((row * nb + block) * 8 + peer); "rowblock": (row, block)
        (row * nb + block), the expert-parallel transfers."""
        if len(self.names) >= self.state.shape[0]:
            grown = torch.zeros(self.state.shape[0] * 2, abft.STATE_COLS, dtype=torch.int64, device=self.device)
            grown[: self.state.shape[0]] = self.state
            self.state = grown
        self.names.append(name)
        self.nbs.append(nb)
        self.kinds.append(kind)
        return len(self.names) - 1

    def read(self, reset: bool = False) -> list[dict]:
        """Every row now (one device-to-host copy, which waits for the stream), decoded; reset zeroes the table."""
        rows = self.state[: len(self.names)].cpu().tolist()
        if reset:
            self.state.zero_()
        return self.decode(rows)

    def slot_of(self, state_row_address: int) -> Optional[int]:
        """The slot whose row is at this device address, or None when the row belongs to another table."""
        base = self.state.data_ptr()
        off = state_row_address - base
        row_bytes = abft.STATE_COLS * 8
        if off < 0 or off % row_bytes or off // row_bytes >= len(self.names):
            return None
        return off // row_bytes

    def read_async(self, reset: bool = True) -> "PendingRead":
        """Start a read that never waits: on the current stream, the rows are copied to a device snapshot (and the
        table zeroed when reset), the snapshot to pinned host memory, and an event is recorded. The returned read
        is decoded once its event has completed (`PendingRead.result`)."""
        n = len(self.names)
        snap = self.state[:n].clone()
        if reset:
            self.state.zero_()
        host = torch.empty(snap.shape, dtype=snap.dtype, pin_memory=True)
        host.copy_(snap, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        return PendingRead(self, host, ev, snap)

    def decode(self, rows) -> list[dict]:
        out = []
        for i, r in enumerate(rows):
            d = abft.decode_state_row(r)
            d["name"] = self.names[i]
            d["slot"] = i
            if d["z"] > 0 and self.kinds[i] == "collective":
                rb, d["peer"] = divmod(d["flat"], 8)
                d["row"], d["block"] = divmod(rb, self.nbs[i])
            elif d["z"] > 0 and self.kinds[i] == "rowblock":
                d["row"], d["block"] = divmod(d["flat"], self.nbs[i])
            elif d["z"] > 0:
                d["row"], d["block"], d["signed"] = abft.locate(d["flat"], self.nbs[i])
            out.append(d)
        return out


class PendingRead:
    """A state-table read in flight (see StateTable.read_async)."""

    def __init__(self, table: "StateTable", host: torch.Tensor, event, snap: torch.Tensor):
        self.table, self.host, self.event, self._snap = table, host, event, snap

    def ready(self) -> bool:
        return self.event.query()

    def result(self, wait: bool = False):
        """The decoded rows, or None while the copy is still in flight (wait=True blocks until it lands)."""
        if not wait and not self.event.query():
            return None
        self.event.synchronize()
        self._snap = None
        return self.table.decode(self.host.tolist())


class CheckedWeight:
    """A bf16 weight W (n, k) with its checksum rows and block statistics, ready for `checked_linear`."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, mask: Optional[tuple] = None,
                 c1: float = abft.C1, c2: float = abft.C2, c3: float = abft.C3):
        if weight.dtype != torch.bfloat16 or weight.dim() != 2:
            raise ValueError("CheckedWeight needs a 2-D bf16 weight")
        n, k = weight.shape
        if k % 8 or n % 8:
            raise ValueError(f"checked GEMM needs n and k multiples of 8 (got n={n}, k={k})")
        self.weight = weight.contiguous()
        self.bias = None if bias is None else bias.detach().float().contiguous()
        self.cs = abft.weight_checksums(self.weight, bias, mask)
        self.mask = self.cs.mask
        self.prod_coef, self.out_coef = abft.coefficients(k, c1, c2, c3)
        self.n, self.k, self.nb = n, k, self.cs.nb

    def refresh(self) -> None:
        """Recompute the checksums after the weight was changed on purpose (e.g. a reload)."""
        self.cs = abft.weight_checksums(self.weight, self.bias, self.mask)

    @classmethod
    def _assemble(cls, b: torch.Tensor, cs: abft.WeightChecksums, bias, c1, c2, c3) -> "CheckedWeight":
        self = cls.__new__(cls)
        self.weight = b
        self.bias = None if bias is None else bias.detach().float().contiguous()
        self.cs, self.mask = cs, cs.mask
        n, k = b.shape
        self.prod_coef, self.out_coef = abft.coefficients(k, c1, c2, c3)
        self.n, self.k, self.nb = n, k, cs.nb
        return self

    @classmethod
    def on_device(cls, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, c1: float = abft.C1,
                  c2: float = abft.C2, c3: float = abft.C3) -> "CheckedWeight":
        """As CheckedWeight(weight, bias), with the checksum rows and block statistics built by one device pass
        (`sdc_prep_colblock`) instead of fp64 PyTorch reductions: the forward weight after each optimizer step."""
        w = weight.detach().contiguous()
        if not w.is_cuda:
            return cls(w, bias, c1=c1, c2=c2, c3=c3)
        n, k = w.shape
        if n % 8 or k % 8:
            raise ValueError(f"checked GEMM needs n and k multiples of 8 (got n={n}, k={k})")
        # the bias's block sums come from the same launch; its largest magnitude is not read back (a host read per
        # layer would stall a training step): 0 means a non-finite output counts as corruption unless the weights
        # and inputs can produce it
        b32 = None if bias is None else bias.detach().float().contiguous()
        cs = _prep(w, transposed=False, bias=b32)
        return cls._assemble(w, cs, b32, c1, c2, c3)

    @classmethod
    def of_transpose(cls, m: torch.Tensor, c1: float = abft.C1, c2: float = abft.C2,
                     c3: float = abft.C3) -> "CheckedWeight":
        """CheckedWeight of B = m^T for m (r, c) bf16, built in one device pass over m (`sdc_prep_rowblock`): the
        transpose and its checksum rows together. The training guard's W^T (for dX) and X^T (for dW)."""
        m = m.detach()
        if m.stride(-1) != 1:
            m = m.contiguous()
        if not m.is_cuda:
            return cls(m.t().contiguous(), c1=c1, c2=c2, c3=c3)
        r, c = m.shape
        if r % 8 or c % 8:
            raise ValueError(f"checked GEMM needs n and k multiples of 8 (got {c} x {r})")
        cs, t = _prep(m, transposed=True)
        return cls._assemble(t, cs, None, c1, c2, c3)


def transpose(m: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """m^T as a new contiguous bf16 tensor, by a tiled shared-memory transpose kernel (PyTorch's strided copy of
    `.t().contiguous()` is several times slower at these sizes)."""
    if m.dtype != torch.bfloat16 or m.dim() != 2 or m.stride(1) != 1 or not m.is_cuda:
        return m.t().contiguous()
    r, c = m.shape
    if out is None:
        out = torch.empty(c, r, dtype=torch.bfloat16, device=m.device)
    _native.check(_native.lib().sdc_transpose_bf16(m.data_ptr(), m.stride(0), r, c, out.data_ptr(),
                                                   _stream_ptr(m.device)), "transpose")
    return out


_PREP_ACC: dict = {}


def _prep(m: torch.Tensor, transposed: bool, bias: Optional[torch.Tensor] = None):
    """Device checksum data: of B = m (transpose False; with its bias's block sums when given) or of B = m^T (True,
    also returning m^T). The kernels' statistics scratch (nb * 4 floats and a ticket) is zero between calls: the
    last CTA of each launch finalizes the statistics and clears it."""
    dev = m.device
    r, c = m.shape
    mask = abft.sign_mask()
    nb = -(-(c if transposed else r) // abft.BLOCK)
    acc = _PREP_ACC.get(dev)
    if acc is None or acc.numel() < nb * 4 + 1:
        acc = _PREP_ACC[dev] = torch.zeros(max(nb * 4 + 1, 1025), dtype=torch.float32, device=dev)
    wstat = torch.empty(nb, 4, dtype=torch.float32, device=dev)
    lib = _native.lib()
    if transposed:
        t = transpose(m)
        wc = torch.empty(nb * abft.CS_ROWS, r, dtype=torch.bfloat16, device=dev)
        _native.check(lib.sdc_prep_rowblock(m.data_ptr(), m.stride(0), r, c, mask[0], mask[1], mask[2], mask[3],
                                            None, wc.data_ptr(), wstat.data_ptr(), acc.data_ptr(),
                                            _stream_ptr(dev)), "checksum prep (rows)")
        cs = abft.WeightChecksums(n=c, k=r, nb=nb, wc=wc, wstat=wstat, bsum=None, bias_max=0.0, mask=mask)
        return cs, t
    wc = torch.empty(nb * abft.CS_ROWS, c, dtype=torch.bfloat16, device=dev)
    bsum = None
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != r or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous fp32 vector of the weight's rows")
        bsum = torch.empty(nb, 2, dtype=torch.float32, device=dev)
    _native.check(lib.sdc_prep_colblock(m.data_ptr(), m.stride(0), r, c, mask[0], mask[1], mask[2], mask[3],
                                        wc.data_ptr(), wstat.data_ptr(), acc.data_ptr(),
                                        None if bias is None else bias.data_ptr(),
                                        None if bsum is None else bsum.data_ptr(), _stream_ptr(dev)),
                  "checksum prep (columns)")
    return abft.WeightChecksums(n=r, k=c, nb=nb, wc=wc, wstat=wstat, bsum=bsum, bias_max=0.0, mask=mask)


def row_sqnorm(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    m, k = x.shape
    if out is None:
        out = torch.empty(m, dtype=torch.float32, device=x.device)
    _native.check(_native.lib().sdc_row_sqnorm_bf16(x.data_ptr(), x.stride(0), m, k, out.data_ptr(),
                                                     _stream_ptr(x.device)), "row_sqnorm")
    return out


LONG_K = 8192


def pick_bn(m: int, n: int, num_sms: int = 148, k: int = 0) -> int:
    """256-wide tiles when there are enough of them to fill the GPU, else 128. With a long K (the training dW GEMMs,
    K = tokens) 256-wide CTA-pair tiles whenever there are two bands: split-K spreads them over the GPU, and a pair
    tile streams half the operand bytes per FLOP of a 128 x 128 one."""
    if k >= LONG_K and m > 128:
        return 256
    tiles256 = -(-m // 128) * -(-n // 256)
    return 256 if tiles256 >= num_sms * 0.75 else 128


def checked_linear(x: torch.Tensor, cw: CheckedWeight, state: torch.Tensor, slot: int,
                   row_sq: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                   z_alarm: float = abft.Z_ALARM, bn: Optional[int] = None, max_ctas: int = 0,
                   inject: Optional[tuple] = None, dbg: Optional[torch.Tensor] = None,
                   seal: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ W^T (+ b) on tcgen05 with the ABFT check folded into `state[slot]`.
    x: (m, k) bf16 with unit column stride. inject=(row, col, xor_bits) flips bits of one fp32 accumulator
    element before the check and the rounding (fault-injection experiments). seal: optional (m, nb) int32 output,
    an exact hash of the stored bf16 bits of every (row, 128-column block) (see `seal_reference`)."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("checked_linear needs a 2-D bf16 x with unit column stride")
    m, k = x.shape
    if k != cw.k:
        raise ValueError(f"x has {k} columns, the weight {cw.k}")
    dev = x.device
    if out is None:
        out = torch.empty(m, cw.n, dtype=torch.bfloat16, device=dev)
    if m == 0:
        return out
    if row_sq is None:
        row_sq = row_sqnorm(x)
    lib = _native.lib()
    ws = workspace(dev, int(lib.sdc_gemm_ws_bytes(m, cw.n)))
    err = error_word(dev)
    if bn is None:
        bn = pick_bn(m, cw.n, k=k)
    s = cw.mask
    inj_row, inj_col, inj_xor = (-1, -1, 0) if inject is None else (int(inject[0]), int(inject[1]), int(inject[2]))
    rc = lib.sdc_gemm_bf16(
        x.data_ptr(), x.stride(0), cw.weight.data_ptr(), cw.cs.wc.data_ptr(), m, cw.n, k, out.data_ptr(),
        out.stride(0), None if cw.bias is None else cw.bias.data_ptr(),
        None if cw.cs.bsum is None else cw.cs.bsum.data_ptr(), float(cw.cs.bias_max), row_sq.data_ptr(),
        cw.cs.wstat.data_ptr(), ws.data_ptr(), state.data_ptr(), int(slot), s[0], s[1], s[2], s[3],
        float(z_alarm), float(cw.prod_coef), float(cw.out_coef), float(abft.ABS_FLOOR), float(math.sqrt(k)),
        err.data_ptr(), int(bn), int(max_ctas), inj_row, inj_col, inj_xor,
        None if dbg is None else dbg.data_ptr(), None if seal is None else seal.data_ptr(), _stream_ptr(dev))
    _native.check(rc, "checked GEMM launch")
    return out


class CheckedWeightStack:
    """The weights of several experts (each (n, k) bf16, no bias) stacked for `checked_linear_grouped`: W as
    (experts * n, k), the checksum rows as (experts * 6 nb, k), block statistics (experts, nb, 4)."""

    def __init__(self, weights: list, c1: float = abft.C1, c2: float = abft.C2, c3: float = abft.C3):
        if not weights:
            raise ValueError("CheckedWeightStack needs at least one weight")
        n, k = weights[0].shape
        if any(w.shape != (n, k) or w.dtype != torch.bfloat16 for w in weights):
            raise ValueError("expert weights must share one (n, k) shape and be bf16")
        if n % abft.BLOCK or k % 8:
            raise ValueError(f"grouped checked GEMM needs n a multiple of 128 and k of 8 (got n={n}, k={k})")
        css = [abft.weight_checksums(w) for w in weights]
        self.mask = css[0].mask
        self.weight = torch.cat([w.contiguous() for w in weights]).contiguous()
        self.wc = torch.cat([c.wc for c in css]).contiguous()
        self.wstat = torch.cat([c.wstat for c in css]).contiguous()
        self.experts, self.n, self.k, self.nb = len(weights), n, k, css[0].nb
        self.prod_coef, self.out_coef = abft.coefficients(k, c1, c2, c3)

    def expert(self, e: int) -> torch.Tensor:
        return self.weight[e * self.n:(e + 1) * self.n]


def checked_linear_grouped(x: torch.Tensor, stack: CheckedWeightStack, gband: torch.Tensor, gcount: torch.Tensor,
                           state: torch.Tensor, slot: int, row_sq: Optional[torch.Tensor] = None,
                           out: Optional[torch.Tensor] = None, z_alarm: float = abft.Z_ALARM,
                           bn: Optional[int] = None, inject: Optional[tuple] = None) -> torch.Tensor:
    """y[r] = x[r] @ W_e^T for the rows r of every expert e, in one launch with the ABFT check folded into
    `state[slot]`. x (cap, k) holds the experts' rows grouped on 128-row bands (ops.moe.group or the
    expert-parallel receive); gband (cap / 128) int32 is the expert of each band and gcount (1,) int32 the bands in
    use, both on the device: nothing is read back, so the call can be graph-captured. Rows past the bands in use
    are neither read nor written."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("checked_linear_grouped needs a 2-D bf16 x with unit column stride")
    m, k = x.shape
    if k != stack.k:
        raise ValueError(f"x has {k} columns, the weights {stack.k}")
    dev = x.device
    if out is None:
        out = torch.empty(m, stack.n, dtype=torch.bfloat16, device=dev)
    if m == 0:
        return out
    if row_sq is None:
        row_sq = row_sqnorm(x)
    lib = _native.lib()
    ws = workspace(dev, int(lib.sdc_gemm_ws_bytes(m, stack.n)))
    err = error_word(dev)
    if bn is None:
        bn = 256 if stack.n % 256 == 0 and pick_bn(m, stack.n) == 256 else 128
    s = stack.mask
    inj_row, inj_col, inj_xor = (-1, -1, 0) if inject is None else (int(inject[0]), int(inject[1]), int(inject[2]))
    rc = lib.sdc_gemm_bf16_grouped(
        x.data_ptr(), x.stride(0), stack.weight.data_ptr(), stack.wc.data_ptr(), stack.experts, m, stack.n, k,
        out.data_ptr(), out.stride(0), row_sq.data_ptr(), stack.wstat.data_ptr(), gband.data_ptr(),
        gcount.data_ptr(), ws.data_ptr(), state.data_ptr(), int(slot), s[0], s[1], s[2], s[3], float(z_alarm),
        float(stack.prod_coef), float(stack.out_coef), float(abft.ABS_FLOOR), float(math.sqrt(k)), err.data_ptr(),
        int(bn), inj_row, inj_col, inj_xor, _stream_ptr(dev))
    _native.check(rc, "grouped checked GEMM launch")
    return out


SEAL_MUL = 0x85EBCA6B


def seal_reference(y: torch.Tensor) -> torch.Tensor:
    """(m, nb) int32 seals of a bf16 (m, n) tensor: per (row, 128-column block, zero-padded past column n), sum over
    its 64 words of two bf16 of ((word ^ (w + 1) * 0x9E3779B9) * 0x85EBCA6B) mod 2^32 (what the kernels compute)."""
    m, n = y.shape
    nb = -(-n // 128)
    pad = torch.zeros(m, nb * 128, dtype=torch.bfloat16, device=y.device)
    pad[:, :n] = y
    words = pad.view(torch.int32).view(m, nb, 64).to(torch.int64) & 0xFFFFFFFF
    w = torch.arange(64, dtype=torch.int64, device=y.device)
    keys = ((w + 1) * 0x9E3779B9) & 0xFFFFFFFF
    terms = ((words ^ keys) * SEAL_MUL) & 0xFFFFFFFF
    s = terms.sum(-1) & 0xFFFFFFFF
    return torch.where(s >= 2 ** 31, s - 2 ** 32, s).to(torch.int32)

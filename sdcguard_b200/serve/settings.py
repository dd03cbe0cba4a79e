"""Which checks the checked decoder runs, from constructor arguments or the `SDCGUARD_*` environment.

    SDCGUARD_SHARE    share of the linear layers whose GEMMs carry the ABFT check: 1 (default), 0.125, 1/8 or 12.5%
    SDCGUARD_OFFSET   which window of that share this replica takes (0 .. 1/share - 1): replicas with offsets 0 to
                      R - 1 at share 1/R check disjoint sets of layers that together cover every layer once
    SDCGUARD_NORMS    replay the RMSNorm rows (default 1)
    SDCGUARD_ROPE     replay the q/k norm + RoPE + KV-cache write rows (default 1)
    SDCGUARD_ATTN     replay the attention rows (default 1)
    SDCGUARD_ACT      replay the SwiGLU rows (default 1)
    SDCGUARD_SPOT     sampled exact spot check of one linear layer per prefill step (default 1)
    SDCGUARD_Z        alarm line of the checks in noise units (default 6)

A projection left out by the share runs unchecked on the library GEMM, as an unregistered layer does in the
reference's plugin: a share trades coverage for cost. Values that cannot be read fall back to the safe reading (every layer, every
check on) with a warning, as the reference's plugin does (src/sdcguard/vllm_plugin.py:181-236, serve.py:104).

The share uses a Weyl sequence: layer i sits at frac(i / phi) on the unit circle and is checked when that point falls
in the window [offset * share, (offset + 1) * share). The golden-ratio stride spreads a share over every depth and
every projection (taking every R-th layer would pick the same projection of every block).
"""
from __future__ import annotations

import logging
import math
import os
from dataclasses import dataclass, field

log = logging.getLogger("sdcguard")

INV_PHI = (math.sqrt(5.0) - 1.0) / 2.0


def parse_share(text: str) -> float:
    """'0.125', '1/8' or '12.5%' -> 0.125; raises ValueError for anything else (or a value outside [0, 1])."""
    t = str(text).strip()
    if t.endswith("%"):
        v = float(t[:-1]) / 100.0
    elif "/" in t:
        num, den = t.split("/", 1)
        v = float(num) / float(den)
    else:
        v = float(t)
    if not math.isfinite(v) or v < 0.0 or v > 1.0:
        raise ValueError(f"share {text!r} is not in [0, 1]")
    return v


def layer_selected(i: int, share: float, offset: int = 0) -> bool:
    """Is linear layer number i (model order) in this replica's share?"""
    if share >= 1.0:
        return True
    if share <= 0.0:
        return False
    start = (offset * share) % 1.0
    return (((i * INV_PHI) % 1.0) - start) % 1.0 < share


def _flag(name: str, default: bool = True) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    v = v.strip().lower()
    if v in ("0", "false", "off", "no"):
        return False
    if v in ("1", "true", "on", "yes", ""):
        return True
    log.warning("sdcguard: %s=%r is not 0 or 1; the check stays %s", name, v, "on" if default else "off")
    return default


@dataclass
class CheckSettings:
    share: float = 1.0
    offset: int = 0
    norms: bool = True
    rope: bool = True
    attn: bool = True
    act: bool = True
    spot: bool = True
    z_alarm: float = 6.0
    notes: list = field(default_factory=list)

    @classmethod
    def from_env(cls) -> "CheckSettings":
        s = cls()
        raw = os.environ.get("SDCGUARD_SHARE")
        if raw is not None:
            try:
                s.share = parse_share(raw)
            except ValueError:
                log.warning("sdcguard: SDCGUARD_SHARE=%r is not a share (use 0.125, 1/8 or 12.5%%); checking every "
                            "layer", raw)
                s.notes.append("SDCGUARD_SHARE unreadable: every layer checked")
        try:
            s.offset = int(os.environ.get("SDCGUARD_OFFSET", "0"))
        except ValueError:
            s.notes.append("SDCGUARD_OFFSET unreadable: offset 0")
        s.norms, s.rope = _flag("SDCGUARD_NORMS"), _flag("SDCGUARD_ROPE")
        s.attn, s.act, s.spot = _flag("SDCGUARD_ATTN"), _flag("SDCGUARD_ACT"), _flag("SDCGUARD_SPOT")
        try:
            z = float(os.environ.get("SDCGUARD_Z", "6"))
            if not math.isfinite(z) or z <= 0:
                raise ValueError
            s.z_alarm = z
        except ValueError:
            s.notes.append("SDCGUARD_Z unreadable: 6")
        return s

    def gemm_checked(self, layer: int, proj: int, n_proj: int = 4) -> bool:
        """Is projection `proj` of layer `layer` (numbered layer * n_proj + proj) in the share?"""
        return layer_selected(layer * n_proj + proj, self.share, self.offset)

    def describe(self) -> dict:
        return {"share": self.share, "offset": self.offset, "norms": self.norms, "rope": self.rope,
                "attn": self.attn, "act": self.act, "spot": self.spot, "z_alarm": self.z_alarm, "notes": self.notes}

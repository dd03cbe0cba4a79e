"""GPU information for reports: nvidia-smi queries (read only: this module never changes a GPU setting),
datasheet peaks, and a background sampler of clocks, power and throttle reasons.

Reference: `datasheet` (src/sdcguard/gpuinfo.py:36), `health` (:121), `Sampler` (:156).
"""
from __future__ import annotations

import os
import statistics
import subprocess
import tempfile
from typing import Optional

# dense (non-sparse) per-GPU peaks, TFLOP/s and TB/s, from the public datasheets
DATASHEET = {
    "B200": {"bf16": 2250.0, "fp16": 2250.0, "fp8": 4500.0, "fp4": 9000.0, "tf32": 1100.0, "hbm_tbs": 7.7},
    "H100": {"bf16": 989.0, "fp16": 989.0, "fp8": 1979.0, "tf32": 495.0, "hbm_tbs": 3.35},
    "A100": {"bf16": 312.0, "fp16": 312.0, "tf32": 156.0, "hbm_tbs": 2.0},
}

REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def datasheet(name: str) -> Optional[dict]:
    for k, v in DATASHEET.items():
        if k in name:
            return dict(v)
    return None


def query(fields: str, index: Optional[int] = None) -> list[list[str]]:
    """Rows of `nvidia-smi --query-gpu=<fields>` (empty when nvidia-smi is missing)."""
    cmd = ["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits"]
    if index is not None:
        cmd[1:1] = ["-i", str(index)]
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=20).stdout
    except (OSError, subprocess.TimeoutExpired):
        return []
    return [[p.strip() for p in line.split(",")] for line in out.splitlines() if line.strip()]


def health(index: Optional[int] = None) -> list[dict]:
    """Name, UUID, temperature, power, clocks, ECC error counts and active throttle reasons per GPU."""
    f = ("index,name,uuid,temperature.gpu,power.draw,clocks.sm,clocks.max.sm,ecc.errors.uncorrected.volatile.total,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    out = []
    for r in query(f, index):
        if len(r) < 12:
            continue
        out.append({"index": r[0], "name": r[1], "uuid": r[2], "temp_c": r[3], "power_w": r[4], "sm_mhz": r[5],
                    "sm_max_mhz": r[6], "ecc_uncorrected": r[7],
                    "throttle": [n for n, v in zip(REASONS, r[8:12]) if v.lower().startswith("active")]})
    return out


def parse_samples(lines) -> dict:
    """Summary of sampler CSV lines (index, sm, max sm, power, active, four reason columns)."""
    sm, mx, pw, reasons = [], None, [], set()
    for line in lines:
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 9:
            continue
        try:
            sm.append(float(parts[1]))
            mx = float(parts[2])
            pw.append(float(parts[3]))
        except ValueError:
            continue
        for nm, v in zip(REASONS, parts[5:9]):
            if v.lower().startswith("active"):
                reasons.add(nm)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
            "samples": len(sm), "power_w_median": statistics.median(pw) if pw else None}


class Sampler:
    """Samples SM clock, max clock, power and throttle reasons every 200 ms while active (nvidia-smi -lms)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period_ms: int = 200):
        self.index, self.period = index, period_ms
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix="sdcguard_clocks_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        try:
            with open(self.path) as fh:
                return parse_samples(fh.readlines())
        except OSError:
            return parse_samples([])
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass

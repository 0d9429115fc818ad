"""FLOP accounting and MFU against the measured B200 peak."""

from __future__ import annotations

import json
from pathlib import Path

# Nominal dense bf16 peak of one B200; used only when no measurement exists.
NOMINAL_BF16_FLOPS = 2.25e15


def peak_flops(kind: str = "bf16_tflops") -> float:
    """Measured bf16 peak (FLOP/s) from MEASURED_PEAKS.json at the repo root,
    or the nominal figure."""
    root = Path(__file__).resolve().parents[2]
    p = root / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            v = json.loads(p.read_text()).get(kind)
            if v:
                return float(v) * 1e12
        except Exception:
            pass
    return NOMINAL_BF16_FLOPS


def mfu(config, seq_len: int, tokens_per_sec: float, num_gpus: int) -> float:
    flops = config.train_flops_per_token(seq_len) * tokens_per_sec
    return flops / (peak_flops() * max(1, num_gpus))


def measured_peaks() -> dict:
    """{"hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"} measured on this
    machine pool (MEASURED_PEAKS.json), else the pool's earlier fallback
    figures (6.65 TB/s copy, 1.59 PFLOP/s burst, 1.4 PFLOP/s sustained)."""
    root = Path(__file__).resolve().parents[2]
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
           "source": "fallback"}
    p = root / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
                if d.get(k):
                    out[k] = float(d[k])
            out["source"] = "measured"
        except Exception:
            pass
    return out

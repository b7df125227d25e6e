"""Ladder constants and the APAConfig dataclass.

Same names, values and defaults as the reference (apa/config.py:5-92) so that
code written against it runs unchanged. ``gamma`` is kept as a field but, as
in the reference, the overflow thresholds are fixed at 0.90 of each format's
maximum (apa/config.py:9-13); no code path reads ``gamma``.

``fp8_simulation_mode`` is accepted for compatibility and ignored: this
package has one compute path, the sm_100a kernels, and no simulated or CPU
fallback.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

LEVEL_FP8 = 0
LEVEL_FP16 = 1
LEVEL_TF32 = 2

# apa/config.py:9-13: overflow threshold per level (0.90 x format maximum)
THRESHOLDS_MAX = {
    LEVEL_FP8: 0.90 * 448.0,
    LEVEL_FP16: 0.90 * 65504.0,
    LEVEL_TF32: float("inf"),
}

# apa/config.py:15-19: underflow threshold per level (smallest normal-ish value)
THRESHOLDS_MIN = {
    LEVEL_FP8: 0.015625,
    LEVEL_FP16: 6.1035e-5,
    LEVEL_TF32: 0.0,
}

DTYPE_MAP = {
    LEVEL_FP8: getattr(torch, "float8_e4m3fn", None),
    LEVEL_FP16: torch.float16,
    LEVEL_TF32: torch.float32,
}


@dataclass
class APAConfig:
    """Configuration of the ladder (apa/config.py:32-74)."""

    gamma: float = 0.90
    theta_underflow: float = 0.40
    ema_alpha: float = 0.95
    check_interval: int = 1
    fp8_simulation_mode: bool = False
    log_file: Optional[str] = None
    device: str = "cuda"

    # Forensic logging: opt-in, one JSON snapshot per escalation; it reads
    # tensor statistics back to the host for every tracked tensor while on.
    enable_forensic_logging: bool = False
    forensic_log_file: Optional[str] = None
    forensic_capture_argmax_index: bool = False
    forensic_capture_tensor_stats: bool = True

    def __post_init__(self):
        if DTYPE_MAP[LEVEL_FP8] is None:
            self.fp8_simulation_mode = True
        if self.enable_forensic_logging and self.forensic_log_file is None:
            if self.log_file is not None:
                stem, dot, _ext = self.log_file.rpartition(".")
                self.forensic_log_file = (stem if dot else self.log_file) + "_forensic.jsonl"
            else:
                self.forensic_log_file = "apa_forensic.jsonl"

    @classmethod
    def conservative(cls, **kwargs):
        return cls(**{"gamma": 0.80, "theta_underflow": 0.30, "check_interval": 1, **kwargs})

    @classmethod
    def aggressive(cls, **kwargs):
        return cls(**{"gamma": 0.95, "theta_underflow": 0.50, "check_interval": 8, **kwargs})

    @classmethod
    def research_default(cls, **kwargs):
        return cls(**{"gamma": 0.90, "theta_underflow": 0.40, "check_interval": 4, **kwargs})

"""Telemetry reductions and the JSONL loggers.

``track_telemetry_on_tensor`` and ``compute_underflow_ratio`` keep the
reference's signatures (apa/telemetry.py:7-39) but run as single-pass CUDA
reductions (``apa_amax`` / ``apa_underflow_ratio``). On the hot path they are
not called at all: the cast and GEMM kernels fold the same reductions into
the passes that produce the tensors. The loggers are plain Python, as in the
reference (apa/telemetry.py:41-122); they run only when an event occurs.
"""
from __future__ import annotations

import json
import os
from datetime import datetime, timezone
from typing import Optional

import torch

from . import _lib

_COUNTERS = {}


def _scratch_counters(device) -> torch.Tensor:
    """Three zeroed u64 words per device for the standalone ratio reduction
    (the kernel leaves them zero again). Calls on one device share them, so
    they are serialised on the caller's stream."""
    key = torch.device(device)
    c = _COUNTERS.get(key)
    if c is None:
        c = torch.zeros(3, dtype=torch.int64, device=key)
        _COUNTERS[key] = c
    return c


def track_telemetry_on_tensor(tensor: torch.Tensor, gpu_amax: torch.Tensor,
                              gpu_has_nonfinite: torch.Tensor) -> None:
    """gpu_amax = max(gpu_amax, max|tensor|) (NaN-propagating) and
    gpu_has_nonfinite = max(flag, 1) if any element is NaN/Inf
    (apa/telemetry.py:7-21)."""
    _lib.require_cuda(tensor, "track_telemetry_on_tensor")
    t = tensor.detach()
    if not t.is_contiguous():
        t = t.contiguous()
    st = _lib.lib().apa_amax(t.data_ptr(), _lib.dt_code(t.dtype), t.numel(), _lib.ptr(gpu_amax),
                             _lib.ptr(gpu_has_nonfinite), _lib.stream_handle(t.device))
    _lib.check(st, "apa_amax")


def _underflow(grad: torch.Tensor, v_min: float, out: torch.Tensor, running_max: bool) -> None:
    _lib.require_cuda(grad, "compute_underflow_ratio")
    g = grad.detach()
    if not g.is_contiguous():
        g = g.contiguous()
    st = _lib.lib().apa_underflow_ratio(g.data_ptr(), _lib.dt_code(g.dtype), g.numel(), float(v_min),
                                        _scratch_counters(g.device).data_ptr(), out.data_ptr(),
                                        1 if running_max else 0, _lib.stream_handle(g.device))
    _lib.check(st, "apa_underflow_ratio")


def compute_underflow_ratio(grad_tensor: torch.Tensor, v_min_threshold: float) -> torch.Tensor:
    """#(0 < |g| < v_min) / #(|g| > 0) as an fp32 scalar tensor on the
    gradient's device, 0 when no element is nonzero (apa/telemetry.py:23-39).
    The threshold is applied in fp32, as torch applies a Python float to an
    fp32 tensor. Unlike the reference there is no host synchronisation."""
    out = torch.empty((), dtype=torch.float32, device=grad_tensor.device)
    _underflow(grad_tensor, v_min_threshold, out, running_max=False)
    return out


def update_running_underflow(grad: torch.Tensor, v_min: float, ratio_buf: torch.Tensor) -> None:
    """ratio_buf = max(ratio_buf, compute_underflow_ratio(grad, v_min)) in one launch."""
    _underflow(grad, v_min, ratio_buf, running_max=True)


def _utc_now() -> str:
    return datetime.now(timezone.utc).replace(tzinfo=None).isoformat() + "Z"


class APAEventLogger:
    """Escalation / skip-batch events as JSONL plus a stdout line
    (apa/telemetry.py:41-75)."""

    def __init__(self, log_file: Optional[str]):
        self.log_file = log_file

    def _log_event(self, event_data: dict):
        event_data["timestamp"] = _utc_now()
        line = json.dumps(event_data)
        print(f"APA Event: {line}")
        if self.log_file:
            try:
                os.makedirs(os.path.dirname(os.path.abspath(self.log_file)), exist_ok=True)
                with open(self.log_file, "a") as fh:
                    fh.write(line + "\n")
            except Exception as e:  # the reference reports and carries on
                print(f"Failed to write to APA log file {self.log_file}: {e}")

    def log_escalation(self, step: int, module_name: str, reason: str, old_level: int, new_level: int,
                       trigger_value: float):
        self._log_event({"event": "escalation", "step": step, "module": module_name, "reason": reason,
                         "old_level": old_level, "new_level": new_level,
                         "trigger_value": float(trigger_value)})

    def log_skip_batch(self, step: int, reason: str, trigger_modules: list):
        self._log_event({"event": "skip_batch", "step": step, "reason": reason,
                         "trigger_modules": trigger_modules})


class APAForensicLogger:
    """One JSON line per escalation with per-role tensor statistics
    (apa/telemetry.py:78-122). Written only when an escalation happens."""

    def __init__(self, forensic_log_file: str) -> None:
        self.forensic_log_file = forensic_log_file
        try:
            os.makedirs(os.path.dirname(os.path.abspath(forensic_log_file)), exist_ok=True)
        except Exception as e:
            print(f"[APA Forensic] Warning: could not create log directory: {e}")

    def log_forensic_event(self, record: dict) -> None:
        record = dict(record)
        record["timestamp_utc"] = _utc_now()
        line = json.dumps(record, default=str)
        print(f"[APA Forensic] {line}")
        try:
            with open(self.forensic_log_file, "a", encoding="utf-8") as fh:
                fh.write(line + "\n")
        except Exception as e:
            print(f"[APA Forensic] Warning: failed to write forensic log: {e}")

"""Torch-CPU port of the reference's ``fp8_simulation_mode`` training step.

TEST INFRASTRUCTURE AND CPU BASELINE ONLY. ``bench.py`` times this port on
the host cores as the reference arm (``--impl reference``) and as the
``cpu_baseline`` leg whenever the reference package itself is not installed
beside the repository; the CPU tests check it against the numpy oracle
(``apa_oracle``) and the golden fixtures made by running the reference. The
product never imports it.

It restates, as torch CPU operations, the work the reference does on its
simulation path, with the same operations on the same dtypes so that its
cost is the reference's cost:

* ``PortLinear``: fp32 master weight and bias, working copies made each step
  (``apa/layers.py:368-372``), a boundary-cast child module
  (``layers.py:10-21``), and the autograd function of ``layers.py:109-303``:
  telemetry passes on x_cast, W, y, dy (``telemetry.py:7-21``), fp32 GEMMs on
  E4M3-upcast operands at FP8 (``layers.py:158-163, 223-241``), working-dtype
  GEMMs at FP16 / fp32 at "TF32" (``layers.py:179-182, 267-275``), and the
  underflow ratio with its host read (``telemetry.py:23-39``,
  ``layers.py:404-407``). The autograd engine then casts each gradient to
  its input's dtype, exactly as it does for the reference.
* ``PortManager``: leaf-module backward hooks (``manager.py:70-84``),
  ``pre_step`` (``manager.py:145-172``), the gradient copy to the masters
  (``manager.py:191-204``), the hard check with its host read
  (``manager.py:178-189``) and the full evaluation with three host reads per
  module (``manager.py:206-261``), whose decisions come from
  ``apa_oracle.ladder_step``.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import apa_oracle as O

E4M3 = torch.float8_e4m3fn
WORK_DTYPE = {O.LEVEL_FP8: E4M3, O.LEVEL_FP16: torch.float16, O.LEVEL_TF32: torch.float32}
_REDUCIBLE = (torch.float32, torch.float16, torch.bfloat16)


def track(t: torch.Tensor, amax: torch.Tensor, flag: torch.Tensor) -> None:
    """Running amax and NaN/Inf flag of one tensor (telemetry.py:7-21)."""
    with torch.no_grad():
        v = (t if t.dtype in _REDUCIBLE else t.to(torch.float32)).abs().max().to(torch.float32)
        torch.maximum(amax, v, out=amax)
        torch.maximum(flag, (~torch.isfinite(v)).to(torch.int32).view(1), out=flag)


def underflow_ratio(g: torch.Tensor, vmin: float) -> torch.Tensor:
    """#(0 < |g| < vmin) / #(|g| > 0), with the host read of the nonzero
    count that the reference takes (telemetry.py:23-39)."""
    with torch.no_grad():
        a = (g if g.dtype in _REDUCIBLE else g.to(torch.float32)).abs()
        nz = a > 0
        n = nz.sum().to(torch.float32)
        if n.item() == 0:
            return torch.zeros((), dtype=torch.float32)
        return ((a < vmin) & nz).sum().to(torch.float32) / n


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xc, w, b, mod):
        ctx.mod = mod
        ctx.save_for_backward(xc, w, b)
        track(xc, mod.gpu_amax, mod.gpu_has_nonfinite)
        track(w, mod.gpu_amax, mod.gpu_has_nonfinite)
        if mod.level == O.LEVEL_FP8:
            y = F.linear(xc.to(torch.float32), w.to(torch.float32), None if b is None else b.to(torch.float32))
        else:
            y = F.linear(xc, w, b)
        track(y, mod.gpu_amax, mod.gpu_has_nonfinite)
        return y

    @staticmethod
    def backward(ctx, gy):
        xc, w, b = ctx.saved_tensors
        mod = ctx.mod
        track(gy, mod.gpu_amax, mod.gpu_has_nonfinite)
        if mod.level == O.LEVEL_FP8:
            g = gy.to(E4M3).to(torch.float32)
            xs, ws = xc.to(torch.float32), w.to(torch.float32)
        else:
            g, xs, ws = gy, xc, w
        g2 = g.reshape(-1, g.shape[-1])
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = (g @ ws).to(torch.float32)
        if ctx.needs_input_grad[1]:
            gw = (g2.t() @ xs.reshape(-1, xs.shape[-1])).to(torch.float32)
            r = underflow_ratio(gw, O.THRESHOLDS_MIN[mod.level])
            torch.maximum(mod.gpu_underflow_ratio, r, out=mod.gpu_underflow_ratio)
        if b is not None and ctx.needs_input_grad[2]:
            gb = g2.sum(dim=0).to(torch.float32)
        return gx, gw, gb, None


class _Cast(nn.Module):
    """The boundary cast: ``x.to(working dtype)``, identity when x already has it."""

    def __init__(self, parent):
        super().__init__()
        object.__setattr__(self, "parent", parent)

    def forward(self, x):
        dt = WORK_DTYPE[self.parent.level]
        return x if x.dtype == dt else x.to(dt)


class PortLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.weight_master = nn.Parameter(torch.empty(out_features, in_features))
        self.bias_master = nn.Parameter(torch.empty(out_features)) if bias else None
        # the module's own initialisation, same draws in the same order
        nn.init.kaiming_uniform_(self.weight_master, a=math.sqrt(5))
        if self.bias_master is not None:
            bound = 1.0 / math.sqrt(in_features) if in_features > 0 else 0.0
            nn.init.uniform_(self.bias_master, -bound, bound)
        self.register_buffer("gpu_amax", torch.zeros(1))
        self.register_buffer("gpu_underflow_ratio", torch.zeros(1))
        self.register_buffer("gpu_has_nonfinite", torch.zeros(1, dtype=torch.int32))
        self.level = O.LEVEL_FP8
        self.ema_underflow_ratio = 0.0
        self.weight_work: Optional[torch.Tensor] = None
        self.bias_work: Optional[torch.Tensor] = None
        self.boundary_cast = _Cast(self)

    def refresh(self):
        dt = WORK_DTYPE[self.level]
        with torch.no_grad():
            self.weight_work = self.weight_master.to(dt).requires_grad_(self.weight_master.requires_grad)
            if self.bias_master is not None:
                self.bias_work = self.bias_master.to(dt).requires_grad_(self.bias_master.requires_grad)

    def forward(self, x):
        if self.weight_work is None:
            self.refresh()
        return _LinearFn.apply(self.boundary_cast(x), self.weight_work, self.bias_work, self)


class PortManager:
    """pre_step / post_backward_sync_and_eval of the reference on PortLinear
    models; ``events`` collects the escalation / skip records (no timestamps)."""

    def __init__(self, model: nn.Module, theta: float = 0.4, alpha: float = 0.95, check_interval: int = 1):
        self.model = model
        self.theta, self.alpha, self.check_interval = theta, alpha, check_interval
        self.step_count = 0
        self.apa: Dict[str, PortLinear] = {}
        self.other: Dict[str, nn.Module] = {}
        self.events: List[dict] = []
        for name, m in model.named_modules():
            if isinstance(m, PortLinear):
                self.apa[name] = m
            elif len(list(m.children())) == 0:
                self.other[name] = m
                m.register_buffer("gpu_amax", torch.zeros(1), persistent=False)
                m.register_buffer("gpu_has_nonfinite", torch.zeros(1, dtype=torch.int32), persistent=False)

                def hook(mod, gin, gout):
                    for g in gout:
                        if g is not None:
                            track(g, mod.gpu_amax, mod.gpu_has_nonfinite)
                m.register_full_backward_hook(hook)

    def trainable(self) -> List[nn.Parameter]:
        seen, out = set(), []
        for m in self.apa.values():
            for p in (m.weight_master, m.bias_master):
                if p is not None and p.requires_grad and id(p) not in seen:
                    out.append(p)
                    seen.add(id(p))
        for p in self.model.parameters():
            if p.requires_grad and id(p) not in seen:
                out.append(p)
                seen.add(id(p))
        return out

    def pre_step(self):
        with torch.no_grad():
            for m in self.apa.values():
                m.refresh()
                m.gpu_has_nonfinite.zero_()
            for m in self.other.values():
                m.gpu_has_nonfinite.zero_()

    def _sync_grads(self):
        with torch.no_grad():
            for m in self.apa.values():
                for work, master in ((m.weight_work, m.weight_master), (m.bias_work, m.bias_master)):
                    if work is None or work.grad is None:
                        continue
                    g = work.grad.to(torch.float32)
                    if master.grad is None:
                        master.grad = g.clone()
                    else:
                        master.grad.copy_(g)

    def post_backward_sync_and_eval(self) -> bool:
        self.step_count += 1
        self._sync_grads()
        flag = torch.zeros(1, dtype=torch.int32)
        for m in list(self.apa.values()) + list(self.other.values()):
            flag.bitwise_or_(m.gpu_has_nonfinite)
        if not (flag.item() > 0 or self.step_count % self.check_interval == 0):
            return True
        apa, oth = list(self.apa.values()), list(self.other.values())
        st = O.LadderState(levels=[m.level for m in apa], ema=[m.ema_underflow_ratio for m in apa],
                           amax=[m.gpu_amax.item() for m in apa], ratio=[m.gpu_underflow_ratio.item() for m in apa],
                           flag=[m.gpu_has_nonfinite.item() for m in apa],
                           other_amax=[m.gpu_amax.item() for m in oth], other_flag=[m.gpu_has_nonfinite.item() for m in oth])
        ok, events = O.ladder_step(st, self.step_count, 1, self.theta, self.alpha, list(self.apa), list(self.other))
        for m, lv, e in zip(apa, st.levels, st.ema):
            m.level, m.ema_underflow_ratio = lv, e
            m.gpu_amax.zero_()
            m.gpu_underflow_ratio.zero_()
            m.gpu_has_nonfinite.zero_()
        for m in oth:
            m.gpu_amax.zero_()
            m.gpu_has_nonfinite.zero_()
        self.events.extend(events)
        return ok

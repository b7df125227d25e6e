"""Generate the golden fixtures in this folder by running the reference itself.

Run in a container that has the reference checkout (read-only) and torch:

    python tests/golden/make_golden.py /path/to/reference [fixture ...]

(or set APA_REFERENCE_DIR instead of the first argument). With fixture names
(casts, underflow, linear_small, ladder, cfg0_trajectory, cfg1_variants) only
those are regenerated.

It imports the reference's ``apa`` package from that checkout, drives it on
CPU with ``fp8_simulation_mode=True`` (the reference's CPU path) and writes:

* ``casts.npz``       element conversions as torch performs them for the
                      reference (``x.to(dtype)``): exhaustive over bf16 and
                      fp16 inputs, every E4M3 byte, and fp32 edge/random values.
* ``underflow.json``  ``compute_underflow_ratio`` on seeded tensors.
* ``linear_small.npz`` APALinear forward+backward per rung on small ragged
                      shapes: outputs, grads, telemetry buffers.
* ``ladder.json``     APAManager evaluations on injected buffer values.
* ``cfg0_trajectory.json`` the quick-start MLP run (200 steps, two input
                      spikes): escalation events, skipped steps, final levels.
* ``cfg1_variants.json`` the single 8192x4096x4096 APALinear (check_interval
                      1): the outlier variant's first step and the underflow
                      variant run until its SILENT_UNDERFLOW escalation: per
                      step underflow ratio, events and skipped steps.

The fixtures are small; the GPU box never runs this script.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
_ARGS = [a for a in sys.argv[1:]]
REF = os.environ.get("APA_REFERENCE_DIR") or (_ARGS.pop(0) if _ARGS else None)
if not REF or not os.path.isdir(os.path.join(REF, "apa")):
    sys.exit("usage: make_golden.py /path/to/reference [fixture ...]  (or set APA_REFERENCE_DIR)")
sys.path.insert(0, REF)

import apa  # noqa: E402  (the reference package)
from apa import APAConfig, APALinear, APAManager  # noqa: E402
from apa.telemetry import compute_underflow_ratio  # noqa: E402
import apa.telemetry as ref_telemetry  # noqa: E402

assert os.path.abspath(os.path.dirname(apa.__file__)).startswith(os.path.abspath(REF)), apa.__file__


def u16(t):
    return t.view(torch.int16).numpy().view(np.uint16)


def u8(t):
    return t.view(torch.uint8).numpy()


def casts():
    out = {}
    # every bf16 pattern -> e4m3 / fp16 / fp32
    bf = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    out["bf16_all_to_e4m3"] = u8(bf.to(torch.float8_e4m3fn))
    out["bf16_all_to_f16"] = u16(bf.to(torch.float16))
    # every fp16 pattern -> e4m3 / bf16
    hf = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.float16)
    out["f16_all_to_e4m3"] = u8(hf.to(torch.float8_e4m3fn))
    out["f16_all_to_bf16"] = u16(hf.to(torch.bfloat16))
    # every e4m3 byte -> fp32 / bf16 / fp16
    e8 = torch.arange(0, 256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn)
    out["e4m3_all_to_f32"] = e8.to(torch.float32).view(torch.int32).numpy().view(np.uint32)
    out["e4m3_all_to_bf16"] = u16(e8.to(torch.bfloat16))
    out["e4m3_all_to_f16"] = u16(e8.to(torch.float16))
    # fp32 inputs: edges of every rounding boundary plus seeded randoms
    rng = np.random.default_rng(1234)
    hi = np.arange(0, 1 << 12, dtype=np.uint32) << 20              # every sign/exponent/3 mantissa bits
    lows = np.array([0, 1, 0x7FFFF, 0x80000, 0x80001, 0xFFFFF, 0x3FFFF, 0x40000, 0x40001,
                     0xFFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0x2001], dtype=np.uint32)
    edge = (hi[:, None] | lows[None, :]).ravel()
    rnd = rng.integers(0, 1 << 32, size=1 << 18, dtype=np.uint64).astype(np.uint32)
    f32_bits = np.concatenate([edge, rnd])
    f = torch.from_numpy(f32_bits.view(np.int32).copy()).view(torch.float32)
    out["f32_in_bits"] = f32_bits
    out["f32_to_e4m3"] = u8(f.to(torch.float8_e4m3fn))
    out["f32_to_f16"] = u16(f.to(torch.float16))
    out["f32_to_bf16"] = u16(f.to(torch.bfloat16))
    np.savez_compressed(os.path.join(HERE, "casts.npz"), **out)


def underflow():
    rng = np.random.default_rng(7)
    cases = []
    for level, vmin in sorted(apa.config.THRESHOLDS_MIN.items()):
        for scale in (1e-6, 1e-4, 1e-3, 1e-2, 1.0):
            g = (rng.standard_normal(257) * scale).astype(np.float32)
            g[::7] = 0.0
            r = compute_underflow_ratio(torch.from_numpy(g.copy()), vmin).item()
            cases.append(dict(level=level, vmin=vmin, g=g.tolist(), ratio=r))
    # boundary: exactly the fp32 threshold and its neighbours
    for vmin in (0.015625, 6.1035e-5):
        t = np.float32(vmin)
        g = np.array([t, np.nextafter(t, np.float32(0)), np.nextafter(t, np.float32(1)), 0.0, -t,
                      np.float32(np.nan), np.float32(np.inf)], dtype=np.float32)
        r = compute_underflow_ratio(torch.from_numpy(g.copy()), vmin).item()
        cases.append(dict(level=-1, vmin=vmin, g=[float(v) for v in g], ratio=r))
    with open(os.path.join(HERE, "underflow.json"), "w") as fh:
        json.dump(cases, fh)


SHAPES = [(64, 96, 80), (17, 48, 10), (1, 16, 16), (130, 272, 65), (33, 40, 24)]


def linear_small():
    out = {}
    rng = np.random.default_rng(2024)
    idx = 0
    for (M, K, N) in SHAPES:
        for level in (0, 1, 2):
            for xdt in ("bf16", "f32"):
                for bias in (True, False):
                    if (M, K, N) != (64, 96, 80) and not bias:
                        continue
                    cfg = APAConfig(fp8_simulation_mode=True, device="cpu", check_interval=1)
                    lin = APALinear(K, N, bias=bias, config=cfg)
                    model = nn.Sequential(lin)
                    mgr = APAManager(model, cfg)
                    W = (rng.standard_normal((N, K)) * rng.choice([0.05, 0.3, 2.0])).astype(np.float32)
                    b = (rng.standard_normal(N) * 0.5).astype(np.float32) if bias else None
                    with torch.no_grad():
                        lin.weight_master.copy_(torch.from_numpy(W))
                        if bias:
                            lin.bias_master.copy_(torch.from_numpy(b))
                    lin.level = level
                    mgr.pre_step()
                    x = torch.from_numpy((rng.standard_normal((M, K)) * rng.choice([0.1, 1.0, 30.0])).astype(np.float32))
                    if xdt == "bf16":
                        x = x.to(torch.bfloat16)
                    x.requires_grad_(True)
                    y = lin(x)
                    dy = torch.from_numpy((rng.standard_normal((M, N)) * rng.choice([1e-3, 0.05, 1.0])).astype(np.float32))
                    dy = dy.to(y.dtype)
                    y.backward(dy)
                    mgr._sync_grads_to_master()
                    p = f"c{idx}_"
                    out[p + "meta"] = np.array([M, K, N, level, 1 if xdt == "bf16" else 0, 1 if bias else 0])
                    out[p + "x"] = x.detach().float().numpy()
                    out[p + "W"] = W
                    if bias:
                        out[p + "b"] = b
                        out[p + "db"] = lin.bias_master.grad.numpy()
                    out[p + "dy"] = dy.float().numpy()
                    out[p + "y"] = y.detach().float().numpy()
                    out[p + "dx"] = x.grad.float().numpy()
                    out[p + "dW"] = lin.weight_master.grad.numpy()
                    out[p + "tele"] = np.array([lin.gpu_amax.item(), lin.gpu_has_nonfinite.item(),
                                                lin.gpu_underflow_ratio.item(),
                                                lin.boundary_cast.gpu_amax.item(),
                                                lin.boundary_cast.gpu_has_nonfinite.item()], dtype=np.float64)
                    idx += 1
    out["count"] = np.array([idx])
    np.savez_compressed(os.path.join(HERE, "linear_small.npz"), **out)


def _capture_events():
    events = []

    def cap(self, d):
        d = dict(d)
        d.pop("timestamp", None)
        events.append(d)

    ref_telemetry.APAEventLogger._log_event = cap
    return events


def ladder():
    """Random manager evaluations with injected buffer values."""
    events = _capture_events()
    rng = np.random.default_rng(99)
    cases = []
    for case in range(300):
        cfg = APAConfig(fp8_simulation_mode=True, device="cpu",
                        check_interval=int(rng.choice([1, 2, 4])),
                        theta_underflow=float(rng.choice([0.3, 0.4, 0.5])),
                        ema_alpha=float(rng.choice([0.95, 0.9])))
        L = int(rng.integers(1, 5))
        model = nn.Sequential(*[APALinear(8, 8, config=cfg) for _ in range(L)], nn.LayerNorm(8), nn.GELU())
        mgr = APAManager(model, cfg)
        names = list(mgr.apa_modules.keys())
        onames = list(mgr.other_modules.keys())
        steps = int(rng.integers(1, 6))
        mgr.step_count = int(rng.integers(0, 8))
        init = dict(levels=[int(rng.integers(0, 3)) for _ in range(L)],
                    ema=[float(rng.choice([0.0, 0.2, 0.39, 0.41, 0.6])) for _ in range(L)],
                    step_count=mgr.step_count)
        for i, m in enumerate(mgr.apa_modules.values()):
            m.level = init["levels"][i]
            m.ema_underflow_ratio = init["ema"][i]
        seq = []
        for s in range(steps):
            mgr.pre_step()
            inj = dict(amax=[], ratio=[], flag=[], oamax=[], oflag=[])
            for m in mgr.apa_modules.values():
                a = float(rng.choice([0.0, 1.0, 403.2, 403.3, 58953.6, 58953.7, 1e6, np.inf, np.nan,
                                      float(rng.uniform(0, 500))]))
                r = float(np.float32(rng.choice([0.0, 0.35, 0.45, 0.9, float(rng.uniform(0, 1))])))
                f = int(rng.random() < 0.15)
                m.gpu_amax.fill_(max(m.gpu_amax.item(), a) if not math.isnan(a) else a)
                m.gpu_underflow_ratio.fill_(max(m.gpu_underflow_ratio.item(), r))
                if f:
                    m.gpu_has_nonfinite.fill_(1)
                inj["amax"].append(m.gpu_amax.item()); inj["ratio"].append(m.gpu_underflow_ratio.item())
                inj["flag"].append(int(m.gpu_has_nonfinite.item()))
            for m in mgr.other_modules.values():
                a = float(rng.choice([0.0, 2.0, 500.0, 70000.0, np.inf, np.nan]))
                f = int(rng.random() < 0.1)
                m.gpu_amax.fill_(max(m.gpu_amax.item(), a) if not math.isnan(a) else a)
                if f:
                    m.gpu_has_nonfinite.fill_(1)
                inj["oamax"].append(m.gpu_amax.item()); inj["oflag"].append(int(m.gpu_has_nonfinite.item()))
            events.clear()
            ok = mgr.post_backward_sync_and_eval()
            seq.append(dict(inject=inj, should_step=bool(ok), events=list(events),
                            levels=[m.level for m in mgr.apa_modules.values()],
                            ema=[m.ema_underflow_ratio for m in mgr.apa_modules.values()],
                            amax=[m.gpu_amax.item() for m in mgr.apa_modules.values()],
                            ratio=[m.gpu_underflow_ratio.item() for m in mgr.apa_modules.values()],
                            flag=[m.gpu_has_nonfinite.item() for m in mgr.apa_modules.values()],
                            oamax=[m.gpu_amax.item() for m in mgr.other_modules.values()],
                            oflag=[m.gpu_has_nonfinite.item() for m in mgr.other_modules.values()]))
        cases.append(dict(check_interval=cfg.check_interval, theta=cfg.theta_underflow,
                          alpha=cfg.ema_alpha, names=names, other_names=onames, init=init, seq=seq))
    with open(os.path.join(HERE, "ladder.json"), "w") as fh:
        json.dump(cases, fh, allow_nan=True)


CFG0_SPIKES = (50, 150)


def cfg0_trajectory():
    """Quick-start MLP: APALinear(768,768) -> ReLU -> LayerNorm -> APALinear(768,10);
    AdamW lr 1e-3, research_default, one fixed seeded batch of 64, 200 steps;
    at steps 50 and 150 (0-based) 49 seeded elements (0.1%) are scaled by 1e3."""
    events = _capture_events()
    torch.manual_seed(0)
    cfg = APAConfig.research_default(fp8_simulation_mode=True, device="cpu")

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = APALinear(768, 768, config=cfg)
            self.relu = nn.ReLU()
            self.norm = nn.LayerNorm(768)
            self.fc2 = APALinear(768, 10, config=cfg)

        def forward(self, x):
            return self.fc2(self.norm(self.relu(self.fc1(x))))

    m = MLP()
    W0 = {k: v.detach().clone() for k, v in m.state_dict().items()}
    mgr = APAManager(m, cfg)
    opt = torch.optim.AdamW(mgr.get_trainable_parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(0)
    x0 = torch.randn(64, 768, generator=g)
    y0 = torch.randint(0, 10, (64,), generator=g)
    spikes = {}
    for s in CFG0_SPIKES:
        spikes[s] = torch.randperm(x0.numel(), generator=g)[:49]
    skips, losses, levels = [], [], []
    for step in range(200):
        x = x0.clone()
        if step in spikes:
            x.view(-1)[spikes[step]] *= 1e3
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        loss = F.cross_entropy(m(x), y0)
        loss.backward()
        ok = mgr.post_backward_sync_and_eval()
        if ok:
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
            skips.append(step)
        losses.append(loss.item())
        levels.append([m.fc1.level, m.fc2.level])
    res = dict(spike_steps=list(CFG0_SPIKES), spike_idx={str(k): v.tolist() for k, v in spikes.items()},
               events=events, skips=skips, losses=losses, levels=levels,
               w0_checksum={k: float(v.double().sum()) for k, v in W0.items()})
    with open(os.path.join(HERE, "cfg0_trajectory.json"), "w") as fh:
        json.dump(res, fh, allow_nan=True)


def _cfg1_layer():
    """The cfg1 layer as the bench builds it: APALinear(4096, 4096) initialised
    under torch.manual_seed(0), default config with check_interval 1."""
    torch.manual_seed(0)
    cfg = APAConfig(fp8_simulation_mode=True, device="cpu", check_interval=1)
    lin = APALinear(4096, 4096, config=cfg)
    return lin, APAManager(nn.Sequential(lin), cfg)


def cfg1_inputs(variant):
    """cfg1 variant inputs from CPU generators: x [8192, 4096] N(0,1) (seed 0)
    and dy N(0,1) (seed 1), in bf16 / fp32.
    outlier: 0.05 % of x (a randperm of the same generator) scaled by 500;
    underflow: a rand() < 0.5 mask of the same generator selects elements of
    x scaled by 1e-4, and dy is scaled by 5e-4."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(8192, 4096, generator=g)
    if variant == "outlier":
        n = int(x.numel() * 0.0005)
        idx = torch.randperm(x.numel(), generator=g)[:n]
        x.view(-1)[idx] *= 500
        dscale = 1.0
    else:
        mask = torch.rand(8192, 4096, generator=g) < 0.5
        x = torch.where(mask, x * 1e-4, x)
        dscale = 5e-4
    dy = torch.randn(8192, 4096, generator=torch.Generator().manual_seed(1)) * dscale
    return x.to(torch.bfloat16), dy


def cfg1_variants(max_steps=80):
    events = _capture_events()
    out = {}
    for variant in ("outlier", "underflow"):
        lin, mgr = _cfg1_layer()
        x, dy = cfg1_inputs(variant)
        x.requires_grad_(True)
        events.clear()
        ratios, skips, nevents = [], [], 0
        for step in range(1, max_steps + 1):
            mgr.pre_step()
            lin(x).backward(dy)
            x.grad = None
            ratios.append(lin.gpu_underflow_ratio.item())
            amax = lin.gpu_amax.item()
            if not mgr.post_backward_sync_and_eval():
                skips.append(step)
            if lin.level > 0:
                break
        out[variant] = dict(events=list(events), ratios=ratios, skips=skips, steps=step, level=lin.level,
                            first_amax=amax if step == 1 else None)
    with open(os.path.join(HERE, "cfg1_variants.json"), "w") as fh:
        json.dump(out, fh, allow_nan=True)


if __name__ == "__main__":
    todo = _ARGS or ["casts", "underflow", "linear_small", "ladder", "cfg0_trajectory", "cfg1_variants"]
    for name in todo:
        globals()[name]()
    print("golden fixtures written to", HERE, ":", ", ".join(todo))

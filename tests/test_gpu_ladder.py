"""Device ladder (apa_ladder_eval) driven through APAManager on the 300
injected-telemetry scenarios the reference itself evaluated
(tests/golden/ladder.json): identical skip decisions, levels, EMAs (exact
doubles), buffer resets and logged events."""
import json
import math
import os

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")

with open(os.path.join(G, "ladder.json")) as fh:
    CASES = json.load(fh)


def _same(a, b):
    if isinstance(b, float) and math.isnan(b):
        return isinstance(a, float) and math.isnan(a)
    return a == b


@pytest.mark.parametrize("ci", range(0, len(CASES), 1))
def test_ladder_case(ci):
    from apa import APAConfig, APALinear, APAManager
    c = CASES[ci]
    cfg = APAConfig(device="cuda", check_interval=c["check_interval"], theta_underflow=c["theta"],
                    ema_alpha=c["alpha"])
    L = len(c["names"])
    model = nn.Sequential(*[APALinear(8, 8, config=cfg) for _ in range(L)], nn.LayerNorm(8), nn.GELU()).cuda()
    mgr = APAManager(model, cfg)
    assert list(mgr.apa_modules) == c["names"] and list(mgr.other_modules) == c["other_names"]
    events = []
    mgr.logger._log_event = lambda d: events.append({k: v for k, v in d.items() if k != "timestamp"})
    mgr.step_count = c["init"]["step_count"]
    for m, lv, e in zip(mgr.apa_modules.values(), c["init"]["levels"], c["init"]["ema"]):
        m.level = lv
        m.ema_underflow_ratio = e
    for s in c["seq"]:
        mgr.pre_step()
        inj = s["inject"]
        for m, a, r, f in zip(mgr.apa_modules.values(), inj["amax"], inj["ratio"], inj["flag"]):
            m.gpu_amax.fill_(a)
            m.gpu_underflow_ratio.fill_(r)
            m.gpu_has_nonfinite.fill_(f)
        for m, a, f in zip(mgr.other_modules.values(), inj["oamax"], inj["oflag"]):
            m.gpu_amax.fill_(a)
            m.gpu_has_nonfinite.fill_(f)
        events.clear()
        ok = mgr.post_backward_sync_and_eval()
        assert ok == s["should_step"]
        assert [m.level for m in mgr.apa_modules.values()] == s["levels"]
        assert [m.ema_underflow_ratio for m in mgr.apa_modules.values()] == s["ema"]
        got_amax = [m.gpu_amax.item() for m in mgr.apa_modules.values()]
        assert all(_same(a, b) for a, b in zip(got_amax, s["amax"]))
        assert [m.gpu_underflow_ratio.item() for m in mgr.apa_modules.values()] == pytest.approx(s["ratio"])
        assert [m.gpu_has_nonfinite.item() for m in mgr.apa_modules.values()] == s["flag"]
        assert [m.gpu_has_nonfinite.item() for m in mgr.other_modules.values()] == s["oflag"]
        assert len(events) == len(s["events"])
        for a, b in zip(events, s["events"]):
            assert set(a) == set(b)
            for k in b:
                assert _same(a[k], b[k]), (k, a, b)

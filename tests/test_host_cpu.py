"""Host-side behaviour that needs no GPU: config presets and defaults,
forensic file derivation, constants, module construction and discovery."""
import math

import pytest
import torch
import torch.nn as nn


def test_constants_match_reference():
    from apa import config as C
    assert (C.LEVEL_FP8, C.LEVEL_FP16, C.LEVEL_TF32) == (0, 1, 2)
    assert C.THRESHOLDS_MAX[0] == 0.90 * 448.0 and C.THRESHOLDS_MAX[1] == 0.90 * 65504.0
    assert math.isinf(C.THRESHOLDS_MAX[2])
    assert C.THRESHOLDS_MIN == {0: 0.015625, 1: 6.1035e-5, 2: 0.0}
    assert C.DTYPE_MAP[0] == torch.float8_e4m3fn and C.DTYPE_MAP[1] == torch.float16


def test_presets_and_defaults():
    from apa import APAConfig
    d = APAConfig()
    assert (d.gamma, d.theta_underflow, d.ema_alpha, d.check_interval, d.device) == (0.9, 0.4, 0.95, 1, "cuda")
    c = APAConfig.conservative()
    assert (c.gamma, c.theta_underflow, c.check_interval) == (0.8, 0.3, 1)
    a = APAConfig.aggressive(check_interval=3)
    assert (a.gamma, a.theta_underflow, a.check_interval) == (0.95, 0.5, 3)
    r = APAConfig.research_default()
    assert (r.gamma, r.theta_underflow, r.check_interval) == (0.9, 0.4, 4)


@pytest.mark.parametrize("log,expect", [("a/b/log.jsonl", "a/b/log_forensic.jsonl"),
                                        ("noext", "noext_forensic.jsonl"),
                                        ("x.y.z", "x.y_forensic.jsonl"),
                                        (None, "apa_forensic.jsonl")])
def test_forensic_file_derivation(log, expect):
    from apa import APAConfig
    c = APAConfig(log_file=log, enable_forensic_logging=True)
    assert c.forensic_log_file == expect
    assert APAConfig(log_file=log).forensic_log_file is None


def test_module_discovery_and_state_dict_on_cpu_construction():
    """Construction needs no GPU; the same seed gives the same weights as
    nn.Linear's initialisation rule on the CPU generator."""
    from apa import APAConfig, APALinear, APAManager
    cfg = APAConfig(device="cpu")
    torch.manual_seed(3)
    lin = APALinear(32, 8, config=cfg)
    torch.manual_seed(3)
    ref = nn.Linear(32, 8)
    assert torch.equal(lin.weight_master, ref.weight) and torch.equal(lin.bias_master, ref.bias)
    model = nn.Sequential(nn.Embedding(10, 32), lin, nn.LayerNorm(8))
    mgr = APAManager(model, cfg)
    assert list(mgr.apa_modules) == ["1"]
    assert list(mgr.other_modules) == ["0", "1.boundary_cast", "2"]
    assert len(mgr.get_trainable_parameters()) == 5
    assert set(lin.state_dict()) == {"weight_master", "bias_master", "gpu_amax", "gpu_underflow_ratio",
                                     "gpu_has_nonfinite"}


def test_no_cpu_compute_path():
    """The product refuses to compute on CPU tensors instead of falling back."""
    from apa import APAConfig, APALinear
    from apa._lib import APAKernelError
    lin = APALinear(16, 16, config=APAConfig(device="cpu"))
    with pytest.raises(APAKernelError):
        lin(torch.randn(2, 16))


def test_apa_adamw_host_path_matches_torch_adamw():
    """APAAdamW's bookkeeping without the fused kernel (CPU parameters: every
    weight takes torch's update): same parameters and state as
    torch.optim.AdamW over several steps, bit for bit, and no fused update
    counted."""
    from apa import APAConfig, APALinear, APAManager
    from apa.optim import APAAdamW
    cfg = APAConfig(device="cpu")
    torch.manual_seed(0)
    model = nn.Sequential(APALinear(12, 8, config=cfg), nn.LayerNorm(8), APALinear(8, 4, config=cfg))
    mgr = APAManager(model, cfg)
    params = mgr.get_trainable_parameters()
    twins = [p.detach().clone().requires_grad_(True) for p in params]
    opt = APAAdamW(mgr, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    ref = torch.optim.AdamW(twins, lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    g = torch.Generator().manual_seed(1)
    for _ in range(4):
        for p, t in zip(params, twins):
            grad = torch.randn(p.shape, generator=g)
            p.grad = grad.clone()
            t.grad = grad.clone()
        opt.step()
        ref.step()
    for p, t in zip(params, twins):
        assert torch.equal(p.detach(), t.detach())
        assert torch.equal(opt.state[p]["exp_avg"], ref.state[t]["exp_avg"])
        assert torch.equal(opt.state[p]["exp_avg_sq"], ref.state[t]["exp_avg_sq"])
        assert float(opt.state[p]["step"]) == float(ref.state[t]["step"]) == 4.0
    assert opt.fused_steps == 0


def test_event_log_lines_match_reference_records(tmp_path):
    """The event logger writes the reference's JSONL records (telemetry.py:41-75):
    the same keys in the same order and the same values as the events the
    reference logged on the cfg0 trajectory, plus a timestamp."""
    import json
    import os
    from apa.telemetry import APAEventLogger
    golden = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "cfg0_trajectory.json")))
    log = tmp_path / "events.jsonl"
    lg = APAEventLogger(str(log))
    for e in golden["events"]:
        if e["event"] == "escalation":
            lg.log_escalation(e["step"], e["module"], e["reason"], e["old_level"], e["new_level"], e["trigger_value"])
        else:
            lg.log_skip_batch(e["step"], e["reason"], e["trigger_modules"])
    got = [json.loads(line) for line in open(log)]
    assert len(got) == len(golden["events"])
    for g, e in zip(got, golden["events"]):
        assert list(g)[:-1] == list(e) and list(g)[-1] == "timestamp"
        for k, v in e.items():
            if isinstance(v, float) and math.isnan(v):
                assert math.isnan(g[k])
            else:
                assert g[k] == v, k

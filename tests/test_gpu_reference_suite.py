"""The reference's own behavioural tests (tests/test_escalation.py,
test_hard_overflow.py, test_underflow.py, test_parameter_registry.py,
test_smoke.py, test_forensic_logging.py), restated for this package on the
CUDA device. The reference ran them on CPU with fp8_simulation_mode=True;
that flag is still accepted (and ignored: there is one compute path)."""
import json
import os
import tempfile

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture
def apa():
    import apa as pkg
    return pkg


def one_layer(apa, **kw):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, **kw)
    mod = apa.APALinear(16, 16, config=cfg)
    model = nn.Sequential(mod)
    return cfg, mod, model, apa.APAManager(model, config=cfg)


# ---- tests/test_escalation.py ------------------------------------------------
def test_escalation_ladder(apa):
    from apa.config import LEVEL_FP8, LEVEL_FP16, LEVEL_TF32, DTYPE_MAP
    cfg, mod, model, mgr = one_layer(apa)
    assert mod.level == LEVEL_FP8
    mgr._escalate_module("0", mod, "OVERFLOW", 999.0)
    assert mod.level == LEVEL_FP16
    mgr._escalate_module("0", mod, "OVERFLOW", 999.0)
    assert mod.level == LEVEL_TF32
    mgr._escalate_module("0", mod, "OVERFLOW", 999.0)
    assert mod.level == LEVEL_TF32
    mod.level = LEVEL_FP8
    assert mod.working_dtype == DTYPE_MAP[LEVEL_FP8]
    mod.level = LEVEL_FP16
    assert mod.working_dtype == torch.float16
    mod.refresh_working_copy()
    assert mod.weight_work.dtype == torch.float16
    mod.level = LEVEL_TF32
    assert mod.working_dtype == torch.float32
    mod.refresh_working_copy()
    assert mod.weight_work.dtype == torch.float32


# ---- tests/test_hard_overflow.py ---------------------------------------------
@pytest.mark.parametrize("bad", [float("nan"), float("inf"), float("-inf")])
def test_nonfinite_sets_flag(apa, bad):
    _, mod, _, _ = one_layer(apa)
    mod.track_telemetry(torch.tensor([1.0, bad, 3.0], device=DEV))
    assert mod.gpu_has_nonfinite.item() > 0


def test_normal_values_no_flag_and_accumulation(apa):
    _, mod, _, mgr = one_layer(apa)
    mod.track_telemetry(torch.tensor([1.0, 2.0, 3.0], device=DEV))
    assert mod.gpu_has_nonfinite.item() == 0
    mod.track_telemetry(torch.tensor([float("nan")], device=DEV))
    mod.track_telemetry(torch.tensor([3.0, 4.0], device=DEV))
    assert mod.gpu_has_nonfinite.item() > 0
    mgr.pre_step()
    assert mod.gpu_has_nonfinite.item() == 0


def test_pre_step_keeps_amax_and_nan_skips(apa):
    _, mod, _, mgr = one_layer(apa)
    mod.track_telemetry(torch.tensor([100.0, -200.0], device=DEV))
    assert mod.gpu_amax.item() >= 200.0
    mgr.pre_step()
    assert mod.gpu_amax.item() >= 200.0
    mgr.pre_step()
    mod.track_telemetry(torch.tensor([1.0, float("nan")], device=DEV))
    assert mgr.post_backward_sync_and_eval() is False


# ---- tests/test_underflow.py ---------------------------------------------------
def test_underflow_ratio_values(apa):
    from apa.telemetry import compute_underflow_ratio
    from apa.config import THRESHOLDS_MIN, LEVEL_FP8
    v = THRESHOLDS_MIN[LEVEL_FP8]
    f = lambda t: compute_underflow_ratio(t.to(DEV), v).item()
    assert f(torch.full((10,), v / 2)) == pytest.approx(1.0)
    assert f(torch.full((10,), v * 2)) == pytest.approx(0.0)
    assert f(torch.cat([torch.full((5,), v / 2), torch.full((5,), v * 2)])) == pytest.approx(0.5)
    assert f(torch.cat([torch.full((5,), v / 2), torch.zeros(5)])) == pytest.approx(1.0)


def test_underflow_running_max_and_no_skip(apa):
    from apa.config import THRESHOLDS_MIN, LEVEL_FP8
    cfg, mod, _, mgr = one_layer(apa)
    v = THRESHOLDS_MIN[LEVEL_FP8]
    t = torch.full((100,), v / 2, device=DEV)
    for _ in range(50):
        mod.update_underflow_metric(t)
    assert mod.gpu_underflow_ratio.item() >= 0.9
    mgr.pre_step()
    mod.ema_underflow_ratio = cfg.theta_underflow + 0.1
    mod.gpu_underflow_ratio.fill_(cfg.theta_underflow + 0.1)
    assert mgr.post_backward_sync_and_eval() is True
    assert mod.level == 1


# ---- tests/test_parameter_registry.py ------------------------------------------
def test_parameter_registry(apa):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV)

    class TestModel(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(100, 64)
            self.linear1 = apa.APALinear(64, 128, config=cfg)
            self.norm = nn.LayerNorm(128)
            self.linear2 = apa.APALinear(128, 10, config=cfg)

    model = TestModel().to(DEV)
    mgr = apa.APAManager(model, config=cfg)
    mgr.pre_step()
    params = mgr.get_trainable_parameters()
    ids = [id(p) for p in params]
    for p in (model.linear1.weight_master, model.linear1.bias_master, model.linear2.weight_master,
              model.linear2.bias_master, model.norm.weight, model.norm.bias, model.embed.weight):
        assert id(p) in ids
    assert id(model.linear1.weight_work) not in ids and id(model.linear1.bias_work) not in ids
    assert len(params) == 7 and all(p.requires_grad for p in params)


# ---- tests/test_smoke.py --------------------------------------------------------
class SmokeModel(nn.Module):
    def __init__(self, apa, cfg):
        super().__init__()
        self.linear1 = apa.APALinear(16, 16, config=cfg)
        self.linear2 = apa.APALinear(16, 2, config=cfg)

    def forward(self, x):
        return self.linear2(torch.relu(self.linear1(x)))


def _train(apa, cfg, model, steps, x_scale, lr):
    mgr = apa.APAManager(model, config=cfg)
    opt = torch.optim.SGD(mgr.get_trainable_parameters(), lr=lr)
    for _ in range(steps):
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        loss = model(torch.randn(8, 16, device=DEV) * x_scale).sum()
        loss.backward()
        if mgr.post_backward_sync_and_eval():
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
        if model.linear1.level > 0 or model.linear2.level > 0:
            return True
    return False


def test_forced_overflow_escalation(apa):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1)
    model = SmokeModel(apa, cfg)
    nn.init.constant_(model.linear1.weight_master, 400.0)
    assert _train(apa, cfg, model, 5, 1.0, 0.1)


def test_normal_training_no_escalation(apa):
    """The reference's version draws unseeded data and is borderline by
    construction (after 10 steps the EMA is 0.4013 x the mean underflow ratio,
    whose mean is close to 1): run on CPU it escalates for about 1 seed in 15.
    Here weights, biases and inputs come from a fixed CPU generator (seed 1);
    the reference, run on exactly these values, ends with fc1's EMA at 0.3836
    and no escalation."""
    g = torch.Generator().manual_seed(1)
    W1 = torch.empty(16, 16).normal_(0, 0.01, generator=g)
    b1 = (torch.rand(16, generator=g) - 0.5) * 0.5
    W2 = torch.empty(2, 16).normal_(0, 0.01, generator=g)
    b2 = (torch.rand(2, generator=g) - 0.5) * 0.5
    xs = [torch.randn(8, 16, generator=g) * 0.1 for _ in range(10)]
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1)
    l1 = apa.APALinear(16, 16, config=cfg)
    l2 = apa.APALinear(16, 2, config=cfg)
    with torch.no_grad():
        l1.weight_master.copy_(W1); l1.bias_master.copy_(b1)
        l2.weight_master.copy_(W2); l2.bias_master.copy_(b2)
    model = nn.Sequential(l1, nn.ReLU(), l2)
    mgr = apa.APAManager(model, config=cfg)
    opt = torch.optim.SGD(mgr.get_trainable_parameters(), lr=0.001)
    for x in xs:
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        model(x.to(DEV)).sum().backward()
        if mgr.post_backward_sync_and_eval():
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
    assert l1.level == 0 and l2.level == 0
    assert l1.ema_underflow_ratio == pytest.approx(0.3836, abs=0.01)


def test_check_interval_window_accumulation(apa):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=4)
    model = SmokeModel(apa, cfg)
    mgr = apa.APAManager(model, config=cfg)
    mgr.pre_step()
    model.linear1.track_telemetry(torch.tensor([100000.0], device=DEV))
    mgr.post_backward_sync_and_eval()
    for _ in range(2):
        mgr.pre_step()
        model.linear1.track_telemetry(torch.tensor([1.0], device=DEV))
        mgr.post_backward_sync_and_eval()
    assert model.linear1.level == 0
    mgr.pre_step()
    model.linear1.track_telemetry(torch.tensor([1.0], device=DEV))
    mgr.post_backward_sync_and_eval()
    assert model.linear1.level > 0


def test_skip_batch_on_flag(apa):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1)
    model = SmokeModel(apa, cfg)
    mgr = apa.APAManager(model, config=cfg)
    mgr.pre_step()
    model(torch.randn(8, 16, device=DEV)).sum().backward()
    model.linear1.gpu_has_nonfinite.fill_(1)
    assert mgr.post_backward_sync_and_eval() is False


def test_escalation_log_file(apa, tmp_path):
    log = str(tmp_path / "log.jsonl")
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1, log_file=log)
    model = SmokeModel(apa, cfg)
    mgr = apa.APAManager(model, config=cfg)
    mgr.pre_step()
    model.linear1.gpu_has_nonfinite.fill_(1)
    model.linear1.gpu_amax.fill_(float("inf"))
    mgr.post_backward_sync_and_eval()
    with open(log) as fh:
        data = json.loads(fh.readline())
    for k in ("module", "old_level", "new_level", "reason"):
        assert k in data


# ---- tests/test_forensic_logging.py ---------------------------------------------
def _two(apa, cfg):
    return nn.Sequential(apa.APALinear(16, 16, config=cfg), apa.APALinear(16, 8, config=cfg))


def _overflow_step(mgr):
    mgr.pre_step()
    list(mgr.apa_modules.values())[0].gpu_amax.fill_(500.0)
    mgr.post_backward_sync_and_eval()


def test_forensic_off_by_default(apa, tmp_path):
    log = str(tmp_path / "apa_log.jsonl")
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, log_file=log)
    assert not cfg.enable_forensic_logging and cfg.forensic_log_file is None
    mgr = apa.APAManager(_two(apa, cfg), cfg)
    _overflow_step(mgr)
    assert not os.path.exists(str(tmp_path / "apa_log_forensic.jsonl"))
    assert mgr.forensic_logger is None and len(mgr._forward_hook_handles) == 0


def test_forensic_records(apa, tmp_path):
    log = str(tmp_path / "apa_log.jsonl")
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1, log_file=log,
                        enable_forensic_logging=True)
    assert cfg.forensic_log_file == str(tmp_path / "apa_log_forensic.jsonl")
    mgr = apa.APAManager(_two(apa, cfg), cfg)
    for _ in range(3):
        _overflow_step(mgr)
    with open(cfg.forensic_log_file, encoding="utf-8") as fh:
        records = [json.loads(line) for line in fh if line.strip()]
    assert records
    required = {"step", "timestamp_utc", "module_name", "reason", "level_before", "level_after",
                "culprit_tensor_role", "per_role_amax", "amax_value", "threshold_at_time", "tensor_shape",
                "dtype_at_time", "preceding_module_in_forward_order", "underflow_ratio", "argmax_flat_index"}
    for r in records:
        assert required <= set(r)
        assert r["culprit_tensor_role"] in {"input_activation", "weight", "output", "grad_output",
                                            "grad_weight", "grad_input", None}
        assert isinstance(r["per_role_amax"], dict)
    assert records[0]["level_before"] == "FP8" and records[0]["level_after"] == "FP16"


def test_forensic_no_file_without_escalation_and_order_reset(apa, tmp_path):
    cfg = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=1,
                        log_file=str(tmp_path / "l.jsonl"), enable_forensic_logging=True)
    model = _two(apa, cfg)
    mgr = apa.APAManager(model, cfg)
    mgr.pre_step()
    list(mgr.apa_modules.values())[0].gpu_amax.fill_(1.0)
    mgr.post_backward_sync_and_eval()
    assert not os.path.exists(cfg.forensic_log_file)
    cfg2 = apa.APAConfig(fp8_simulation_mode=True, device=DEV, check_interval=100, enable_forensic_logging=True,
                         forensic_log_file=str(tmp_path / "f.jsonl"))
    model2 = _two(apa, cfg2)
    mgr2 = apa.APAManager(model2, cfg2)
    for _ in range(3):
        mgr2.pre_step()
        assert mgr2._forward_execution_order == []
        model2(torch.randn(4, 16, device=DEV))
        assert len(mgr2._forward_execution_order) > 0
        mgr2.post_backward_sync_and_eval()

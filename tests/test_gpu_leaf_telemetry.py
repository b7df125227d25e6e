"""Leaf-module telemetry (manager.py:70-84) taken from the dgrad kernel.

A LayerNorm (or GELU) whose output feeds exactly one APALinear receives that
layer's dgrad output as grad_output; the dgrad kernel already folded its
amax / NaN flag into the layer's boundary-cast buffers, so the leaf hook
merges those instead of reading the tensor again. The leaf's telemetry must
equal torch's own amax / nonfinite check of the grad_output it received."""
import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


class LayerNorm32(nn.LayerNorm):
    def forward(self, x):
        return F.layer_norm(x.float(), self.normalized_shape, self.weight, self.bias, self.eps)


@pytest.mark.parametrize("plant_inf", [False, True])
@pytest.mark.parametrize("level", [0, 1, 2])
def test_leaf_hook_merges_dgrad_telemetry(plant_inf, level):
    from apa import APAConfig, APALinear, APAManager
    from apa.layers import dgrad_telemetry_source
    cfg = APAConfig(device="cuda", check_interval=1)
    torch.manual_seed(0)
    model = nn.Sequential(APALinear(64, 128, config=cfg), nn.ReLU(), LayerNorm32(128),
                          APALinear(128, 32, config=cfg)).cuda()
    for m in (model[0], model[3]):
        m.level = level
    mgr = APAManager(model, cfg)
    seen = {}

    def spy(mod, grad_in, grad_out):
        seen["g"] = grad_out[0].detach().float().clone()
        seen["src"] = dgrad_telemetry_source(grad_out[0])

    model[2].register_full_backward_hook(spy)
    if plant_inf:
        with torch.no_grad():
            model[3].weight_master[3, 5] = float("inf")
    x = torch.randn(256, 64, device="cuda")
    mgr.pre_step()
    model(x).float().pow(2).mean().backward()
    torch.cuda.synchronize()
    assert seen["src"] is model[3].boundary_cast        # the shortcut was taken
    g = seen["g"]
    ref_amax = g.abs().max().item()
    ref_flag = 0 if torch.isfinite(g).all().item() else 1
    amax = model[2].gpu_amax.item()
    assert (math.isnan(amax) and math.isnan(ref_amax)) or amax == ref_amax
    assert model[2].gpu_has_nonfinite.item() == ref_flag
    assert ref_flag == (1 if plant_inf else 0)


def test_no_shortcut_when_a_leaf_output_has_two_consumers():
    """A leaf whose output feeds two layers receives the sum of their
    gradients: a new tensor, so the hook reads it."""
    from apa import APAConfig, APALinear, APAManager
    from apa.layers import dgrad_telemetry_source
    cfg = APAConfig(device="cuda", check_interval=1)
    torch.manual_seed(0)
    ln = LayerNorm32(64).cuda()
    a, b = APALinear(64, 32, config=cfg).cuda(), APALinear(64, 32, config=cfg).cuda()
    model = nn.ModuleDict({"ln": ln, "a": a, "b": b})
    mgr = APAManager(model, cfg)
    seen = {}
    ln.register_full_backward_hook(lambda m, gi, go: seen.update(src=dgrad_telemetry_source(go[0]),
                                                                  g=go[0].detach().clone()))
    x = torch.randn(128, 64, device="cuda", requires_grad=True)
    mgr.pre_step()
    h = ln(x)
    (a(h).float().sum() + b(h).float().pow(2).sum()).backward()
    torch.cuda.synchronize()
    assert seen["src"] is None
    assert ln.gpu_amax.item() == seen["g"].abs().max().item()

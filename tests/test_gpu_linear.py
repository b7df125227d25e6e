"""APALinear forward+backward through the drop-in API against the reference's
own outputs (tests/golden/linear_small.npz, produced by running the reference
on CPU) and against the oracle."""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")
TOL = {0: 2e-2, 1: 2e-2, 2: 1e-3}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (d if d > 0 else 1.0)


def _cases():
    z = np.load(os.path.join(G, "linear_small.npz"))
    return z, int(z["count"][0])


Z, COUNT = _cases()


@pytest.mark.parametrize("i", range(COUNT))
def test_linear_matches_reference(i):
    from apa import APAConfig, APALinear, APAManager
    z = Z
    p = f"c{i}_"
    M, K, N, level, is_bf16, has_bias = (int(v) for v in z[p + "meta"])
    cfg = APAConfig(device="cuda", check_interval=1)
    lin = APALinear(K, N, bias=bool(has_bias), config=cfg)
    mgr = APAManager(nn.Sequential(lin), cfg)
    with torch.no_grad():
        lin.weight_master.copy_(torch.from_numpy(z[p + "W"]))
        if has_bias:
            lin.bias_master.copy_(torch.from_numpy(z[p + "b"]))
    lin.level = level
    mgr.pre_step()
    x = torch.from_numpy(z[p + "x"]).to(torch.bfloat16 if is_bf16 else torch.float32).cuda().requires_grad_(True)
    y = lin(x)
    assert y.dtype == (torch.float16 if level == 1 else torch.float32)
    dy = torch.from_numpy(z[p + "dy"]).to(y.dtype).cuda()
    y.backward(dy)
    torch.cuda.synchronize()
    tol = TOL[level]
    assert rel(y.detach().float().cpu().numpy(), z[p + "y"]) < (tol if level == 2 else max(tol * 0.1, 1e-5))
    assert x.grad.dtype == x.dtype
    # x.grad is delivered in x's dtype: one bf16 rounding step on top of the tolerance
    assert rel(x.grad.float().cpu().numpy(), z[p + "dx"]) < tol + (4e-3 if is_bf16 else 0.0)
    assert rel(lin.weight_master.grad.cpu().numpy(), z[p + "dW"]) < tol
    if has_bias:
        assert rel(lin.bias_master.grad.cpu().numpy(), z[p + "db"]) < tol
    amax, flag, ratio, bc_amax, bc_flag = z[p + "tele"]
    assert lin.gpu_has_nonfinite.item() == flag
    if math.isnan(amax):
        assert math.isnan(lin.gpu_amax.item())
    else:
        assert lin.gpu_amax.item() == pytest.approx(amax, rel=1e-3)
    assert lin.gpu_underflow_ratio.item() == pytest.approx(ratio, abs=5e-3)
    assert lin.boundary_cast.gpu_has_nonfinite.item() == bc_flag
    assert lin.boundary_cast.gpu_amax.item() == pytest.approx(bc_amax, rel=0.13 if level == 0 else 2e-3)


def test_working_copy_dtypes_and_state_dict():
    from apa import APAConfig, APALinear
    from apa.config import LEVEL_FP8, LEVEL_FP16, LEVEL_TF32
    cfg = APAConfig(device="cuda")
    lin = APALinear(40, 24, config=cfg)
    lin.refresh_working_copy()
    assert lin.weight_work.dtype == torch.float8_e4m3fn and lin.bias_work.dtype == torch.float8_e4m3fn
    lin.level = LEVEL_FP16
    lin.refresh_working_copy()
    assert lin.weight_work.dtype == torch.float16
    lin.level = LEVEL_TF32
    lin.refresh_working_copy()
    assert lin.weight_work is lin.weight_master
    sd = lin.state_dict()
    assert set(sd) == {"weight_master", "bias_master", "gpu_amax", "gpu_underflow_ratio", "gpu_has_nonfinite"}
    lin2 = APALinear(40, 24, config=cfg)
    lin2.load_state_dict(sd)
    assert torch.equal(lin2.weight_master, lin.weight_master)
    # a reference checkpoint taken at TF32 carries aliased working-copy keys
    ref_sd = dict(sd, weight_work=sd["weight_master"], bias_work=sd["bias_master"])
    lin2.load_state_dict(ref_sd)
    lin.level = LEVEL_FP16
    lin.refresh_working_copy()
    assert lin.weight_work.dtype == torch.float16


def test_working_copy_bytes_bit_exact():
    """The pre_step working copy equals the oracle's E4M3 / fp16 bytes."""
    from apa import APAConfig, APALinear
    from oracle import apa_oracle as O
    cfg = APAConfig(device="cuda")
    lin = APALinear(100, 36, config=cfg)
    with torch.no_grad():
        lin.weight_master.mul_(3000.0)     # push some weights past 464 (NaN in E4M3)
    W = lin.weight_master.detach().cpu().numpy()
    lin.refresh_working_copy()
    got = lin.weight_work.contiguous().view(torch.uint8).cpu().numpy()
    assert np.array_equal(got, O.f32_to_e4m3_bits(W))
    lin.level = 1
    lin.refresh_working_copy()
    got = lin.weight_work.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, O.f32_to_f16_bits(W))


def test_3d_input_and_no_grad_paths():
    from apa import APAConfig, APALinear
    cfg = APAConfig(device="cuda")
    lin = APALinear(64, 32, config=cfg)
    x = torch.randn(2, 5, 64, device="cuda")
    with torch.no_grad():
        y = lin(x)
    assert y.shape == (2, 5, 32)
    lin.weight_master.requires_grad_(False)
    lin.bias_master.requires_grad_(False)
    x.requires_grad_(True)
    lin(x).sum().backward()
    assert x.grad is not None and x.grad.shape == x.shape
    assert lin.weight_master.grad is None

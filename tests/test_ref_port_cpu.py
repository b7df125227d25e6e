"""The torch-CPU port of the reference's simulation path (oracle/ref_port.py),
which bench.py times as the reference arm and the CPU baseline when the
reference package is not installed, is pinned to the reference itself:

* every APALinear forward/backward case of tests/golden/linear_small.npz
  (produced by running the reference) is reproduced bit for bit: output,
  input gradient, master weight and bias gradients, module and boundary-cast
  telemetry;
* the cfg0 quick-start MLP run of tests/golden/cfg0_trajectory.json (200
  steps with AdamW and two input spikes) is reproduced bit for bit: initial
  weights, every step's loss, the escalation events with their trigger values,
  and the skipped steps.
"""
import json
import os

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from oracle import ref_port as P

G = os.path.join(os.path.dirname(__file__), "golden")


def test_port_linear_cases_bit_exact():
    z = np.load(os.path.join(G, "linear_small.npz"))
    for i in range(int(z["count"][0])):
        p = f"c{i}_"
        M, K, N, level, is_bf16, bias = (int(v) for v in z[p + "meta"])
        lin = P.PortLinear(K, N, bias=bool(bias))
        mgr = P.PortManager(nn.Sequential(lin))
        with torch.no_grad():
            lin.weight_master.copy_(torch.from_numpy(z[p + "W"]))
            if bias:
                lin.bias_master.copy_(torch.from_numpy(z[p + "b"]))
        lin.level = level
        mgr.pre_step()
        x = torch.from_numpy(z[p + "x"])
        x = (x.to(torch.bfloat16) if is_bf16 else x).requires_grad_(True)
        y = lin(x)
        y.backward(torch.from_numpy(z[p + "dy"]).to(y.dtype))
        mgr._sync_grads()
        got = {"y": y.detach().float().numpy(), "dx": x.grad.float().numpy(), "dW": lin.weight_master.grad.numpy()}
        if bias:
            got["db"] = lin.bias_master.grad.numpy()
        for k, v in got.items():
            assert np.array_equal(v, z[p + k], equal_nan=True), (i, k)
        tele = [lin.gpu_amax.item(), lin.gpu_has_nonfinite.item(), lin.gpu_underflow_ratio.item(),
                lin.boundary_cast.gpu_amax.item(), lin.boundary_cast.gpu_has_nonfinite.item()]
        assert np.array_equal(np.array(tele), z[p + "tele"], equal_nan=True), i


def test_port_cfg0_trajectory_bit_exact():
    with open(os.path.join(G, "cfg0_trajectory.json")) as fh:
        gold = json.load(fh)
    torch.manual_seed(0)

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = P.PortLinear(768, 768)
            self.relu = nn.ReLU()
            self.norm = nn.LayerNorm(768)
            self.fc2 = P.PortLinear(768, 10)

        def forward(self, x):
            return self.fc2(self.norm(self.relu(self.fc1(x))))

    m = MLP()
    for k, v in m.state_dict().items():
        if k in gold["w0_checksum"]:
            assert float(v.double().sum()) == gold["w0_checksum"][k], k
    # research_default: theta 0.40, check_interval 4 (alpha 0.95)
    mgr = P.PortManager(m, theta=0.40, alpha=0.95, check_interval=4)
    opt = torch.optim.AdamW(mgr.trainable(), lr=1e-3)
    g = torch.Generator().manual_seed(0)
    x0 = torch.randn(64, 768, generator=g)
    y0 = torch.randint(0, 10, (64,), generator=g)
    spikes = {int(k): torch.tensor(v) for k, v in gold["spike_idx"].items()}
    skips, losses = [], []
    for step in range(200):
        x = x0.clone()
        if step in spikes:
            x.view(-1)[spikes[step]] *= 1e3
        mgr.pre_step()
        opt.zero_grad(set_to_none=True)
        loss = F.cross_entropy(m(x), y0)
        loss.backward()
        if mgr.post_backward_sync_and_eval():
            opt.step()
        else:
            opt.zero_grad(set_to_none=True)
            skips.append(step)
        losses.append(loss.item())
    assert skips == gold["skips"]
    assert np.array_equal(np.array(losses), np.array(gold["losses"]), equal_nan=True)
    assert len(mgr.events) == len(gold["events"])
    for a, b in zip(mgr.events, gold["events"]):
        b = {k: v for k, v in b.items() if k != "timestamp"}
        assert set(a) == set(b)
        for k in b:
            if k == "trigger_value":
                assert np.array_equal(np.array(a[k]), np.array(b[k]), equal_nan=True)
            elif k == "trigger_modules":
                assert list(a[k]) == list(b[k])
            else:
                assert a[k] == b[k], (k, a, b)
    assert [m.fc1.level, m.fc2.level] == gold["levels"][-1]


@pytest.mark.parametrize("level", [0, 1, 2])
def test_port_matches_numpy_oracle(level):
    """The port and the numpy restatement agree on a seeded case per rung
    (the numpy oracle accumulates in fp64, so GEMM results agree to fp32
    rounding; casts, telemetry flags and counts agree exactly)."""
    from oracle import apa_oracle as O
    rng = np.random.default_rng(11 + level)
    M, K, N = 48, 80, 40
    W = (rng.standard_normal((N, K)) * 0.2).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    lin = P.PortLinear(K, N)
    mgr = P.PortManager(nn.Sequential(lin))
    with torch.no_grad():
        lin.weight_master.copy_(torch.from_numpy(W))
        lin.bias_master.copy_(torch.from_numpy(b))
    lin.level = level
    mgr.pre_step()
    xt = torch.from_numpy(x).requires_grad_(True)
    y = lin(xt)
    dy = (torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)) * 0.5).to(y.dtype)
    y.backward(dy)
    mgr._sync_grads()
    ref = O.linear_fwd_bwd(x, "f32", W, b, level, dy.float().numpy())
    tol = 1e-5 if level != 1 else 2e-3

    def rel(a, r):
        return np.linalg.norm(np.asarray(a, np.float64) - r) / max(np.linalg.norm(r), 1e-30)

    assert rel(y.detach().float().numpy(), ref.y) < tol
    assert rel(xt.grad.numpy(), ref.dx) < 2e-2
    assert rel(lin.weight_master.grad.numpy(), ref.dW) < 2e-2
    assert lin.gpu_has_nonfinite.item() == ref.flag

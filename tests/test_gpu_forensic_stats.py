"""Device-side forensic statistics (apa_tensor_stats) against torch: max |x|
exact, the first index of the largest magnitude exact (torch.argmax returns
the first maximal index), mean and unbiased standard deviation within fp64
summation-order tolerance, the NaN/Inf flag; and a forensic-mode layer whose
per-role dictionaries, read back once, match torch on the tensors it saw."""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def stats(L, t):
    rec = torch.zeros(5, dtype=torch.int64, device="cuda")
    L.check(L.lib().apa_tensor_stats(t.data_ptr(), L.dt_code(t.dtype), t.numel(), rec.data_ptr(), L.stream_handle()),
            "apa_tensor_stats")
    w = rec.cpu().numpy().view(np.uint64)
    key = int(w[0])
    amax = float(np.array([key >> 32], dtype=np.uint32).view(np.float32)[0])
    return amax, (~key) & 0xFFFFFFFF, float(w[1:2].view(np.float64)[0]), float(w[2:3].view(np.float64)[0]), \
        int(w[3]), int(w[4])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("n", [1, 1000, (1 << 20) + 7])
def test_stats_match_torch(L, dtype, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    x = (torch.randn(n, device="cuda", generator=g) * 3 + 0.5).to(dtype)
    if n > 10:
        x[n // 3] = 100.0 if dtype != torch.float8_e4m3fn else 448.0     # a tie in magnitude above
        x[n // 2] = -100.0 if dtype != torch.float8_e4m3fn else -448.0   # all others: the first wins
    xf = x.float()
    amax, idx, s1, s2, cnt, bad = stats(L, x)
    a = xf.abs()
    assert amax == a.max().item()
    assert idx == a.argmax().item()
    assert cnt == n and bad == 0
    mean = s1 / n
    assert mean == pytest.approx(xf.double().mean().item(), rel=1e-9, abs=1e-9)
    if n > 1:
        std = math.sqrt(max((s2 - s1 * s1 / n) / (n - 1), 0.0))
        assert std == pytest.approx(xf.double().std().item(), rel=1e-7)


@pytest.mark.parametrize("special", [float("nan"), float("inf"), float("-inf")])
def test_stats_nonfinite(L, special):
    x = torch.randn(5000, device="cuda")
    x[1234] = special
    amax, idx, s1, s2, cnt, bad = stats(L, x)
    assert bad == 1 and idx == 1234
    assert (math.isnan(amax) if math.isnan(special) else math.isinf(amax))


def test_forensic_layer_role_stats(tmp_path):
    """A layer in forensic mode: after one step the synced per-role amax,
    mean/std and argmax equal torch's on the same tensors."""
    from apa import APAConfig, APALinear
    cfg = APAConfig(device="cuda", enable_forensic_logging=True, forensic_capture_tensor_stats=True,
                    forensic_capture_argmax_index=True, log_file=str(tmp_path / "l.jsonl"))
    torch.manual_seed(0)
    lin = APALinear(96, 40, config=cfg).cuda()
    lin.level = 1
    x = torch.randn(64, 96, device="cuda", requires_grad=True)
    lin(x).float().pow(2).sum().backward()
    torch.cuda.synchronize()
    lin._forensic_sync()
    w = lin.weight_master.detach().half().float()               # the FP16 working weight
    assert lin._forensic_role_amax["weight"] == w.abs().max().item()
    assert lin._forensic_role_argmax["weight"] == w.abs().flatten().argmax().item()
    st = lin._forensic_role_stats["weight"]
    assert st["mean"] == pytest.approx(w.double().mean().item(), rel=1e-6, abs=1e-9)
    assert st["std"] == pytest.approx(w.double().std().item(), rel=1e-6)
    gw = lin.weight_master.grad
    assert lin._forensic_role_amax["grad_weight"] == gw.abs().max().item()
    assert set(lin._forensic_role_amax) >= {"input_activation", "weight", "output", "grad_output",
                                            "grad_weight", "grad_input"}

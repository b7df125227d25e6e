"""apa_bias_grad_noalloc: the bias gradient for callers that cannot allocate
device memory at call time (a framework that owns every device buffer, code
that must not trigger the device-wide synchronisation of cudaMalloc/cudaFree,
foreign bindings holding only borrowed pointers). It must give the same
result as the allocating path, apa_cast with caller-allocated column partials
followed by apa_colsum_finalize, on consecutive calls that share its fixed
scratch array.

This file is collected last on purpose, and passes both alone in a fresh
process and after the rest of the suite."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# the bias-gradient tolerance the other parity tests use, per working dtype
TOL = {3: 2e-2, 1: 2e-2, 0: 1e-3}


def _allocating_path(L, dy, work):
    rows, cols = dy.shape
    nparts = (rows + 63) // 64
    part = torch.empty(nparts, cols, device="cuda")
    out = torch.empty(cols, device="cuda")
    s = L.stream_handle()
    L.check(L.lib().apa_cast(dy.data_ptr(), L.dt_code(dy.dtype), rows, cols, dy.stride(0), None, work, cols, None, 0,
                             None, None, 1, None, part.data_ptr(), s), "apa_cast")
    L.check(L.lib().apa_colsum_finalize(part.data_ptr(), nparts, cols, work, out.data_ptr(), 0, s), "finalize")
    return out


def _noalloc_path(L, dy, work):
    rows, cols = dy.shape
    out = torch.empty(cols, device="cuda")
    L.check(L.lib().apa_bias_grad_noalloc(dy.data_ptr(), L.dt_code(dy.dtype), rows, cols, dy.stride(0), work,
                                          out.data_ptr(), 0, L.stream_handle()), "apa_bias_grad_noalloc")
    return out


def _rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    d = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (d if d > 0 else 1.0)


@pytest.mark.parametrize("work,dt", [(3, torch.float32), (1, torch.float16), (0, torch.float32)])
def test_noalloc_matches_allocating_path_on_consecutive_calls(work, dt):
    from apa import _lib as L
    g = torch.Generator(device="cuda").manual_seed(7)
    first = torch.randn(8192, 4096, device="cuda", generator=g).to(dt)
    second = (torch.randn(1000, 300, device="cuda", generator=g) * 0.01).to(dt)
    for dy in (first, second):
        want = _allocating_path(L, dy, work)
        got = _noalloc_path(L, dy, work)
        torch.cuda.synchronize()
        assert _rel(got, want) <= TOL[work]
        assert torch.equal(got, want)      # same kernels, same summation order
    assert L.device_status() == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    from apa import _lib as L
    dy = torch.zeros(1, 8, device="cuda")
    out = torch.zeros(8, device="cuda")
    # ceil(rows / 64) * cols = 65536 * 4096 > 4 Mi partial sums: rejected before any launch
    st = L.lib().apa_bias_grad_noalloc(dy.data_ptr(), L.DT_F32, 65536 * 64, 4096, 4096, 3, out.data_ptr(), 0,
                                       L.stream_handle())
    assert st == L.ERR_NOALLOC_LIMIT
    assert b"no-allocation scratch" in L.lib().apa_status_string(st)

"""Stream-K split of the last, partial wave of a weight-gradient GEMM
(apa_linear_wgrad_ws with the workspace apa_wgrad_workspace_bytes asks for).

At the bench shape (4096 x 4096 weight over 8192 tokens: 256 CTA-pair tiles
on 74 pairs, a last wave of 34 tiles) the tail tiles are each split in two
along the tokens; every split stores its fp32 partial and the warp that
finishes last adds them in split order and applies the epilogue.

* Exact operands (every fp32 partial sum exact, so no summation order can
  change the accumulator): weight gradient, underflow counts and ratio equal
  the oracle bit for bit, on every rung and on a ragged shape (edges of both
  output dimensions and of the token range inside tiles).
* N(0,1) operands: deterministic (two calls give identical bits), equal to the
  unsplit kernel except for the order of the tail tiles' fp32 sums (carried
  through the working-dtype rounding: one E4M3 / fp16 step at most), the same
  ratio to within a few counts, and the counters left at zero.
"""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

WD = {0: "e4m3", 1: "f16", 2: "f32"}
TDT = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}
VMIN = {0: 0.015625, 1: 6.1035e-5, 2: 0.0}


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def seeded(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


def exact_operand(rng, rows, cols):
    return (rng.integers(-8, 9, size=(rows, cols)) / 32.0).astype(np.float32)


def padded_t(a, dtype):
    """a [rows, cols] -> CUDA tensor of dtype with a 16-byte row pitch."""
    rows, cols = a.shape
    es = torch.empty((), dtype=dtype).element_size()
    ld = (cols + 16 // es - 1) // (16 // es) * (16 // es)
    buf = torch.zeros(rows, ld, dtype=dtype, device="cuda")
    buf[:, :cols] = torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)
    return buf


def workspace(L, rung, M, N, K):
    nb = ctypes.c_int64(0)
    L.check(L.lib().apa_wgrad_workspace_bytes(rung, M, N, K, ctypes.addressof(nb)), "apa_wgrad_workspace_bytes")
    return nb.value


def wgrad(L, rung, DYT, XT, N, K, M, ws=None, out=None):
    dw = out if out is not None else torch.empty(N, K, device="cuda")
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    rmax = torch.zeros(1, device="cuda")
    if ws is None:
        L.check(L.lib().apa_linear_wgrad(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0),
                                         dw.data_ptr(), dw.stride(0), M, N, K, 0, cnt.data_ptr(), rmax.data_ptr(),
                                         L.stream_handle()), "wgrad")
    else:
        L.check(L.lib().apa_linear_wgrad_ws(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0),
                                            dw.data_ptr(), dw.stride(0), M, N, K, 0, cnt.data_ptr(), rmax.data_ptr(),
                                            ws.data_ptr(), ws.numel(), L.stream_handle()), "wgrad_ws")
    torch.cuda.synchronize()
    return dw, cnt, rmax


# (tokens M, out N, in K): the bench shape and a ragged one (16 x 16 tiles of
# 256, the last ones partial; 8000 tokens end inside a 128-byte slab)
SHAPES = [(8192, 4096, 4096), (8000, 4000, 3850)]


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_streamk_tail_exact(L, rung, shape):
    M, N, K = shape
    nb = workspace(L, rung, M, N, K)
    assert nb > 0, "the last wave of this shape is split (stream-K)"
    rng = seeded("streamk", rung, shape)
    dy, x = exact_operand(rng, M, N), exact_operand(rng, M, K)
    dy[rng.random((M, N)) < 0.9] = 0.0
    DYT, XT = padded_t(dy.T, TDT[rung]), padded_t(x.T, TDT[rung])
    acc = (torch.from_numpy(dy).cuda().double().T @ torch.from_numpy(x).cuda().double()).float().cpu().numpy()
    seen = O.quantize(acc, "f16") if rung == 1 else acc
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    dw, cnt, rmax = wgrad(L, rung, DYT, XT, N, K, M, ws)
    assert np.array_equal(dw.cpu().numpy(), O.quantize(seen, WD[rung]), equal_nan=True)
    if rung != 2:
        nz, uf = O.underflow_counts(seen, VMIN[rung])
        assert rmax.item() == O.ratio_from_counts(nz, uf)
    assert cnt.cpu().tolist() == [0, 0, 0]
    assert L.device_status() == 0


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_streamk_tail_realistic(L, rung):
    M, N, K = 8192, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(5 + rung)
    dyt = torch.randn(N, M, device="cuda", generator=g)
    xt = torch.randn(K, M, device="cuda", generator=g)
    if rung == 2:
        DYT, XT = (torch.from_numpy(O.tf32_rn(t.cpu().numpy())).cuda() for t in (dyt, xt))
    else:
        DYT, XT = dyt.to(TDT[rung]), xt.to(TDT[rung])
    ws = torch.empty(workspace(L, rung, M, N, K), dtype=torch.uint8, device="cuda")
    ws.fill_(0xA5)   # the entry point clears what it needs itself
    a, ca, ra = wgrad(L, rung, DYT, XT, N, K, M, ws)
    b, cb, rb = wgrad(L, rung, DYT, XT, N, K, M, ws)
    ref, _, rr = wgrad(L, rung, DYT, XT, N, K, M, None)
    an, bn, rn = a.cpu().numpy(), b.cpu().numpy(), ref.cpu().numpy()
    assert np.array_equal(an, bn, equal_nan=True)          # deterministic
    assert ca.cpu().tolist() == cb.cpu().tolist() == [0, 0, 0]
    fin = np.isfinite(rn) & np.isfinite(an)
    d = np.abs(an[fin].astype(np.float64) - rn[fin])
    # only the tail tiles differ: the tensor cores' fp32 accumulation in
    # another order (measured up to ~0.007 absolute for sums of 8192 N(0,1)
    # products whose partial sums reach ~300), then the working-dtype rounding
    # of the result (at most one E4M3 / fp16 step more)
    ulp = {0: 2.0 ** -3, 1: 2.0 ** -10, 2: 0.0}[rung]
    assert (d <= (ulp + 2.0 ** -12) * np.abs(rn[fin]) + 2.0 ** -5).all()
    assert (d > 0).mean() < 0.2
    if rung == 2:
        assert (d > 0).mean() > 0.01   # the tail tiles were summed in two parts
    assert ra.item() == pytest.approx(rr.item(), abs=1e-4)
    assert L.device_status() == 0

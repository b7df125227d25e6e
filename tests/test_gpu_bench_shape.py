"""Parity at the bench shape, 8192 tokens x 4096 in x 4096 out, through the
fused entry points with the automatic launch plan (the 256x256 CTA-pair tile
running several persistent waves: 128 or 256 pair tiles on 74 clusters).

1. Exact operands (multiples of 2^-5 with |v| <= 1/4: exactly representable in
   E4M3, fp16 and TF32, and every fp32 partial sum of their products is
   exact), so the accumulator is fixed whatever the summation order: forward
   output and telemetry, input gradient and its boundary-cast telemetry, and
   weight gradient with its underflow ratio equal the oracle bit for bit on
   every rung.
2. Realistic operands (the bench's N(0,1) activations and gradients, cast to
   the working dtype): each fused epilogue is checked bit for bit against the
   oracle's rounding of the kernel's own fp32 accumulator, taken from the
   same GEMM with the raw epilogue (apa_gemm_tn EPI_RAW) forced to the same
   tile plan, so the MMA sequence and therefore the accumulator are the same.
   The weight gradient's nonzero and underflow counts, read before the ratio
   fold (apa_linear_wgrad_block with last = 0), equal the oracle's counts on
   that accumulator exactly.
"""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

M, K, N = 8192, 4096, 4096
WD = {0: "e4m3", 1: "f16", 2: "f32"}
TDT = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}
EPI_FWD, EPI_DGRAD, EPI_WGRAD, EPI_RAW = 0, 1, 2, 3
EPI_FLAG = {4: 1, 8: 2}


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def seeded(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


def exact_operand(rng, rows, cols):
    return (rng.integers(-8, 9, size=(rows, cols)) / 32.0).astype(np.float32)


def plan(L, rung, epi, m, n, k, out_dt):
    t, w = ctypes.c_int(0), ctypes.c_int(0)
    L.check(L.lib().apa_gemm_plan(rung, epi, m, n, k, L.dt_code(out_dt), 0, 0, ctypes.addressof(t),
                                  ctypes.addressof(w)), "apa_gemm_plan")
    return t.value, w.value


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dtype)


def exact_matmul_t(a, b):
    """a @ b.T on the GPU in fp64: exact for the exact operands."""
    return (a.double() @ b.double().T).float().cpu().numpy()


def raw_acc(L, rung, A, B, m, n, k, tile_ew):
    """The fp32 accumulator of A[m,k] . B[n,k]^T with the given (tile, epilogue warps)."""
    tile, ew = tile_ew
    out = torch.empty(m, n, device="cuda")
    L.check(L.lib().apa_gemm_tn(rung, EPI_RAW, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), out.data_ptr(),
                                L.DT_F32, n, m, n, k, tile | EPI_FLAG[ew], 0, L.stream_handle()), "gemm_tn raw")
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_forward_exact_bench_shape(L, rung):
    ydt = torch.float16 if rung == 1 else torch.float32
    assert plan(L, rung, EPI_FWD, M, N, K, ydt)[0] == 512
    rng = seeded("bench-fwd", rung)
    x, W = exact_operand(rng, M, K), exact_operand(rng, N, K)
    b = exact_operand(rng, 1, N)[0]
    X, Wd = dev(x, TDT[rung]), dev(W, TDT[rung])
    B = dev(b, TDT[rung])
    ref = exact_matmul_t(X, Wd) + b
    if rung == 1:
        ref = O.quantize(ref, "f16")
    y = torch.empty(M, N, dtype=ydt, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_linear_fwd(rung, X.data_ptr(), K, Wd.data_ptr(), K, B.data_ptr(), y.data_ptr(), N, M, N, K,
                                   amax.data_ptr(), flag.data_ptr(), L.stream_handle()), "fwd")
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), ref)
    assert amax.item() == float(np.abs(ref).max()) and flag.item() == 0
    assert L.device_status() == 0


@pytest.mark.parametrize("dx_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rung", [0, 1, 2])
def test_dgrad_exact_bench_shape(L, rung, dx_dtype):
    """dx[8192, 4096] = dyq[8192, 4096] . wq[4096, 4096], reduced over the 4096
    outputs, rounded to the working dtype and then to x's dtype."""
    assert plan(L, rung, EPI_DGRAD, M, K, N, dx_dtype)[0] == 512
    rng = seeded("bench-dgrad", rung)
    dy, W = exact_operand(rng, M, N), exact_operand(rng, N, K)
    DY, WT = dev(dy, TDT[rung]), dev(W.T, TDT[rung])
    acc = exact_matmul_t(DY, WT)
    wq = O.quantize(acc, WD[rung])
    ref = O.quantize(wq, "bf16" if dx_dtype == torch.bfloat16 else "f32")
    dx = torch.full((M, K), 3.0, dtype=dx_dtype, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_linear_dgrad(rung, DY.data_ptr(), N, WT.data_ptr(), N, dx.data_ptr(), L.dt_code(dx_dtype), K,
                                     M, N, K, amax.data_ptr(), flag.data_ptr(), L.stream_handle()), "dgrad")
    torch.cuda.synchronize()
    assert np.array_equal(dx.float().cpu().numpy(), ref)
    assert amax.item() == float(np.abs(wq).max()) and flag.item() == 0
    assert L.device_status() == 0


def _bench_operands(rung):
    """The bench's inputs in the working dtype: x bf16 N(0,1) (seed 0), dy
    N(0,1) (seed 1; fp16 at the FP16 rung) and a uniform weight of the
    module's initial scale, cast as the layer casts them."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).float()
    dy = torch.randn(M, N, generator=torch.Generator().manual_seed(1))
    if rung == 1:
        dy = dy.half().float()
    # the TF32 rung's operands are stored rounded to the TF32 grid, as the layer's casts store them
    rnd = (lambda a: O.tf32_rn(a)) if rung == 2 else (lambda a: O.quantize(a, WD[rung]))
    to = lambda t: torch.from_numpy(rnd(t.numpy())).cuda().to(TDT[rung])
    torch.manual_seed(0)
    bound = 1.0 / np.sqrt(K)
    W = (torch.rand(N, K) * 2 - 1) * bound
    return to(x), to(dy), to(W)


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_epilogues_bit_exact_on_bench_inputs(L, rung):
    xq, dyq, wq = _bench_operands(rung)
    # forward: y = acc + bias (fp16 output at FP16), amax of y
    ydt = torch.float16 if rung == 1 else torch.float32
    pf = plan(L, rung, EPI_FWD, M, N, K, ydt)
    acc = raw_acc(L, rung, xq, wq, M, N, K, pf)
    b = (torch.rand(N, generator=torch.Generator().manual_seed(3)) * 0.1).numpy()
    bq = O.quantize(b, WD[rung])
    ref = (acc + bq[None, :]).astype(np.float32)
    if rung == 1:
        ref = O.quantize(ref, "f16")
    y = torch.empty(M, N, dtype=ydt, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    B = dev(bq, TDT[rung])
    L.check(L.lib().apa_linear_fwd(rung, xq.data_ptr(), K, wq.data_ptr(), K, B.data_ptr(), y.data_ptr(), N, M, N, K,
                                   amax.data_ptr(), flag.data_ptr(), L.stream_handle()), "fwd")
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), ref)
    assert amax.item() == O.amax_nan(ref)
    # input gradient: dx = bf16(working(acc)), boundary-cast amax of working(acc)
    wqt = wq.t().contiguous()
    pd = plan(L, rung, EPI_DGRAD, M, K, N, torch.bfloat16)
    acc = raw_acc(L, rung, dyq, wqt, M, K, N, pd)
    work = O.quantize(acc, WD[rung])
    dx = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    amax.zero_()
    flag.zero_()
    L.check(L.lib().apa_linear_dgrad(rung, dyq.data_ptr(), N, wqt.data_ptr(), N, dx.data_ptr(), L.DT_BF16, K, M, N, K,
                                     amax.data_ptr(), flag.data_ptr(), L.stream_handle()), "dgrad")
    torch.cuda.synchronize()
    assert np.array_equal(dx.float().cpu().numpy(), O.quantize(work, "bf16"), equal_nan=True)
    assert amax.item() == O.amax_nan(work)
    # weight gradient: counts on the (FP16: fp16-rounded) accumulator, then
    # master.grad = f32(working(acc))
    dyqt, xqt = dyq.t().contiguous(), xq.t().contiguous()
    pw = plan(L, rung, EPI_WGRAD, N, K, M, torch.float32)
    assert pw[0] == 512
    acc = raw_acc(L, rung, dyqt, xqt, N, K, M, pw)
    seen = O.quantize(acc, "f16") if rung == 1 else acc
    dw = torch.empty(N, K, device="cuda")
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    rmax = torch.zeros(1, device="cuda")
    L.check(L.lib().apa_linear_wgrad_block(rung, dyqt.data_ptr(), M, xqt.data_ptr(), M, dw.data_ptr(), K, M, N, K, 0,
                                           cnt.data_ptr(), rmax.data_ptr(), 0, L.stream_handle()), "wgrad block")
    torch.cuda.synchronize()
    # |dW| reaches ~480 here: above 464 the E4M3 rounding gives NaN (the reference's cast rule)
    assert np.array_equal(dw.cpu().numpy(), O.quantize(seen, WD[rung]), equal_nan=True)
    if rung != 2:
        nz, uf = O.underflow_counts(seen, O.THRESHOLDS_MIN[rung])
        assert cnt.cpu().tolist() == [nz, uf, 0]
        assert rmax.item() == 0.0          # not folded yet (last = 0)
        # the whole-gradient entry point folds exactly that ratio
        cnt.zero_()
        L.check(L.lib().apa_linear_wgrad(rung, dyqt.data_ptr(), M, xqt.data_ptr(), M, dw.data_ptr(), K, M, N, K, 0,
                                         cnt.data_ptr(), rmax.data_ptr(), L.stream_handle()), "wgrad")
        torch.cuda.synchronize()
        assert rmax.item() == O.ratio_from_counts(nz, uf)
        assert cnt.cpu().tolist() == [0, 0, 0]
    assert L.device_status() == 0

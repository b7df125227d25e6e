"""K2-K4 tcgen05 GEMMs with their fused epilogues, through the C ABI.

Tolerances (normwise relative error ||got - ref|| / ||ref||):
  FP8 / FP16 rungs  2e-2   (the parity tolerance for GEMM outputs and gradients)
  TF32 rung         1e-3
Telemetry (amax, NaN flag) is bit-exact against the kernel's own output, and
the underflow counts are bit-exact against the oracle on inputs whose fp32
sums are exact (so no summation order can change them)."""
import math
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

TOL = {0: 2e-2, 1: 2e-2, 2: 1e-3}
WD = {0: "e4m3", 1: "f16", 2: "f32"}
TDT = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}
SHAPES = [(128, 128, 128), (17, 48, 10), (64, 96, 80), (130, 272, 65), (300, 200, 520), (1000, 256, 384),
          (257, 1024, 129)]


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (d if d > 0 else 1.0)


def padded(q: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """Exactly-representable values -> CUDA tensor of dtype with a 16-byte row pitch."""
    rows, cols = q.shape
    es = torch.empty((), dtype=dtype).element_size()
    step = 16 // es
    ld = (cols + step - 1) // step * step
    buf = torch.zeros(rows, ld, dtype=dtype, device="cuda")
    buf[:, :cols] = torch.from_numpy(np.ascontiguousarray(q)).to(dtype).cuda()
    return buf[:, :cols]


def seeded(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_forward(L, rung, shape):
    M, K, N = shape
    rng = seeded("fwd", rung, shape)
    x = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.3).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    xq, Wq, bq = O.quantize(x, WD[rung]), O.quantize(W, WD[rung]), O.quantize(b, WD[rung])
    ref = (xq.astype(np.float64) @ Wq.astype(np.float64).T + bq).astype(np.float32)
    if rung == 1:
        ref = O.quantize(ref, "f16")
    X, Wt = padded(xq, TDT[rung]), padded(Wq, TDT[rung])
    B = torch.from_numpy(bq).to(TDT[rung]).cuda()
    ydt = torch.float16 if rung == 1 else torch.float32
    y = torch.empty(M, N, dtype=ydt, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_linear_fwd(rung, X.data_ptr(), X.stride(0), Wt.data_ptr(), Wt.stride(0), B.data_ptr(),
                                   y.data_ptr(), N, M, N, K, amax.data_ptr(), flag.data_ptr(), L.stream_handle()),
            "fwd")
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    assert rel(got, ref) < (1e-5 if rung == 0 else TOL[rung]), rel(got, ref)
    assert amax.item() == float(np.abs(got).max())
    assert flag.item() == 0
    assert L.device_status() == 0


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("shape", SHAPES[:5])
def test_dgrad(L, rung, xdt, shape):
    M, K, N = shape
    rng = seeded("dgrad", rung, shape, str(xdt))
    dy = (rng.standard_normal((M, N)) * 0.5).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.3).astype(np.float32)
    dyq, Wq = O.quantize(dy, WD[rung]), O.quantize(W, WD[rung])
    acc = (dyq.astype(np.float64) @ Wq.astype(np.float64)).astype(np.float32)
    work = O.quantize(acc, WD[rung])
    xname = {torch.bfloat16: "bf16", torch.float32: "f32", torch.float16: "f16"}[xdt]
    ref = O.quantize(work, xname)
    DY, WT = padded(dyq, TDT[rung]), padded(np.ascontiguousarray(Wq.T), TDT[rung])
    dx = torch.empty(M, K, dtype=xdt, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_linear_dgrad(rung, DY.data_ptr(), DY.stride(0), WT.data_ptr(), WT.stride(0), dx.data_ptr(),
                                     L.dt_code(xdt), K, M, N, K, amax.data_ptr(), flag.data_ptr(),
                                     L.stream_handle()), "dgrad")
    torch.cuda.synchronize()
    got = dx.float().cpu().numpy()
    # dx is delivered in x's dtype: allow one rounding step of that dtype on
    # top of the rung's tolerance (a last-bit difference of the fp32 sum can
    # round to the neighbouring bf16/fp16 value)
    out_step = {torch.bfloat16: 4e-3, torch.float16: 1e-3, torch.float32: 0.0}[xdt]
    assert rel(got, ref) < TOL[rung] + out_step, rel(got, ref)
    ref_amax, _ = O.track(0.0, 0, work)
    assert amax.item() == pytest.approx(ref_amax, rel=0.13 if rung == 0 else 1e-3)
    assert flag.item() == 0


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_wgrad_exact_counts(L, rung, shape):
    """Inputs are multiples of 2^-5 with small magnitudes, so every fp32 sum is
    exact: the GEMM result, its quantisation and the underflow counts must
    equal the oracle's exactly."""
    M, K, N = shape
    rng = seeded("wgrad", rung, shape)
    x = (rng.integers(-8, 9, size=(M, K)) / 32.0).astype(np.float32)
    dy = (rng.integers(-8, 9, size=(M, N)) / 32.0).astype(np.float32)
    dy[rng.random((M, N)) < 0.9] = 0.0
    acc = (dy.astype(np.float64).T @ x.astype(np.float64)).astype(np.float32)
    if rung == 1:
        acc = O.quantize(acc, "f16")
    nz, uf = O.underflow_counts(acc, O.THRESHOLDS_MIN[rung])
    ratio = O.ratio_from_counts(nz, uf) if rung != 2 else 0.0
    ref = O.quantize(acc, WD[rung])
    DYT, XT = padded(np.ascontiguousarray(dy.T), TDT[rung]), padded(np.ascontiguousarray(x.T), TDT[rung])
    dw = torch.full((N, K), 7.0, device="cuda")
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    rmax = torch.zeros(1, device="cuda")
    L.check(L.lib().apa_linear_wgrad(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0), dw.data_ptr(),
                                     K, M, N, K, 0, cnt.data_ptr(), rmax.data_ptr(), L.stream_handle()), "wgrad")
    torch.cuda.synchronize()
    got = dw.cpu().numpy()
    assert np.array_equal(got, ref)
    assert rmax.item() == ratio
    assert cnt.cpu().tolist() == [0, 0, 0]
    # accumulate mode adds onto the existing gradient; running max keeps the larger ratio
    rmax.fill_(0.75)
    L.check(L.lib().apa_linear_wgrad(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0), dw.data_ptr(),
                                     K, M, N, K, 1, cnt.data_ptr(), rmax.data_ptr(), L.stream_handle()), "wgrad")
    torch.cuda.synchronize()
    assert np.array_equal(dw.cpu().numpy(), (ref + ref).astype(np.float32))
    assert rmax.item() == max(0.75, ratio)


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_wgrad_random_tolerance(L, rung):
    M, K, N = 777, 320, 200
    rng = seeded("wgrad-rand", rung)
    x = (rng.standard_normal((M, K))).astype(np.float32)
    dy = (rng.standard_normal((M, N)) * 0.01).astype(np.float32)
    xq, dyq = O.quantize(x, WD[rung]), O.quantize(dy, WD[rung])
    acc = (dyq.astype(np.float64).T @ xq.astype(np.float64)).astype(np.float32)
    if rung == 1:
        acc = O.quantize(acc, "f16")
    ref = O.quantize(acc, WD[rung])
    DYT, XT = padded(np.ascontiguousarray(dyq.T), TDT[rung]), padded(np.ascontiguousarray(xq.T), TDT[rung])
    dw = torch.empty(N, K, device="cuda")
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    rmax = torch.zeros(1, device="cuda")
    L.check(L.lib().apa_linear_wgrad(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0), dw.data_ptr(),
                                     K, M, N, K, 0, cnt.data_ptr(), rmax.data_ptr(), L.stream_handle()), "wgrad")
    torch.cuda.synchronize()
    assert rel(dw.cpu().numpy(), ref) < TOL[rung]
    nz, uf = O.underflow_counts(acc, O.THRESHOLDS_MIN[rung])
    ratio = O.ratio_from_counts(nz, uf) if rung != 2 else 0.0
    assert rmax.item() == pytest.approx(ratio, abs=2e-3)


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_bench_shape_against_torch_fp32(L, rung):
    """cfg1 shape, M=8192 K=4096 N=4096: forward GEMM against a torch fp32
    matmul of the same quantised operands (TF32 disabled in the checker)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    M, K, N = 8192, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).to(TDT[rung])
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(TDT[rung])
    y = torch.empty(M, N, dtype=torch.float16 if rung == 1 else torch.float32, device="cuda")
    L.check(L.lib().apa_linear_fwd(rung, x.data_ptr(), K, W.data_ptr(), K, None, y.data_ptr(), N, M, N, K, None,
                                   None, L.stream_handle()), "fwd")
    ref = x.float() @ W.float().T
    err = ((y.float() - ref).norm() / ref.norm()).item()
    assert err < (1e-5 if rung == 0 else TOL[rung]), err
    assert L.device_status() == 0

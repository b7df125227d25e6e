"""Every GEMM tile shape (128x128 and 128x256 on one CTA, 256x256 on a CTA
pair with tcgen05 cta_group::2) with 4 and with 8 epilogue warps, for every
rung and epilogue, through apa_gemm_tn, plus the fused entry points at shapes
where the automatic choice is the CTA pair.

Operands are multiples of 2^-5 with |v| <= 1/4: exactly representable in
E4M3, fp16 and TF32, and every fp32 partial sum of their products is exact.
The accumulator is therefore fixed whatever the summation order, and each
epilogue's output must equal the oracle's rounding of the exact result bit
for bit. Ragged shapes put the edges of A, B and K inside a tile, including a
CTA pair whose odd CTA holds no valid row at all (M <= 128)."""
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

WD = {0: "e4m3", 1: "f16", 2: "f32"}
TDT = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}
TILES = {"128x128": 128, "128x256": 256, "pair256x256": 512}
EPI_WARPS = {"epi4": 1, "epi8": 2}   # flag bits OR-ed into the tile code
EPI_FWD, EPI_DGRAD, EPI_WGRAD = 0, 1, 2
# (M, K, N)
SHAPES = [(100, 64, 72), (300, 200, 520), (257, 1024, 129), (640, 160, 384), (1024, 512, 1024)]


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def seeded(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


def exact_operand(rng, rows, cols):
    return (rng.integers(-8, 9, size=(rows, cols)) / 32.0).astype(np.float32)


def padded(q, dtype):
    rows, cols = q.shape
    es = torch.empty((), dtype=dtype).element_size()
    step = 16 // es
    ld = (cols + step - 1) // step * step
    buf = torch.zeros(rows, ld, dtype=dtype, device="cuda")
    buf[:, :cols] = torch.from_numpy(np.ascontiguousarray(q)).to(dtype).cuda()
    return buf[:, :cols]


def expected(acc, rung, epi, out_name):
    if epi == EPI_FWD:
        return O.quantize(acc, "f16") if rung == 1 else acc
    if epi == EPI_DGRAD:
        return O.quantize(O.quantize(acc, WD[rung]), out_name)
    a = O.quantize(acc, "f16") if rung == 1 else acc
    return O.quantize(a, WD[rung])


@pytest.mark.parametrize("warps", list(EPI_WARPS))
@pytest.mark.parametrize("tile", list(TILES))
@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("epi", [EPI_FWD, EPI_DGRAD, EPI_WGRAD])
@pytest.mark.parametrize("shape", SHAPES)
def test_tile_epilogue_exact(L, warps, tile, rung, epi, shape):
    M, K, N = shape
    rng = seeded("tiles", rung, epi, shape)
    a = exact_operand(rng, M, K)
    b = exact_operand(rng, N, K)
    acc = (a.astype(np.float64) @ b.astype(np.float64).T).astype(np.float32)
    if epi == EPI_FWD:
        out_dt, out_name = (torch.float16, "f16") if rung == 1 else (torch.float32, "f32")
    elif epi == EPI_DGRAD:
        out_dt, out_name = torch.bfloat16, "bf16"
    else:
        out_dt, out_name = torch.float32, "f32"
    ref = expected(acc, rung, epi, out_name)
    A, B = padded(a, TDT[rung]), padded(b, TDT[rung])
    out = torch.full((M, N), 3.0, dtype=out_dt, device="cuda")
    for cap in (0, 6):   # one CTA (pair) per SM, and a few CTAs looping over many tiles
        out.fill_(3.0)
        L.check(L.lib().apa_gemm_tn(rung, epi, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), out.data_ptr(),
                                    L.dt_code(out_dt), N, M, N, K, TILES[tile] | EPI_WARPS[warps], cap,
                                    L.stream_handle()), "gemm_tn")
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.array_equal(got, ref.astype(np.float32)), (cap, np.abs(got - ref).max())
    assert L.device_status() == 0


def plan(L, rung, epi, M, N, K, out_dt):
    import ctypes
    t, w = ctypes.c_int(0), ctypes.c_int(0)
    L.check(L.lib().apa_gemm_plan(rung, epi, M, N, K, L.dt_code(out_dt), 0, 0, ctypes.addressof(t),
                                  ctypes.addressof(w)), "apa_gemm_plan")
    return t.value, w.value


def exact_matmul_t(a, b):
    """a @ b.T for operands whose products and sums are exact in fp32 (float64 on the GPU)."""
    return (torch.from_numpy(a).cuda().double() @ torch.from_numpy(b).cuda().double().T).float().cpu().numpy()


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_wgrad_counts_on_pair_tiles(L, rung):
    """dw[4096, 4096] reduced over 8192 tokens: the automatic plan is the CTA
    pair with 4 epilogue warps. Counts, ratio and quantised gradient are exact
    against the oracle."""
    M, K, N = 8192, 4096, 4096
    assert plan(L, rung, EPI_WGRAD, N, K, M, torch.float32) == (512, 4)
    rng = seeded("wgrad-pair", rung)
    x = exact_operand(rng, M, K)
    dy = exact_operand(rng, M, N)
    dy[rng.random((M, N)) < 0.9] = 0.0
    acc = exact_matmul_t(np.ascontiguousarray(dy.T), np.ascontiguousarray(x.T))
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
    assert np.array_equal(dw.cpu().numpy(), ref)
    assert rmax.item() == ratio
    assert cnt.cpu().tolist() == [0, 0, 0]
    assert L.device_status() == 0


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_forward_telemetry_on_pair_tiles(L, rung):
    """y[4096, 4096] = x . W^T + b with K = 4096: the automatic plan is the
    CTA pair with 4 epilogue warps; output and amax exact against the oracle,
    one planted Inf raises the flag."""
    M, K, N = 4096, 4096, 4096
    ydt = torch.float16 if rung == 1 else torch.float32
    assert plan(L, rung, EPI_FWD, M, N, K, ydt) == (512, 4)
    rng = seeded("fwd-pair", rung)
    x = exact_operand(rng, M, K)
    W = exact_operand(rng, N, K)
    b = exact_operand(rng, 1, N)[0]
    acc = exact_matmul_t(x, W) + b
    ref = O.quantize(acc, "f16") if rung == 1 else acc
    X, Wt = padded(x, TDT[rung]), padded(W, TDT[rung])
    B = torch.from_numpy(b).to(TDT[rung]).cuda()
    y = torch.empty(M, N, dtype=ydt, device="cuda")
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_linear_fwd(rung, X.data_ptr(), X.stride(0), Wt.data_ptr(), Wt.stride(0), B.data_ptr(),
                                   y.data_ptr(), N, M, N, K, amax.data_ptr(), flag.data_ptr(), L.stream_handle()),
            "fwd")
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    assert np.array_equal(got, ref)
    assert amax.item() == float(np.abs(ref).max())
    assert flag.item() == 0
    # an infinite input element in row 1500 (odd CTA of its pair) -> NaN/Inf flag
    X[1500, 3] = float("inf")
    L.check(L.lib().apa_linear_fwd(rung, X.data_ptr(), X.stride(0), Wt.data_ptr(), Wt.stride(0), B.data_ptr(),
                                   y.data_ptr(), N, M, N, K, amax.data_ptr(), flag.data_ptr(), L.stream_handle()),
            "fwd")
    torch.cuda.synchronize()
    assert flag.item() == 1
    assert L.device_status() == 0


def test_plan_long_reductions(L):
    """Shapes whose CTAs run only one or two tiles but long reductions keep
    the deeper four-warp pipeline; a long TF32 reduction takes the CTA pair."""
    assert plan(L, 0, EPI_FWD, 8192, 1024, 4096, torch.float32) == (256, 4)
    assert plan(L, 1, EPI_DGRAD, 8192, 1024, 4096, torch.bfloat16) == (256, 4)
    assert plan(L, 2, EPI_DGRAD, 8192, 1024, 50304, torch.float32) == (512, 4)


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_small_k_plan_uses_eight_epilogue_warps(L, rung):
    """Epilogue-bound shapes (K = 1024 at FP8, a GPT-2-medium layer; K = 256 at
    FP16 / TF32) take 8 epilogue warps; the fused forward stays exact."""
    M, K, N = 2048, 1024 if rung == 0 else 256, 1024
    ydt = torch.float16 if rung == 1 else torch.float32
    assert plan(L, rung, EPI_FWD, M, N, K, ydt)[1] == 8
    rng = seeded("small-k", rung)
    x = exact_operand(rng, M, K)
    W = exact_operand(rng, N, K)
    acc = exact_matmul_t(x, W)
    ref = O.quantize(acc, "f16") if rung == 1 else acc
    X, Wt = padded(x, TDT[rung]), padded(W, TDT[rung])
    y = torch.empty(M, N, dtype=ydt, device="cuda")
    L.check(L.lib().apa_linear_fwd(rung, X.data_ptr(), X.stride(0), Wt.data_ptr(), Wt.stride(0), None, y.data_ptr(),
                                   N, M, N, K, None, None, L.stream_handle()), "fwd")
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), ref)
    assert L.device_status() == 0

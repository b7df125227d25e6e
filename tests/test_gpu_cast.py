"""K1 cast + telemetry kernel against the golden fixtures and the oracle.

Bit-exact: every E4M3/fp16 byte, amax and the NaN/Inf flag. Calls go through
the C ABI (apa_cast / apa_amax / apa_colsum_finalize)."""
import math
import os
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


@pytest.fixture(scope="module")
def casts():
    return np.load(os.path.join(G, "casts.npz"))


def run_cast(L, src, dst_dtype, transpose=False, telem_src=False, colsum=False, amax0=0.0, merge=None):
    """src: 2-D CUDA tensor. Returns (dst, dst_t, amax, flag, partial)."""
    rows, cols = src.shape
    dst = torch.empty(rows, cols, dtype=dst_dtype, device="cuda")
    dst_t = torch.empty(cols, rows, dtype=dst_dtype, device="cuda") if transpose else None
    amax = torch.full((1,), amax0, dtype=torch.float32, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    part = torch.empty((rows + 63) // 64, cols, dtype=torch.float32, device="cuda") if colsum else None
    st = L.lib().apa_cast(src.data_ptr(), L.dt_code(src.dtype), rows, cols, src.stride(0), dst.data_ptr(),
                          L.dt_code(dst_dtype), dst.stride(0), L.ptr(dst_t), dst_t.stride(0) if transpose else 0,
                          amax.data_ptr(), flag.data_ptr(), 1 if telem_src else 0, L.ptr(merge), L.ptr(part),
                          L.stream_handle())
    L.check(st, "apa_cast")
    torch.cuda.synchronize()
    return dst, dst_t, amax.item(), flag.item(), part


def bits(t):
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).cpu().numpy()
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def f16_equal(a, b):
    an = (a & 0x7FFF) > 0x7C00
    bn = (b & 0x7FFF) > 0x7C00
    return (np.array_equal(an, bn) and np.array_equal(a[~an], b[~bn])
            and np.array_equal(a[an] & 0x8000, b[bn] & 0x8000))


def test_bf16_exhaustive(L, casts):
    src = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).view(256, 256).cuda()
    e8, _, _, _, _ = run_cast(L, src, torch.float8_e4m3fn)
    assert np.array_equal(bits(e8).ravel(), casts["bf16_all_to_e4m3"])
    h, _, _, _, _ = run_cast(L, src, torch.float16)
    assert np.array_equal(bits(h).ravel(), casts["bf16_all_to_f16"])


def test_f16_exhaustive(L, casts):
    src = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.float16).view(256, 256).cuda()
    e8, _, _, _, _ = run_cast(L, src, torch.float8_e4m3fn)
    assert np.array_equal(bits(e8).ravel(), casts["f16_all_to_e4m3"])


def test_f32_edges_and_random(L, casts):
    xb = casts["f32_in_bits"]
    n = xb.size - xb.size % 512
    src = torch.from_numpy(xb[:n].view(np.float32).copy()).view(-1, 512).cuda()
    e8, _, _, _, _ = run_cast(L, src, torch.float8_e4m3fn)
    assert np.array_equal(bits(e8).ravel(), casts["f32_to_e4m3"][:n])
    h, _, _, _, _ = run_cast(L, src, torch.float16)
    assert f16_equal(bits(h).ravel(), casts["f32_to_f16"][:n])


def test_f32_dense_sweep_against_oracle(L):
    """Every fp32 sign/exponent/top-12-mantissa pattern with several low-bit
    tails (covers every E4M3 and fp16 rounding boundary)."""
    hi = np.arange(1 << 20, dtype=np.uint32) << 12
    for low in (0, 1, 0x7FF, 0x800, 0x801, 0xFFF):
        xb = hi | np.uint32(low)
        x = xb.view(np.float32)
        src = torch.from_numpy(x.copy()).view(1024, 1024).cuda()
        e8, _, _, _, _ = run_cast(L, src, torch.float8_e4m3fn)
        assert np.array_equal(bits(e8).ravel(), O.f32_to_e4m3_bits(x)), hex(low)
        h, _, _, _, _ = run_cast(L, src, torch.float16)
        assert f16_equal(bits(h).ravel(), O.f32_to_f16_bits(x)), hex(low)


@pytest.mark.parametrize("shape", [(1, 1), (7, 13), (64, 64), (65, 129), (200, 48), (130, 272), (1000, 10)])
@pytest.mark.parametrize("src_dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dst_dt", [torch.float8_e4m3fn, torch.float16, torch.float32])
def test_cast_transpose_telemetry_colsum(L, shape, src_dt, dst_dt):
    g = torch.Generator().manual_seed(zlib.crc32(repr((shape, str(src_dt), str(dst_dt))).encode()))
    x = (torch.randn(*shape, generator=g) * 40).to(src_dt)
    if x.numel() > 5:
        x.view(-1)[3] = 300.0
    xc = x.cuda()
    for telem_src in (False, True):
        dst, dst_t, amax, flag, part = run_cast(L, xc, dst_dt, transpose=True, telem_src=telem_src, colsum=True)
        xf = x.float().numpy()
        if dst_dt == torch.float8_e4m3fn:
            ref_bits = O.f32_to_e4m3_bits(xf)
            q = O.e4m3_bits_to_f32(ref_bits)
        elif dst_dt == torch.float16:
            ref_bits = O.f32_to_f16_bits(xf)
            q = O.f16_bits_to_f32(ref_bits)
        else:
            ref_bits = xf.view(np.uint32)
            q = xf
        got = dst.view(torch.uint8 if dst_dt == torch.float8_e4m3fn else
                       (torch.int16 if dst_dt == torch.float16 else torch.int32)).cpu().numpy()
        assert np.array_equal(got.view(ref_bits.dtype), ref_bits)
        gt = dst_t.cpu().float().numpy()
        assert np.array_equal(np.isnan(gt), np.isnan(q.T))
        assert np.array_equal(np.nan_to_num(gt), np.nan_to_num(q.T))
        ref_amax, ref_flag = O.track(0.0, 0, xf if telem_src else q)
        assert flag == ref_flag
        assert (math.isnan(amax) and math.isnan(ref_amax)) or amax == ref_amax
        # column partials of the cast values, 64 rows each
        p = part.cpu().numpy()
        for r in range(p.shape[0]):
            blk = q[r * 64:(r + 1) * 64]
            ref = blk.astype(np.float64).sum(axis=0)
            fin = np.isfinite(ref)
            np.testing.assert_allclose(p[r][fin], ref[fin], rtol=1e-4, atol=1e-4)


def test_nan_inf_flag_and_amax_merge(L):
    x = torch.tensor([[1.0, float("inf"), -3.0, 2.0]], device="cuda")
    _, _, amax, flag, _ = run_cast(L, x, torch.float16)
    assert flag == 1 and math.isinf(amax)
    x = torch.tensor([[1.0, 500.0, -3.0, 2.0]], device="cuda")   # > 464 -> NaN in E4M3
    _, _, amax, flag, _ = run_cast(L, x, torch.float8_e4m3fn)
    assert flag == 1 and math.isnan(amax)
    _, _, amax, flag, _ = run_cast(L, x, torch.float8_e4m3fn, telem_src=True)
    assert flag == 0 and amax == 500.0
    pend = torch.tensor([7.5], device="cuda")
    x = torch.tensor([[1.0, -2.0]], device="cuda")
    _, _, amax, flag, _ = run_cast(L, x, torch.float8_e4m3fn, merge=pend)
    assert amax == 7.5 and flag == 0
    pend = torch.tensor([float("nan")], device="cuda")
    _, _, amax, flag, _ = run_cast(L, x, torch.float8_e4m3fn, merge=pend)
    assert math.isnan(amax) and flag == 1
    # running max keeps a larger previous value
    _, _, amax, flag, _ = run_cast(L, x, torch.float8_e4m3fn, amax0=100.0)
    assert amax == 100.0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("n", [1, 17, 4096, 1000003])
def test_amax_kernel(L, dtype, n):
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 10).to(dtype)
    xc = x.cuda()
    amax = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(L.lib().apa_amax(xc.data_ptr(), L.dt_code(dtype), n, amax.data_ptr(), flag.data_ptr(),
                             L.stream_handle()), "apa_amax")
    ref, rflag = O.track(0.0, 0, x.float().numpy())
    assert amax.item() == ref and flag.item() == rflag
    if n > 20:
        xc[n // 2] = float("nan")
        L.check(L.lib().apa_amax(xc.data_ptr(), L.dt_code(dtype), n, amax.data_ptr(), flag.data_ptr(),
                                 L.stream_handle()), "apa_amax")
        assert math.isnan(amax.item()) and flag.item() == 1


@pytest.mark.parametrize("work", [torch.float8_e4m3fn, torch.float16, torch.float32])
def test_colsum_finalize(L, work):
    g = torch.Generator().manual_seed(5)
    part = torch.randn(9, 70, generator=g)
    out = torch.empty(70, device="cuda")
    pc = part.cuda()
    L.check(L.lib().apa_colsum_finalize(pc.data_ptr(), 9, 70, L.dt_code(work), out.data_ptr(), 0,
                                        L.stream_handle()), "finalize")
    s = part.double().sum(0).float().numpy()
    wd = {torch.float8_e4m3fn: "e4m3", torch.float16: "f16", torch.float32: "f32"}[work]
    ref = O.quantize(s, wd)
    got = out.cpu().numpy()
    # the fp32 sum order differs; compare after rounding within one working-dtype step
    np.testing.assert_allclose(got, ref, rtol=0.13 if wd == "e4m3" else 1e-3, atol=1e-6)


def test_underflow_ratio_kernel(L):
    import json
    with open(os.path.join(G, "underflow.json")) as fh:
        cases = json.load(fh)
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    out = torch.zeros((), device="cuda")
    for c in cases:
        gg = torch.tensor(c["g"], dtype=torch.float32, device="cuda")
        L.check(L.lib().apa_underflow_ratio(gg.data_ptr(), L.DT_F32, gg.numel(), float(c["vmin"]), cnt.data_ptr(),
                                            out.data_ptr(), 0, L.stream_handle()), "ratio")
        assert out.item() == pytest.approx(c["ratio"], rel=0, abs=0)
    assert cnt.cpu().tolist() == [0, 0, 0]


def test_tf32_operand_rounding(L):
    """dst TF32: values stored on the TF32 grid (round half to even), while
    telemetry and column sums see the unrounded fp32 values."""
    hi = np.arange(1 << 20, dtype=np.uint32) << 12
    x = (hi | np.uint32(0x1001)).view(np.float32)
    x = x[np.isfinite(x)][: 1024 * 512]
    src = torch.from_numpy(x.copy()).view(1024, 512).cuda()
    rows, cols = src.shape
    dst = torch.empty(rows, cols, device="cuda")
    dst_t = torch.empty(cols, rows, device="cuda")
    amax = torch.zeros(1, device="cuda")
    st = L.lib().apa_cast(src.data_ptr(), L.DT_F32, rows, cols, cols, dst.data_ptr(), L.DT_TF32, cols,
                          dst_t.data_ptr(), rows, amax.data_ptr(), None, 0, None, None, L.stream_handle())
    L.check(st, "apa_cast(tf32)")
    torch.cuda.synchronize()
    ref = O.tf32_rn(x).reshape(rows, cols)
    assert np.array_equal(dst.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(dst_t.cpu().numpy().view(np.uint32), ref.T.copy().view(np.uint32))
    assert amax.item() == float(np.abs(x).max())

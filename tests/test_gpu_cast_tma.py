"""The streaming (TMA) cast kernel, taken by apa_cast whenever the source and
every destination row is 16-byte aligned and the destination is E4M3, fp16 or
fp32 (TF32-rounded at the TF32 rung: stored values rounded, telemetry and
column sums on the unrounded values).

Bit-exact against the oracle: every code of the row-major and transposed
copies, amax and the NaN/Inf flag (on the source or on the cast values); the
per-64-row column partials within fp32 summation-order tolerance. Shapes put
tile edges (64 rows x 128 columns) inside the matrix, and the values include
the E4M3 overflow-to-NaN band (> 464), infinities, NaNs, signed zeros and
subnormals."""
import math
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(16, 16), (64, 128), (80, 144), (192, 400), (1040, 2064)]


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def make_source(shape, src_dt, special):
    g = torch.Generator().manual_seed(zlib.crc32(repr((shape, str(src_dt), special)).encode()))
    x = torch.randn(*shape, generator=g) * 40
    n = x.numel()
    flat = x.view(-1)
    if special and n >= 16:
        idx = torch.randperm(n, generator=g)[:12]
        vals = [470.0, -500.0, 449.0, -464.0, float("inf"), float("-inf"), float("nan"), -0.0, 1e-9, -3e-3,
                2.0 ** -9, 65504.0]
        for i, v in zip(idx.tolist(), vals):
            flat[i] = v
    return x.to(src_dt)


DST = {"e4m3": (torch.float8_e4m3fn, 3), "f16": (torch.float16, 1), "f32": (torch.float32, 0),
       "tf32": (torch.float32, 4)}


def cast_bits(xf, dst):
    if dst == "e4m3":
        b = O.f32_to_e4m3_bits(xf)
        return b, O.e4m3_bits_to_f32(b)
    if dst == "f16":
        b = O.f32_to_f16_bits(xf)
        return b, O.f16_bits_to_f32(b)
    stored = O.tf32_rn(xf) if dst == "tf32" else xf
    return np.ascontiguousarray(stored).view(np.uint32), xf


def got_bits(t):
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).cpu().numpy()
    if t.dtype == torch.float32:
        return t.view(torch.int32).cpu().numpy().view(np.uint32)
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def same_codes(got, ref, dst):
    if dst == "e4m3":
        return np.array_equal(got, ref)
    mag, inf, sign = (0x7FFF, 0x7C00, 0x8000) if dst == "f16" else (0x7FFFFFFF, 0x7F800000, 0x80000000)
    gn = (got & mag) > inf
    rn = (ref & mag) > inf
    return (np.array_equal(gn, rn) and np.array_equal(got[~gn], ref[~rn])
            and np.array_equal(got[gn] & sign, ref[rn] & sign))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("src_dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dst", list(DST))
@pytest.mark.parametrize("special", [False, True])
def test_streaming_cast_exact(L, shape, src_dt, dst, special):
    rows, cols = shape
    dst_dt, dst_code = DST[dst]
    x = make_source(shape, src_dt, special)
    xf = x.float().numpy()
    ref_bits, q = cast_bits(xf, dst)
    xc = x.cuda()
    for mode in ("both", "row", "t"):
        for telem_src in (0, 1):
            out = torch.empty(rows, cols, dtype=dst_dt, device="cuda") if mode != "t" else None
            out_t = torch.empty(cols, rows, dtype=dst_dt, device="cuda") if mode != "row" else None
            amax = torch.zeros(1, device="cuda")
            flag = torch.zeros(1, dtype=torch.int32, device="cuda")
            part = torch.full(((rows + 63) // 64, cols), 5.0, device="cuda")
            L.check(L.lib().apa_cast(xc.data_ptr(), L.dt_code(src_dt), rows, cols, cols, L.ptr(out),
                                     dst_code, cols, L.ptr(out_t), rows, amax.data_ptr(), flag.data_ptr(),
                                     telem_src, None, part.data_ptr(), L.stream_handle()), "apa_cast")
            torch.cuda.synchronize()
            if out is not None:
                assert same_codes(got_bits(out), ref_bits, dst), (mode, telem_src)
            if out_t is not None:
                assert same_codes(got_bits(out_t), np.ascontiguousarray(ref_bits.T), dst), (mode, telem_src)
            ref_amax, ref_flag = O.track(0.0, 0, xf if telem_src else q)
            assert flag.item() == ref_flag
            a = amax.item()
            assert (math.isnan(a) and math.isnan(ref_amax)) or a == ref_amax, (a, ref_amax)
            p = part.cpu().numpy()
            for r in range(p.shape[0]):
                ref = q[r * 64:(r + 1) * 64].astype(np.float64).sum(axis=0)
                fin = np.isfinite(ref)
                np.testing.assert_allclose(p[r][fin], ref[fin], rtol=1e-4, atol=1e-4)
                assert np.array_equal(np.isnan(p[r]), np.isnan(ref))
    assert L.device_status() == 0


@pytest.mark.parametrize("src_dt", [torch.float32, torch.bfloat16])
def test_streaming_cast_matches_fallback_kernel(L, src_dt):
    """The same cast through both kernels (a padded destination pitch that is
    not 16-byte aligned forces the first kernel): identical codes and
    partials up to summation order."""
    rows, cols = 528, 1040
    x = make_source((rows, cols), src_dt, True).cuda()
    out = {}
    for ld in (cols, cols + 3):
        dst = torch.empty(rows, ld, dtype=torch.float8_e4m3fn, device="cuda")
        dst_t = torch.empty(cols, rows + (ld - cols), dtype=torch.float8_e4m3fn, device="cuda")
        part = torch.empty((rows + 63) // 64, cols, device="cuda")
        amax = torch.zeros(1, device="cuda")
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        L.check(L.lib().apa_cast(x.data_ptr(), L.dt_code(src_dt), rows, cols, cols, dst.data_ptr(), L.DT_E4M3, ld,
                                 dst_t.data_ptr(), dst_t.stride(0), amax.data_ptr(), flag.data_ptr(), 0, None,
                                 part.data_ptr(), L.stream_handle()), "apa_cast")
        torch.cuda.synchronize()
        out[ld] = (got_bits(dst)[:, :cols], got_bits(dst_t)[:, :rows], part.cpu().numpy(), amax.item(), flag.item())
    a, b = out[cols], out[cols + 3]
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    fin = np.isfinite(b[2])
    np.testing.assert_allclose(a[2][fin], b[2][fin], rtol=1e-5, atol=1e-5)
    assert (math.isnan(a[3]) and math.isnan(b[3])) or a[3] == b[3]
    assert a[4] == b[4]

"""Split-K weight gradient (apa_linear_wgrad_ws): small N x K outputs over many
tokens are computed as up to 8 fp32 partial sums and reduced in split order
by a second kernel that applies the weight-gradient epilogue.

Operands are multiples of 2^-5 with |v| <= 1/4, so every partial and total
sum is exact in fp32: the gradient, its rounding to the working dtype, the
underflow counts and the ratio must equal the oracle's bit for bit, in
overwrite and accumulate mode, and equal the unsplit kernel's."""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from oracle import apa_oracle as O

pytestmark = pytest.mark.gpu

WD = {0: "e4m3", 1: "f16", 2: "f32"}
TDT = {0: torch.float8_e4m3fn, 1: torch.float16, 2: torch.float32}
# (tokens M, out N, in K): the char-level GPT's projections, ragged cases and
# one whose gradient rows are not a multiple of 4 floats (scalar reduction)
SHAPES = [(16384, 1152, 384), (16384, 384, 1536), (8192, 200, 136), (4096, 64, 64), (8192, 96, 50)]


@pytest.fixture(scope="module")
def L():
    from apa import _lib
    return _lib


def seeded(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


def padded(q, dtype):
    rows, cols = q.shape
    es = torch.empty((), dtype=dtype).element_size()
    step = 16 // es
    ld = (cols + step - 1) // step * step
    buf = torch.zeros(rows, ld, dtype=dtype, device="cuda")
    buf[:, :cols] = torch.from_numpy(np.ascontiguousarray(q)).to(dtype).cuda()
    return buf[:, :cols]


def workspace_bytes(L, rung, M, N, K):
    b = ctypes.c_int64(-1)
    L.check(L.lib().apa_wgrad_workspace_bytes(rung, M, N, K, ctypes.addressof(b)), "apa_wgrad_workspace_bytes")
    return b.value


@pytest.mark.parametrize("rung", [0, 1, 2])
@pytest.mark.parametrize("shape", SHAPES)
def test_split_wgrad_exact(L, rung, shape):
    M, N, K = shape
    nbytes = workspace_bytes(L, rung, M, N, K)
    assert nbytes > 0                                   # these shapes are split
    rng = seeded("splitk", rung, shape)
    x = (rng.integers(-8, 9, size=(M, K)) / 32.0).astype(np.float32)
    dy = (rng.integers(-8, 9, size=(M, N)) / 32.0).astype(np.float32)
    dy[rng.random((M, N)) < 0.9] = 0.0
    acc = (torch.from_numpy(dy).cuda().double().T @ torch.from_numpy(x).cuda().double()).float().cpu().numpy()
    if rung == 1:
        acc = O.quantize(acc, "f16")
    nz, uf = O.underflow_counts(acc, O.THRESHOLDS_MIN[rung])
    ratio = O.ratio_from_counts(nz, uf) if rung != 2 else 0.0
    ref = O.quantize(acc, WD[rung])
    DYT, XT = padded(np.ascontiguousarray(dy.T), TDT[rung]), padded(np.ascontiguousarray(x.T), TDT[rung])
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    rmax = torch.zeros(1, device="cuda")
    s = L.stream_handle()

    def run(dw, accumulate, ws_bytes):
        L.check(L.lib().apa_linear_wgrad_ws(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0),
                                            dw.data_ptr(), K, M, N, K, accumulate, cnt.data_ptr(), rmax.data_ptr(),
                                            ws.data_ptr(), ws_bytes, s), "apa_linear_wgrad_ws")
        torch.cuda.synchronize()

    dw = torch.full((N, K), 7.0, device="cuda")
    run(dw, 0, nbytes)
    assert np.array_equal(dw.cpu().numpy(), ref)
    assert rmax.item() == ratio
    assert cnt.cpu().tolist() == [0, 0, 0]
    rmax.fill_(0.75)
    run(dw, 1, nbytes)                                   # accumulate onto the existing gradient
    assert np.array_equal(dw.cpu().numpy(), (ref + ref).astype(np.float32))
    assert rmax.item() == max(0.75, ratio)
    # too little scratch: the unsplit kernel, same result
    dw2 = torch.full((N, K), 7.0, device="cuda")
    rmax.zero_()
    run(dw2, 0, nbytes - 16)
    assert np.array_equal(dw2.cpu().numpy(), ref)
    assert rmax.item() == ratio
    assert L.device_status() == 0


def test_large_outputs_split_only_their_last_wave(L):
    """The cfg1 weight gradient (4096 x 4096 over 8192 tokens) fills the GPU
    with tiles, so it is not split along the tokens as a whole; only its last,
    partial wave is (stream-K): 256 CTA-pair tiles on 74 pairs leave 34 tail
    tiles, each split in two, whose fp32 partials (256 x 256 each) and one
    ticket per tail tile, CTA and epilogue warp (2 x 4) are the scratch."""
    for rung in (0, 1, 2):
        assert workspace_bytes(L, rung, 8192, 4096, 4096) == 34 * 2 * 256 * 256 * 4 + 34 * 2 * 4 * 4


@pytest.mark.parametrize("rung", [0, 1, 2])
def test_row_blocks_equal_whole(L, rung):
    """apa_linear_wgrad_block over row blocks (ragged ones included) gives the
    whole call's gradient bit for bit and, folded once at the last block, the
    same underflow ratio; the counters are zero again afterwards."""
    M, N, K = 4096, 1000, 384
    rng = seeded("blocks", rung)
    x = (rng.integers(-8, 9, size=(M, K)) / 32.0).astype(np.float32)
    dy = (rng.integers(-8, 9, size=(M, N)) / 32.0).astype(np.float32)
    dy[rng.random((M, N)) < 0.7] = 0.0
    DYT, XT = padded(np.ascontiguousarray(dy.T), TDT[rung]), padded(np.ascontiguousarray(x.T), TDT[rung])
    cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
    s = L.stream_handle()
    whole = torch.empty(N, K, device="cuda")
    r_whole = torch.zeros(1, device="cuda")
    L.check(L.lib().apa_linear_wgrad(rung, DYT.data_ptr(), DYT.stride(0), XT.data_ptr(), XT.stride(0),
                                     whole.data_ptr(), K, M, N, K, 0, cnt.data_ptr(), r_whole.data_ptr(), s),
            "apa_linear_wgrad")
    blocked = torch.full((N, K), 7.0, device="cuda")
    r_blk = torch.zeros(1, device="cuda")
    es = DYT.element_size()
    blocks = [(0, 256), (256, 512), (512, 777), (777, 1000)]
    for i, (r0, r1) in enumerate(blocks):
        L.check(L.lib().apa_linear_wgrad_block(rung, DYT.data_ptr() + r0 * DYT.stride(0) * es, DYT.stride(0),
                                               XT.data_ptr(), XT.stride(0), blocked.data_ptr() + r0 * K * 4, K, M,
                                               r1 - r0, K, 0, cnt.data_ptr(), r_blk.data_ptr(),
                                               int(i == len(blocks) - 1), s), "apa_linear_wgrad_block")
        if i < len(blocks) - 1:
            torch.cuda.synchronize()
            assert r_blk.item() == 0.0                   # nothing folded before the last block
    torch.cuda.synchronize()
    assert torch.equal(blocked, whole)
    assert r_blk.item() == r_whole.item()
    if rung == 0:
        assert r_whole.item() > 0.0                      # sums below 2^-6 underflow at the FP8 rung
    assert cnt.cpu().tolist() == [0, 0, 0]
    assert L.device_status() == 0

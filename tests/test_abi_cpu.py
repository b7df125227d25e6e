"""The C-ABI library loads without a GPU and exports every entry point that
include/apa_kernels.h declares, with the signatures the ctypes binding uses."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "apa_kernels.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(apa_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for must in ("apa_cast", "apa_linear_fwd", "apa_linear_dgrad", "apa_linear_wgrad", "apa_ladder_eval"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from apa import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("libapa_kernels.so not built (run adaptive-precision-ascension_b200/build.py)")
    handle = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared():
        assert hasattr(handle, name), name
    assert set(declared()) == set(_lib.SIGNATURES), "ctypes binding and header disagree"
    lib = _lib.lib()
    assert lib.apa_abi_version() == 1
    assert lib.apa_status_string(0) == b"ok"


def test_invalid_arguments_rejected_without_gpu():
    """Argument validation happens before any CUDA call."""
    from apa import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    lib = _lib.lib()
    assert lib.apa_cast(None, 0, 4, 4, 4, None, 3, 4, None, 0, None, None, 0, None, None, None) == _lib.ERR_INVALID
    assert lib.apa_linear_fwd(0, None, 16, None, 16, None, None, 16, 16, 16, 16, None, None, None) == _lib.ERR_INVALID
    assert lib.apa_linear_fwd(0, 16, 16, 16, 16, None, 16, 16, 0, 16, 16, None, None, None) == _lib.ERR_INVALID
    assert lib.apa_linear_dgrad(0, 16, 16, 16, 16, 16, 9, 16, 16, 16, 16, None, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.apa_linear_wgrad(0, 16, 16, 16, 16, 16, 16, 16, 16, 16, 0, None, None, None) == _lib.ERR_INVALID
    assert lib.apa_ladder_eval(-1, None, None, None, None, None, 0, None, None, None, 1, 1, 0.4, 0.95, None,
                               None, None) == _lib.ERR_INVALID
    assert lib.apa_amax(None, 0, 5, None, None, None) == _lib.ERR_INVALID
    assert lib.apa_zero_list(None, 3, None) == _lib.ERR_INVALID


def _params():
    """name -> list of parameter type strings, from the header's declarations."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(?:int|unsigned|const char\s*\*|void)\s+\**\s*(apa_[a-z0-9_]+)\s*\(([^)]*)\)\s*;",
                                   src, flags=re.S):
        ps = [] if params.strip() in ("", "void") else [" ".join(p.split()) for p in params.split(",")]
        out[name] = ps
    return out


def test_ctypes_argument_types_match_header():
    """Every ctypes argtype has the width of the C parameter it binds: int ->
    c_int, int64_t -> c_int64, float -> c_float, double -> c_double, any
    pointer -> a pointer-sized type."""
    from apa import _lib
    decl = _params()
    assert set(decl) == set(_lib.SIGNATURES)
    for name, ps in decl.items():
        sig = _lib.SIGNATURES[name]
        assert len(sig) == len(ps), (name, len(sig), len(ps))
        for i, (p, t) in enumerate(zip(ps, sig)):
            if "*" in p:
                want = ctypes.sizeof(ctypes.c_void_p)
            elif p.startswith("int64_t"):
                want = 8
            elif p.startswith("double"):
                want = 8
                assert t is ctypes.c_double, (name, i, p)
            elif p.startswith("float"):
                want = 4
                assert t is ctypes.c_float, (name, i, p)
            elif p.startswith("int") or p.startswith("unsigned"):
                want = 4
            else:
                raise AssertionError(f"unparsed parameter {p!r} of {name}")
            assert ctypes.sizeof(t) == want, (name, i, p, t)


def test_new_entry_points_validate_without_gpu():
    """Block weight gradient, fused optimizer and forensic statistics reject
    bad arguments before touching the device."""
    from apa import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    lib = _lib.lib()
    # zero rows / null operands
    assert lib.apa_linear_wgrad_block(0, 16, 16, 16, 16, 16, 16, 16, 0, 16, 0, 16, None, 1, None) == _lib.ERR_INVALID
    assert lib.apa_linear_wgrad_block(0, None, 16, 16, 16, 16, 16, 16, 16, 16, 0, 16, None, 1, None) == _lib.ERR_INVALID
    # step 0, no output copy, ld < cols
    assert lib.apa_adamw_cast(16, 16, 16, 16, 4, 4, 4, 1e-3, 0.9, 0.999, 1e-8, 0.0, 0, 16, 3, 16, None, 0, None,
                              None) == _lib.ERR_INVALID
    assert lib.apa_adamw_cast(16, 16, 16, 16, 4, 4, 4, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, None, 3, 16, None, 0, None,
                              None) == _lib.ERR_INVALID
    assert lib.apa_adamw_cast(16, 16, 16, 16, 4, 8, 4, 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, 16, 3, 16, None, 0, None,
                              None) == _lib.ERR_INVALID
    assert lib.apa_tensor_stats(None, 0, 10, 16, None) == _lib.ERR_INVALID


def test_region_protocol_entry_points_without_gpu():
    """The data-parallel region entry points count regions and reject bad
    arguments before any CUDA call (32 x 64 regions; cols and the row pitch
    multiples of 4; world 2..64)."""
    from apa import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    lib = _lib.lib()
    n = ctypes.c_int64(0)
    for rows, cols, want in ((32, 64, 1), (33, 65, 4), (4096, 4096, 128 * 64), (1, 4, 1)):
        assert lib.apa_dp_regions(rows, cols, ctypes.addressof(n)) == _lib.OK
        assert n.value == want, (rows, cols)
    assert lib.apa_dp_regions(0, 64, ctypes.addressof(n)) == _lib.ERR_INVALID
    assert lib.apa_dp_regions(64, 64, None) == _lib.ERR_INVALID
    fake = 1 << 20   # never dereferenced: validation fails first
    common = (fake, fake, fake, fake, fake)   # ready local, ready mc, done mc, epoch, deferred
    # missing pointer, world 1, rank out of range, cols not a multiple of 4
    assert lib.apa_dp_region_signal(None, 64, 32, 64, *common, 2, 0, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_signal(fake, 64, 32, 64, *common, 1, 0, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_signal(fake, 64, 32, 64, *common, 2, 2, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_signal(fake, 66, 32, 66, *common, 2, 0, None) == _lib.ERR_ALIGN
    assert lib.apa_dp_region_reduce(fake, 64, 32, 64, *common, 2, 0, 2, 4, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_reduce(fake, 64, 32, 64, *common, 2, 0, 0, 0, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_wait(None, fake, 4, None) == _lib.ERR_INVALID
    assert lib.apa_dp_region_wait(fake, fake, 0, None) == _lib.ERR_INVALID
    assert lib.apa_linear_wgrad_dp(0, None, 64, None, 64, None, 64, 64, 64, 64, None, None, None, 0,
                                   fake, *common[:4], fake, 2, 0, None) == _lib.ERR_INVALID
    assert lib.apa_set_pdl(2) == _lib.ERR_INVALID

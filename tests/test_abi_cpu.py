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

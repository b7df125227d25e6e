"""ctypes binding of libapa_kernels.so (declared in include/apa_kernels.h).

The library is the only compute path of this package: there is no CPU or
torch-op fallback. Loading it needs no GPU; calling into it does. A missing
library, or any nonzero status from an entry point, raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libapa_kernels.so")

OK, ERR_INVALID, ERR_ALIGN, ERR_UNSUPPORTED, ERR_CUDA, ERR_NOALLOC_LIMIT = 0, 1, 2, 3, 4, 5
DT_F32, DT_F16, DT_BF16, DT_E4M3, DT_TF32 = 0, 1, 2, 3, 4
RUNG_FP8, RUNG_FP16, RUNG_TF32 = 0, 1, 2
EPI_FWD, EPI_DGRAD, EPI_WGRAD, EPI_RAW = 0, 1, 2, 3

_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> argtypes (all entry points return int status unless noted)
SIGNATURES = {
    "apa_abi_version": [],
    "apa_status_string": [_I],
    "apa_get_device_status": [_VP, _I],
    "apa_cast": [_VP, _I, _I64, _I64, _I64, _VP, _I, _I64, _VP, _I64, _VP, _VP, _I, _VP, _VP, _VP],
    "apa_amax": [_VP, _I, _I64, _VP, _VP, _VP],
    "apa_underflow_ratio": [_VP, _I, _I64, ctypes.c_float, _VP, _VP, _I, _VP],
    "apa_merge_telemetry": [_VP, _VP, _VP, _VP],
    "apa_colsum_finalize": [_VP, _I64, _I64, _I, _VP, _I, _VP],
    "apa_zero_list": [_VP, _I, _VP],
    "apa_linear_fwd": [_I, _VP, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP, _VP],
    "apa_linear_dgrad": [_I, _VP, _I64, _VP, _I64, _VP, _I, _I64, _I64, _I64, _I64, _VP, _VP, _VP],
    "apa_linear_wgrad": [_I, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _I64, _I, _VP, _VP, _VP],
    "apa_wgrad_workspace_bytes": [_I, _I64, _I64, _I64, _VP],
    "apa_linear_wgrad_ws": [_I, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _I64, _I, _VP, _VP, _VP, _I64, _VP],
    "apa_linear_wgrad_block": [_I, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _I64, _I, _VP, _VP, _I, _VP],
    "apa_set_gemm_sm_limit": [_I],
    "apa_set_pdl": [_I],
    "apa_dp_regions": [_I64, _I64, _VP],
    "apa_dp_region_signal": [_VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _I, _I, _VP],
    "apa_dp_region_reduce": [_VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "apa_dp_region_wait": [_VP, _VP, _I64, _VP],
    "apa_linear_wgrad_dp": [_I, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _I64, _VP, _VP, _VP, _I64, _VP,
                            _VP, _VP, _VP, _VP, _VP, _I, _I, _VP],
    "apa_gemm_tn": [_I, _I, _VP, _I64, _VP, _I64, _VP, _I, _I64, _I64, _I64, _I64, _I, _I, _VP],
    "apa_gemm_plan": [_I, _I, _I64, _I64, _I64, _I, _I, _I, _VP, _VP],
    "apa_tensor_stats": [_VP, _I, _I64, _VP, _VP],
    "apa_adamw_cast": [_VP, _VP, _VP, _VP, _I64, _I64, _I64, _F, _F, _F, _F, _F, _I64, _VP, _I, _I64, _VP, _I64,
                       _VP, _VP],
    "apa_bias_grad_noalloc": [_VP, _I, _I64, _I64, _I64, _I, _VP, _I, _VP],
    "apa_ladder_pack": [_I, _VP, _VP, _VP, _I, _VP, _VP, _VP, _VP],
    "apa_ladder_eval": [_I, _VP, _VP, _VP, _VP, _VP, _I, _VP, _VP, _VP, _I64, _I64,
                        ctypes.c_double, ctypes.c_double, _VP, _VP, _VP],
}

_lib = None
_lock = threading.Lock()


class APAKernelError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load (once) and return the kernel library."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python adaptive-precision-ascension_b200/build.py` (nvcc, sm_100a)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = ctypes.c_char_p if name == "apa_status_string" else ctypes.c_int
                _lib = handle
    return _lib


# number of kernel-library calls made (each entry point launches one kernel);
# bench.py reads it to report how many of this library's kernels it timed
calls = 0


def check(status: int, what: str) -> None:
    global calls
    calls += 1
    if status != OK:
        msg = lib().apa_status_string(status).decode()
        raise APAKernelError(f"{what} failed: status {status} ({msg})")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device=None) -> int:
    """Raw cudaStream_t of the current stream of ``device`` (the one torch
    launches on), as an int for the C ABI."""
    if _raw_stream is not None:
        if device is None:
            idx = torch.cuda.current_device()
        elif isinstance(device, int):
            idx = device
        else:
            idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


_DT = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16}
if hasattr(torch, "float8_e4m3fn"):
    _DT[torch.float8_e4m3fn] = DT_E4M3


def dt_code(dtype: torch.dtype) -> int:
    try:
        return _DT[dtype]
    except KeyError:
        raise APAKernelError(f"dtype {dtype} is not supported by the APA kernels") from None


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise APAKernelError(
            f"{what}: tensor on {t.device}; the APA kernels run only on CUDA (sm_100a) devices")


def device_status(clear: bool = True) -> int:
    out = ctypes.c_uint(0)
    check(lib().apa_get_device_status(ctypes.byref(out), 1 if clear else 0), "apa_get_device_status")
    return out.value

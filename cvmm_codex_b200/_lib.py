"""ctypes binding of libcvmm_sm100.so, the sm_100a CUDA library behind CVMM.

The library exports a plain C ABI (include/cvmm_sm100.h): device pointers,
sizes, dtype codes and a cudaStream_t. This module loads it, declares the
signatures and turns non-zero status codes into Python exceptions. There is
no fallback: if the library cannot be loaded, every CVMM operation raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CVMM_SM100_LIB", os.path.join(_HERE, "libcvmm_sm100.so"))

F32, F16, BF16, I32, I64 = 0, 1, 2, 3, 4
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED_DTYPE, ERR_LAUNCH, ERR_WORKSPACE, ERR_DEVICE = 0, -1, -2, -3, -4, -5

DTYPE_CODE = {
    torch.float32: F32,
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.int32: I32,
    torch.int64: I64,
}

# Every symbol the header declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_S = ctypes.c_size_t
SIGNATURES = {
    "cvmm_abi_version": (_I, []),
    "cvmm_last_error": (ctypes.c_char_p, []),
    "cvmm_set_sm_limit": (_I, [_I]),
    "cvmm_set_pdl": (_I, [_I]),
    "cvmm_backward_w_launches": (_I, [_L, _L, _L, _L, _I, _I, _I]),
    "cvmm_device_status": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_longlong), _P]),
    "cvmm_sel_prepare_workspace_size": (_S, [_L]),
    "cvmm_sel_prepare": (_I, [_P, _I, _L, _L, _I, _P, _P, _P, _P, _P, _S, _P]),
    "cvmm_sel_prepare_noalloc": (_I, [_P, _I, _L, _L, _I, _P, _P, _P, _P, _P]),
    "cvmm_expert_offsets": (_I, [_P, _L, _L, _P, _P]),
    "cvmm_gemm_workspace_size": (_S, [_L, _L, _L, _L, _I, _I, _I, _L]),
    "cvmm_forward": (_I, [_P, _I, _L, _L, _P, _P, _P, _L, _P, _I, _L, _L, _L, _L, _L, _L,
                          _P, _I, _L, _I, _P, _P, _P, _P, _S, _P]),
    "cvmm_weighted_combine": (_I, [_P, _I, _P, _I, _P, _I, _L, _L, _L, _P, _P]),
    "cvmm_backward_x": (_I, [_P, _I, _L, _P, _L, _P, _P, _L, _P, _I, _L, _L, _L, _L, _L, _L,
                             _P, _I, _L, _I, _P, _I, _P, _I, _L, _L, _P, _I, _P, _P, _P, _S, _P]),
    "cvmm_backward_w": (_I, [_P, _I, _L, _P, _L, _P, _I, _L, _P, _L, _P, _I, _P, _P, _L, _L,
                             _L, _L, _P, _I, _P, _P, _P, _S, _P]),
    "cvmm_sort_rows_padded": (_I, [_P, _I, _L, _P, _L, _P, _I, _P, _P, _L, _L, _L, _P, _I, _P, _P]),
    "cvmm_sort_rows_padded_ex": (_I, [_P, _I, _L, _P, _L, _P, _I, _P, _P, _L, _L, _L, _P, _I, _P, _I, _P, _P]),
    "cvmm_sum_routes": (_I, [_P, _I, _P, _I, _L, _L, _L, _P, _P]),
    "cvmm_pad_starts": (_I, [_P, _L, _P, _P]),
    "cvmm_padded_route_rows": (_I, [_P, _P, _P, _P, _L, _L, _P, _P]),
    "cvmm_selftest_wait_timeout": (_I, [_L, _P]),
    "cvmm_weighted_token_backward": (_I, [_P, _I, _P, _I, _P, _I, _P, _I, _P, _L, _L, _L, _P]),
    "cvmm_cast": (_I, [_P, _I, _P, _I, _L, _P]),
    "cvmm_cast_ahead": (_I, [_P, _I, _P, _I, _L, _P]),
    "cvmm_forward_gelu": (_I, [_P, _I, _L, _L, _P, _P, _P, _L, _P, _I, _L, _L, _L, _L, _L, _L,
                               _P, _P, _I, _L, _I, _P, _P, _S, _P]),
    "cvmm_gelu_backward": (_I, [_P, _P, _P, _I, _L, _P]),
    "cvmm_router_topk": (_I, [_P, _I, _L, _L, _L, _I, _P, _P, _P]),
}

_lib = None
_lock = threading.Lock()


class CvmmLibraryError(RuntimeError):
    """The native library is missing or was built for a different ABI."""


def load():
    """Returns the loaded library, loading it on first use."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise CvmmLibraryError(
                f"libcvmm_sm100.so not found at {LIB_PATH}; build it with "
                "`python -m cvmm_codex_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.cvmm_abi_version() != 10:
            raise CvmmLibraryError("libcvmm_sm100.so ABI version mismatch; rebuild it")
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    """Raises the Python exception matching a C status code."""
    if rc == OK:
        return
    msg = load().cvmm_last_error().decode(errors="replace")
    if rc in (ERR_INVALID_ARG, ERR_UNSUPPORTED_DTYPE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return DTYPE_CODE[t]
    except KeyError:
        raise ValueError(f"Unknown dtype {t}") from None


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(reset: bool = True, device=None) -> tuple[int, int, int]:
    """(code, where, aux) of the device status word; synchronises the stream."""
    lib = load()
    where = ctypes.c_int(0)
    aux = ctypes.c_longlong(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = lib.cvmm_device_status(int(reset), ctypes.byref(where), ctypes.byref(aux), stream_of(dev))
    if code < 0:
        check(code, "cvmm_device_status")
    return code, where.value, aux.value

"""ctypes binding of ``libraon_cuda.so`` (the C ABI declared in include/raon_cuda.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
Status codes map onto the exception classes the reference raises
(ValueError / KeyError / RuntimeError, npu/backend.py:1433-1437,3609,4866-4900).
"""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libraon_cuda.so"
HEADER = PKG.parent / "include" / "raon_cuda.h"

RC_OK, RC_ERR_INVALID, RC_ERR_NOT_FOUND, RC_ERR_CUDA, RC_ERR_TIMEOUT = 0, 1, 2, 3, 4
RC_DTYPE_BF16, RC_DTYPE_F32 = 0, 1
RC_ACT_SWIGLU, RC_ACT_SITU = 0, 1
RC_ROUTER_SOFTMAX, RC_ROUTER_SIGMOID_BIAS = 0, 1
RC_UPLOAD_SRC_DEVICE, RC_UPLOAD_GATE_UP, RC_UPLOAD_DOWN_BFP16 = 1, 2, 4
RC_EP_MAX_RANKS, RC_EP_HANDLE_BYTES = 8, 128
RC_PREFILL_GEMV, RC_PREFILL_TCGEN05 = 0, 1


class RaonCudaError(RuntimeError):
    """A CUDA-side failure (RuntimeError, as the reference's device errors)."""


class DeviceTimeout(RaonCudaError):
    """A kernel's bounded wait gave up and reported it through the error word."""


_P = ctypes.c_void_p
_I = ctypes.c_int
_U = ctypes.c_uint
_SZ = ctypes.c_size_t
_F = ctypes.c_float
_D = ctypes.c_double

# name -> (restype, argtypes); must list every function of include/raon_cuda.h.
SIGNATURES = {
    "rc_last_error": (ctypes.c_char_p, []),
    "rc_abi_version": (_I, []),
    "rc_init": (_I, [_I, ctypes.POINTER(_P)]),
    "rc_destroy": (_I, [_P]),
    "rc_stream": (_I, [_P, ctypes.POINTER(_P)]),
    "rc_sync": (_I, [_P]),
    "rc_sm_count": (_I, [_P, ctypes.POINTER(_I)]),
    "rc_upload_q4nx": (_I, [_P, _P, _SZ, _I, _I, _U, ctypes.POINTER(_P)]),
    "rc_upload_bfp16": (_I, [_P, _P, _SZ, _I, _I, _U, ctypes.POINTER(_P)]),
    "rc_quantize_q4nx": (_I, [_P, _P, _I, _I, _P, _P]),
    "rc_weight_free": (_I, [_P]),
    "rc_weight_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_SZ), ctypes.POINTER(_U)]),
    "rc_weight_set_bias": (_I, [_P, _P]),
    "rc_weight_bias": (_I, [_P, ctypes.POINTER(_P)]),
    "rc_dequant_q4nx": (_I, [_P, _P, _P, _P]),
    "rc_gemv": (_I, [_P, _P, _P, _I, _I, _I, _P, _I, _I, _I, _I, _P, _P]),
    "rc_gemv_host": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "rc_gemv_noalloc": (_I, [_P, _P, _I, _I, _I, _P, _I, _I, _I, _I, _P, _P]),
    "rc_moe_create": (_I, [_P, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "rc_moe_destroy": (_I, [_P]),
    "rc_moe_set_expert": (_I, [_P, _I, _P, _SZ, _P, _SZ, _U]),
    "rc_moe_set_router": (_I, [_P, _P, _P]),
    "rc_moe_set_fused": (_I, [_P, _I]),
    "rc_moe_set_trace": (_I, [_P, _P, _I]),
    "rc_moe_set_prefill_kernel": (_I, [_P, _I]),
    "rc_moe_ep_init": (_I, [_P, _I, _I, _I, _P]),
    "rc_moe_ep_open": (_I, [_P, _I, _P]),
    "rc_moe_ep_decode": (_I, [_P, _P, _I, _I, _I, _F, _I, _F, _F, _P, _P]),
    "rc_moe_route": (_I, [_P, _P, _I, _I, _I, _I, _F, _P, _P, _P, _P]),
    "rc_moe_experts": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _F, _I, _P, _P]),
    "rc_moe_experts_host": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _F, _I, _P]),
    "rc_moe_experts_grouped": (_I, [_P, _P, _I, _P, _P, _I, _P, _I, _F, _F, _P, _P, _P]),
    "rc_moe_decode": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _P, _P, _P, _P]),
    "rc_moe_decode_host": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _P, _P, _P, _P]),
    "rc_moe_prefill_host": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _P, _P, _P, _P]),
    "rc_moe_ep_decode_host": (_I, [_P, _P, _I, _I, _I, _F, _I, _F, _F, _P, _P]),
    "rc_moe_decode_local": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _I, _I, _I, _I, _P, _P, _P]),
    "rc_moe_combine": (_I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    "rc_moe_prefill": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _P, _P, _P, _P]),
    "rc_moe_prefill_experts": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _F, _I, _P, _P]),
    "rc_moe_prefill_local": (_I, [_P, _P, _I, _I, _I, _I, _F, _I, _F, _F, _I, _I, _I, _I, _P, _P, _P]),
    "rc_moe_prefill_local_routes": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _F, _I, _I, _I, _I, _P, _P, _P]),
    "rc_moe_prefill_combine": (_I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    "rc_sample_tokens": (_I, [_P, _P, _I, _I, _I, _I, _D, _D, _D, _P, _P, _P, _P, _P]),
    "rc_add_bf16": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _P]),
    "rc_add_rms_bf16": (_I, [_P, _P, _P, _P, _I, _I, _F, _P]),
}

_lib = None


def header_functions() -> list[str]:
    """Names of the functions ``include/raon_cuda.h`` declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(rc_\w+)\s*\(", text, re.M)))


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load the library (once) and declare every exported signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RaonCudaError(
            f"{p} is missing: build it with `python -m raon_npu_b200.build` "
            "(the CUDA path has no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    return load().rc_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Raise the reference's exception class for a non-zero status."""
    if status == RC_OK:
        return
    msg = last_error()
    if what:
        msg = f"{what}: {msg}"
    if status == RC_ERR_INVALID:
        raise ValueError(msg)
    if status == RC_ERR_NOT_FOUND:
        raise KeyError(msg)
    if status == RC_ERR_TIMEOUT:
        raise DeviceTimeout(msg)
    raise RaonCudaError(msg)

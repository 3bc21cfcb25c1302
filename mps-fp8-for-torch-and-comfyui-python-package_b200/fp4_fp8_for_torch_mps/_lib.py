"""ctypes binding of libfp8_b200.so, the sm_100a kernel library.

This replaces the reference's shader loader (fp8_mps_native.py:5-23, which
compiles shaders/fp8_matmul.metal with torch.mps.compile_shader on first use).
The library is loaded once, on first use; a missing library or a device that
is not sm_100 is an error, never a silent fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfp8_b200.so")

# dtype codes of include/fp8_b200.h
F32, BF16, F16, E4M3, E5M2, E2M1 = 0, 1, 2, 3, 4, 5
SCALE_NONE, SCALE_F32, SCALE_F16_REF = 0, 1, 2
SCALE_TENSOR, SCALE_ROWWISE = 0, 1
ETIMEOUT = -4

_CODE = {
    torch.float32: F32,
    torch.bfloat16: BF16,
    torch.float16: F16,
    torch.float8_e4m3fn: E4M3,
    torch.float8_e5m2: E5M2,
    torch.float4_e2m1fn_x2: E2M1,
}

_lock = threading.Lock()
_lib = None


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _CODE[dt]
    except KeyError:
        raise RuntimeError(f"dtype {dt} is not supported by the fp8 kernels") from None


def _declare(L):
    vp, i64, i32, u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64
    L.fp8b200_version.restype = i32
    L.fp8b200_last_error.restype = ctypes.c_char_p
    L.fp8b200_launch_count.restype = u64
    sigs = {
        "fp8b200_encode_fp8": [vp, i32, vp, i32, i64, vp, vp],
        "fp8b200_decode_fp8": [vp, i32, vp, i32, i64, vp, i32, vp],
        "fp8b200_decode_fp4": [vp, i64, vp, i32, vp, i32, vp],
        "fp8b200_quantize_fp8": [vp, i32, vp, i32, i64, vp, vp, vp],
        "fp8b200_quantize_fp8_noalloc": [vp, i32, vp, i32, i64, vp, vp],
        "fp8b200_encode_fp4": [vp, i32, vp, i64, vp, vp],
        "fp8b200_quantize_rows_fp8": [vp, i32, i64, i64, i64, vp, i64, i32, vp, vp],
        "fp8b200_silu_mul_quantize_rows_fp8": [vp, i64, i64, i64, vp, i64, i32, vp, vp],
        "fp8b200_rope_bf16": [vp, i64, i64, i32, i32, i32, i32, vp, vp, vp, vp, vp],
        "fp8b200_quantize_fp4": [vp, i32, vp, i64, vp, vp, vp],
        "fp8b200_scaled_mm": [vp, i32, i64, vp, i32, i64, i64, i64, i64,
                              vp, i32, vp, i32, vp, i32, vp, vp, i32, i64, vp],
        "fp8b200_linear_fp8w": [vp, i32, i64, vp, i32, i64, i64, i64, i64, vp, i32, vp, i32, vp, i32, i64, vp],
        "fp8b200_gemm_16bit": [vp, vp, i32, i64, i64, i64, i64, i64, vp, i32, vp, i32, vp, i32, i64, vp],
        "fp8b200_gemm_status": [ctypes.POINTER(ctypes.c_uint32), i32],
        "fp8b200_debug_gemm": [i32, ctypes.c_ulonglong],
        "fp8b200_gemm_set_path": [i32],
    }
    for name, args in sigs.items():
        if hasattr(L, name):
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = i32


def lib():
    """The loaded library (raises RuntimeError if it is missing)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"fp4_fp8_for_torch_mps: kernel library {LIB_PATH} is not built; run "
                        "`python -c 'import __graft_entry__ as g; g.build()'` or `python csrc/build.py`")
                L = ctypes.CDLL(LIB_PATH)
                _declare(L)
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().fp8b200_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def launch_count() -> int:
    return int(lib().fp8b200_launch_count())


def gemm_status(reset: bool = False) -> int:
    """Device status word of the scaled GEMM on the current device (0 = ok).
    Synchronises the device."""
    v = ctypes.c_uint32(0)
    rc = lib().fp8b200_gemm_status(ctypes.byref(v), 1 if reset else 0)
    if rc not in (0, ETIMEOUT):
        check(rc, "gemm status")
    return int(v.value)

"""ORACLE — test infrastructure only (the checker, never the product).

Python face of the CPU oracle: ctypes bindings to ``oracle/liboracle.so``
(a scalar C restatement of the conversion arithmetic, see ``fp8_oracle.c``)
plus a float64 dequantised reference for ``torch._scaled_mm``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` import this module. The product
package never does.

Dtype codes used throughout: ``SRC/OUT``: 0 = float32, 1 = bfloat16,
2 = float16; ``FMT``: 0 = float8_e4m3fn, 1 = float8_e5m2.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, BF16, F16 = 0, 1, 2
E4M3, E5M2 = 0, 1
FP4 = 2  # GEMM operand format: packed float4_e2m1fn_x2 (two values per byte, low nibble first)

_NP_OF = {F32: np.uint32, BF16: np.uint16, F16: np.uint16}


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, sz, i32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
        L.orc_encode_fp8.argtypes = [vp, i32, vp, sz, i32]
        L.orc_encode_fp8_scaled.argtypes = [vp, vp, sz, i32, f32]
        L.orc_decode_fp8.argtypes = [vp, i32, vp, i32, sz]
        L.orc_decode_fp8_scaled.argtypes = [vp, i32, vp, i32, sz, f32]
        L.orc_dequant_ref_f16.argtypes = [vp, i32, vp, sz, f32]
        L.orc_fp4_decode.argtypes = [vp, sz, vp, i32, f32]
        L.orc_fp4_dequant_ref_f16.argtypes = [vp, sz, vp, f32]
        L.orc_fp4_encode_ref.argtypes = [vp, sz, vp, f32, i32]
        L.orc_encode_range.argtypes = [ctypes.c_uint64, ctypes.c_uint64, i32, vp]
        L.orc_e4m3_from_f32_bits.argtypes = [ctypes.c_uint32]
        L.orc_e4m3_from_f32_bits.restype = ctypes.c_uint8
        L.orc_e5m2_from_f32_bits.argtypes = [ctypes.c_uint32]
        L.orc_e5m2_from_f32_bits.restype = ctypes.c_uint8
        L.orc_refshader_e4m3.argtypes = [f32]
        L.orc_refshader_e4m3.restype = ctypes.c_uint8
        L.orc_refshader_fp4.argtypes = [f32]
        L.orc_refshader_fp4.restype = ctypes.c_uint8
        L.orc_fp4_value.argtypes = [i32]
        L.orc_fp4_value.restype = f32
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _chunks(n: int, parts: int):
    step = (n + parts - 1) // max(parts, 1)
    return [(i, min(n, i + step)) for i in range(0, n, step)] if n else []


def _parallel(fn, n: int, threads: int):
    if threads <= 1 or n < (1 << 16):
        fn((0, n))
        return
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(fn, _chunks(n, threads * 4)))


# --------------------------------------------------------------------------
# array API (numpy bit patterns in, numpy bit patterns out)

def encode_fp8(src_bits: np.ndarray, src_dtype: int, fmt: int, threads: int = 1) -> np.ndarray:
    """Encode raw f32/bf16/f16 bit patterns to fp8 bytes (CPU torch semantics)."""
    src = np.ascontiguousarray(src_bits.reshape(-1))
    out = np.empty(src.size, np.uint8)
    L = lib()
    isz = src.itemsize

    def run(lo_hi):
        lo, hi = lo_hi
        L.orc_encode_fp8(_ptr(src) + lo * isz, src_dtype, _ptr(out) + lo, hi - lo, fmt)

    _parallel(run, src.size, threads)
    return out.reshape(src_bits.shape)


def encode_fp8_scaled(src: np.ndarray, scale: float, fmt: int = E4M3) -> np.ndarray:
    s = np.ascontiguousarray(src.reshape(-1), dtype=np.float32)
    out = np.empty(s.size, np.uint8)
    lib().orc_encode_fp8_scaled(_ptr(s), _ptr(out), s.size, fmt, float(np.float32(scale)))
    return out.reshape(src.shape)


def decode_fp8(codes: np.ndarray, fmt: int, out_dtype: int, threads: int = 1,
               scale: float | None = None) -> np.ndarray:
    """Decode fp8 bytes to f32/bf16/f16 bit patterns (optionally x f32 scale)."""
    src = np.ascontiguousarray(codes.reshape(-1), dtype=np.uint8)
    out = np.empty(src.size, _NP_OF[out_dtype])
    L = lib()
    osz = out.itemsize

    def run(lo_hi):
        lo, hi = lo_hi
        if scale is None:
            L.orc_decode_fp8(_ptr(src) + lo, fmt, _ptr(out) + lo * osz, out_dtype, hi - lo)
        else:
            L.orc_decode_fp8_scaled(_ptr(src) + lo, fmt, _ptr(out) + lo * osz, out_dtype,
                                    hi - lo, float(np.float32(scale)))

    _parallel(run, src.size, threads)
    return out.reshape(codes.shape)


def dequant_ref_f16(codes: np.ndarray, fmt: int, scale: float) -> np.ndarray:
    """fp8_mps::dequantize semantics (scale rounded to f16, f16 product)."""
    src = np.ascontiguousarray(codes.reshape(-1), dtype=np.uint8)
    out = np.empty(src.size, np.uint16)
    lib().orc_dequant_ref_f16(_ptr(src), fmt, _ptr(out), src.size, float(np.float32(scale)))
    return out.reshape(codes.shape)


def fp4_decode(packed: np.ndarray, out_dtype: int, scale: float = 1.0,
               threads: int = 1) -> np.ndarray:
    """Unpack (..., B) bytes to (..., 2B) values x f32 scale, low nibble first."""
    src = np.ascontiguousarray(packed, dtype=np.uint8)
    shape = src.shape[:-1] + (src.shape[-1] * 2,) if src.ndim else (2,)
    flat = src.reshape(-1)
    out = np.empty(flat.size * 2, _NP_OF[out_dtype])
    L = lib()
    osz = out.itemsize
    sc = float(np.float32(scale))

    def run(lo_hi):
        lo, hi = lo_hi
        L.orc_fp4_decode(_ptr(flat) + lo, hi - lo, _ptr(out) + 2 * lo * osz, out_dtype, sc)

    _parallel(run, flat.size, threads)
    return out.reshape(shape)


def fp4_dequant_ref_f16(packed: np.ndarray, scale: float) -> np.ndarray:
    """fp8_mps::fp4_dequantize semantics: 1-D f16 [2*numel], f16 scale."""
    flat = np.ascontiguousarray(packed.reshape(-1), dtype=np.uint8)
    out = np.empty(flat.size * 2, np.uint16)
    lib().orc_fp4_dequant_ref_f16(_ptr(flat), flat.size, _ptr(out), float(np.float32(scale)))
    return out


def fp4_encode_ref(values: np.ndarray, scale: float | None = None) -> np.ndarray:
    """Reference-threshold FP4 encode of float32 values into packed bytes."""
    v = np.ascontiguousarray(values.reshape(-1), dtype=np.float32)
    out = np.empty(v.size // 2, np.uint8)
    lib().orc_fp4_encode_ref(_ptr(v), v.size, _ptr(out), float(np.float32(scale or 1.0)),
                             0 if scale is None else 1)
    return out


def encode_range(lo: int, hi: int, fmt: int, threads: int = 1) -> np.ndarray:
    """Encode every f32 bit pattern in [lo, hi)."""
    out = np.empty(hi - lo, np.uint8)
    L = lib()

    def run(a_b):
        a, b = a_b
        L.orc_encode_range(lo + a, lo + b, fmt, _ptr(out) + a)

    _parallel(run, hi - lo, threads)
    return out


def refshader_e4m3(values) -> np.ndarray:
    """The reference shader's saturating e4m3 encoder (divergence documentation)."""
    L = lib()
    return np.array([L.orc_refshader_e4m3(float(v)) for v in values], np.uint8)


def fp4_values() -> np.ndarray:
    return np.array([lib().orc_fp4_value(i) for i in range(16)], np.float32)


# --------------------------------------------------------------------------
# torch._scaled_mm reference: dequantise and multiply in float64.

def fp8_table_f64(fmt: int) -> np.ndarray:
    bits = decode_fp8(np.arange(256, dtype=np.uint8), fmt, F32)
    return bits.view(np.float32).astype(np.float64)


def fp4_unpack_f64(packed: np.ndarray) -> np.ndarray:
    """Values of packed FP4 rows (R, K/2) bytes as float64 (R, K): byte i
    gives elements 2i (low nibble) and 2i+1 (high nibble), the nibble order of
    shaders/fp8_matmul.metal:251-261; the 16 values are the format's table
    (shaders/fp8_matmul.metal:77-80, tests/test_fp4.py:14-20)."""
    t = fp4_values().astype(np.float64)
    p = np.asarray(packed, np.uint8)
    out = np.empty(p.shape[:-1] + (2 * p.shape[-1],), np.float64)
    out[..., 0::2] = t[p & 0xF]
    out[..., 1::2] = t[p >> 4]
    return out


def _operand_f64(codes: np.ndarray, fmt: int) -> np.ndarray:
    return fp4_unpack_f64(codes) if fmt == FP4 else fp8_table_f64(fmt)[codes]


def scaled_mm_ref(a_codes: np.ndarray, b_codes_nk: np.ndarray, scale_a, scale_b,
                  fmt_a: int = E4M3, fmt_b: int = E4M3, bias=None,
                  rows=None) -> tuple[np.ndarray, np.ndarray]:
    """Reference for C = (A*sa) @ (B*sb)^T (+ bias) in float64.

    a_codes (M,K) and b_codes_nk (N,K) are fp8 bytes (fmt E4M3 / E5M2), or
    packed FP4 bytes (M,K/2) / (N,K/2) with fmt FP4; scale_a is a scalar or
    M values, scale_b a scalar or N values. ``rows`` optionally restricts the
    result to a subset of output rows. Returns (C, S) where
    S = |A*sa| @ |B*sb|^T bounds the accumulation error.
    """
    a = a_codes if rows is None else a_codes[rows]
    A = _operand_f64(a, fmt_a)
    B = _operand_f64(b_codes_nk, fmt_b)
    sa = np.asarray(scale_a, np.float64).reshape(-1)
    if sa.size > 1:
        sa = sa.reshape(-1, 1)
        if rows is not None:
            sa = sa[rows]
    else:
        sa = sa.reshape(())
    sb = np.asarray(scale_b, np.float64).reshape(-1)
    sb = sb.reshape(1, -1) if sb.size > 1 else sb.reshape(())
    P = A @ B.T
    C = P * sa * sb
    S = (np.abs(A) @ np.abs(B).T) * np.abs(sa) * np.abs(sb)
    if bias is not None:
        C = C + np.asarray(bias, np.float64).reshape(1, -1)
    return C, S


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bfloat16 values at |x| (2^(floor(log2|x|) - 7))."""
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)

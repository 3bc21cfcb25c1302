"""Host launchers for the B200 FP8/FP4 kernels.

Same function names, argument meaning and return conventions as the
reference's launcher module (fp8_mps_native.py:26-221), so code and tests
written against the reference keep working; the Metal dispatch
(`lib.<kernel>(..., threads=, group_size=)`) becomes a call into the C ABI of
libfp8_b200.so (include/fp8_b200.h) on the tensor's device and current CUDA
stream. Outputs are allocated here with torch.empty (the C ABI never
allocates). There is no CPU fallback: inputs on the CPU are moved to the
current CUDA device, as the reference moves them to "mps".

Additions beyond the reference (used by the aten overrides in ops.py):
`encode_fp8` / `decode_fp8` for both fp8 formats and any float dtype,
`quantize_fp8`, `fp4_decode` (shape-preserving, any float dtype, f32
scale), `scaled_mm` with torch._scaled_mm's full argument set, and
`fp4_scaled_mm` (packed FP4 operands multiplied on the tensor cores).
"""
from __future__ import annotations

import torch

from . import _lib as L

_FP8 = (torch.float8_e4m3fn, torch.float8_e5m2)
_FLOAT = (torch.float32, torch.bfloat16, torch.float16)
_scratch: dict[int, torch.Tensor] = {}


# ----------------------------------------------------------------- helpers
def _on_cuda(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cuda":
        t = t.to("cuda")
    return t


def _as_float_src(t: torch.Tensor) -> torch.Tensor:
    """Contiguous f32/bf16/f16 CUDA tensor (other dtypes are cast to f32 first,
    as the reference does with `.to(dtype=torch.float32)`)."""
    t = _on_cuda(t)
    if t.dtype not in _FLOAT:
        t = t.to(torch.float32)
    return t.contiguous()


def _scale_f32(scale, device) -> torch.Tensor:
    if not isinstance(scale, torch.Tensor):
        scale = torch.tensor([float(scale)], dtype=torch.float32)
    return scale.to(device=device, dtype=torch.float32).reshape(-1)[:1].contiguous()


def _amax_scratch(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _scratch.get(idx)
    if t is None:
        t = torch.empty(1, dtype=torch.int32, device=device)
        _scratch[idx] = t
    return t


def _check_out(out, dtype, numel, device, what):
    if (out.dtype != dtype or out.numel() != numel or not out.is_contiguous()
            or out.device != device):
        raise RuntimeError(f"{what}: `out` must be a contiguous {dtype} tensor of {numel} elements "
                           f"on {device}")


# ----------------------------------------------------------------- fp8 encode / decode
def encode_fp8(x: torch.Tensor, fp8_dtype: torch.dtype = torch.float8_e4m3fn,
               out: torch.Tensor | None = None, scale: torch.Tensor | None = None) -> torch.Tensor:
    """x (f32/bf16/f16, any shape) -> uint8 codes of `fp8_dtype`, bit-exact with
    CPU `x.to(fp8_dtype)`. `out` (contiguous 1-byte tensor, same numel) is
    written in place when given."""
    if fp8_dtype not in _FP8:
        raise RuntimeError(f"encode_fp8: {fp8_dtype} is not an fp8 dtype")
    src = _as_float_src(x)
    if out is None:
        out = torch.empty(src.shape, dtype=torch.uint8, device=src.device)
    if out.numel() != src.numel() or not out.is_contiguous() or out.element_size() != 1:
        raise RuntimeError("encode_fp8: `out` must be a contiguous 1-byte tensor with x's numel")
    if out.device != src.device:
        raise RuntimeError("encode_fp8: `out` is on another device")
    sc = None if scale is None else _scale_f32(scale, src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_encode_fp8(src.data_ptr(), L.dtype_code(src.dtype), out.data_ptr(),
                                           L.dtype_code(fp8_dtype), src.numel(), L.ptr(sc),
                                           L.stream_of(src)), "fp8 encode")
    return out


def decode_fp8(codes: torch.Tensor, fp8_dtype: torch.dtype, out_dtype: torch.dtype,
               scale=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp8 codes (uint8 or fp8 tensor) -> out_dtype, same shape, bit-exact with
    CPU `codes.view(fp8_dtype).to(out_dtype)` (times `scale` in f32 when
    given: one f32 product, one rounding to out_dtype). `out` (contiguous,
    out_dtype, same numel) is written in place when given."""
    if fp8_dtype not in _FP8 or out_dtype not in _FLOAT:
        raise RuntimeError(f"decode_fp8: unsupported {fp8_dtype} -> {out_dtype}")
    src = _on_cuda(codes)
    if src.element_size() != 1:
        raise RuntimeError("decode_fp8: input must hold 1-byte codes")
    src = src.contiguous()
    if out is None:
        out = torch.empty(src.shape, dtype=out_dtype, device=src.device)
    else:
        _check_out(out, out_dtype, src.numel(), src.device, "decode_fp8")
    sc = None if scale is None else _scale_f32(scale, src.device)
    mode = L.SCALE_NONE if sc is None else L.SCALE_F32
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_decode_fp8(src.data_ptr(), L.dtype_code(fp8_dtype), out.data_ptr(),
                                           L.dtype_code(out_dtype), src.numel(), L.ptr(sc), mode,
                                           L.stream_of(src)), "fp8 decode")
    return out


def fp8_encode(input):
    """float -> float8_e4m3fn codes as uint8, same shape (fp8_mps_native.py:85-98)."""
    return encode_fp8(input, torch.float8_e4m3fn)


def fp8_dequantize(input, scale):
    """e4m3 codes -> f16, same shape, times scale with the reference's f16
    arithmetic (fp8_mps_native.py:65-82)."""
    src = _on_cuda(input)
    if src.element_size() != 1:
        raise RuntimeError("fp8_dequantize: input must hold 1-byte codes")
    src = src.contiguous()
    out = torch.empty(src.shape, dtype=torch.float16, device=src.device)
    sc = _scale_f32(scale, src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_decode_fp8(src.data_ptr(), L.E4M3, out.data_ptr(), L.F16,
                                           src.numel(), sc.data_ptr(), L.SCALE_F16_REF,
                                           L.stream_of(src)), "fp8 dequantize")
    return out


def quantize_fp8(input, fp8_dtype: torch.dtype = torch.float8_e4m3fn):
    """Per-tensor dynamic quantisation on the device, no host sync:
    returns (codes uint8 same shape, f32[2] = [scale, 1/scale])."""
    if fp8_dtype not in _FP8:
        raise RuntimeError(f"quantize_fp8: {fp8_dtype} is not an fp8 dtype")
    src = _as_float_src(input)
    out = torch.empty(src.shape, dtype=torch.uint8, device=src.device)
    scales = torch.empty(2, dtype=torch.float32, device=src.device)
    scratch = _amax_scratch(src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_quantize_fp8(src.data_ptr(), L.dtype_code(src.dtype), out.data_ptr(),
                                             L.dtype_code(fp8_dtype), src.numel(), scales.data_ptr(),
                                             scratch.data_ptr(), L.stream_of(src)), "fp8 quantize")
    return out, scales


def quantize_rows_fp8(x: torch.Tensor, fp8_dtype: torch.dtype = torch.float8_e4m3fn):
    """Per-row (per-token) dynamic quantisation over the last dimension, one
    fused launch, no host sync: each row r is encoded as x * (fmax / amax_r),
    the reference's per-tensor quantize (fp8_mps_native.py:101-120) applied
    row by row. Returns (codes as a `fp8_dtype` tensor of x's shape,
    inv_scale float32 of shape (..., 1) = amax_r / fmax), ready to be
    torch._scaled_mm's rowwise scale_a."""
    if fp8_dtype not in _FP8:
        raise RuntimeError(f"quantize_rows_fp8: {fp8_dtype} is not an fp8 dtype")
    src = _as_float_src(x)
    shape = tuple(src.shape)
    cols = shape[-1] if shape else 1
    rows = src.numel() // max(cols, 1) if cols else 0
    out = torch.empty(shape, dtype=torch.uint8, device=src.device)
    inv = torch.empty(shape[:-1] + (1,) if shape else (1,), dtype=torch.float32, device=src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_quantize_rows_fp8(src.data_ptr(), L.dtype_code(src.dtype), rows, cols, cols,
                                                  out.data_ptr(), cols, L.dtype_code(fp8_dtype), inv.data_ptr(),
                                                  L.stream_of(src)), "quantize_rows")
    return out.view(fp8_dtype), inv


def silu_mul_quantize_rows_fp8(gate_up: torch.Tensor, fp8_dtype: torch.dtype = torch.float8_e4m3fn):
    """Fused F.silu(g) * u followed by quantize_rows_fp8, for a bfloat16
    (rows, 2F) gate/up projection whose columns are [g | u]: one launch reads
    the projection once and writes the (rows, F) fp8 codes and the (rows, 1)
    inverse scales; the bf16 activation is never stored. Bit-identical to
    quantize_rows_fp8(F.silu(g) * u)."""
    if fp8_dtype not in _FP8:
        raise RuntimeError(f"silu_mul_quantize_rows_fp8: {fp8_dtype} is not an fp8 dtype")
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or gate_up.shape[1] % 2:
        raise RuntimeError("silu_mul_quantize_rows_fp8: expected a bfloat16 (rows, 2F) tensor")
    rows, f = gate_up.shape[0], gate_up.shape[1] // 2
    if gate_up.stride(1) != 1 or (rows > 1 and gate_up.stride(0) < 2 * f):
        gate_up = gate_up.contiguous()
    ld = gate_up.stride(0) if rows > 1 else 2 * f
    out = torch.empty((rows, f), dtype=torch.uint8, device=gate_up.device)
    inv = torch.empty((rows, 1), dtype=torch.float32, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        L.check(L.lib().fp8b200_silu_mul_quantize_rows_fp8(gate_up.data_ptr(), rows, f, ld,
                                                           out.data_ptr(), f, L.dtype_code(fp8_dtype), inv.data_ptr(),
                                                           L.stream_of(gate_up)), "silu_mul_quantize_rows")
    return out.view(fp8_dtype), inv


def rope_bf16(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_q_heads: int, n_k_heads: int,
              head_dim: int, seq: int):
    """Rotary embedding of the q and k heads of a bf16 (tokens, ld) qkv
    projection in one launch, bit-identical to PyTorch's bf16
    cat([x1*cos - x2*sin, x2*cos + x1*sin], -1). cos / sin: (seq, head_dim/2)
    bf16 (any shape with that many contiguous elements). Returns q
    (tokens, n_q_heads, head_dim) and k (tokens, n_k_heads, head_dim)."""
    if qkv.dtype != torch.bfloat16 or qkv.dim() != 2 or qkv.stride(1) != 1:
        raise RuntimeError("rope_bf16: expected a bfloat16 (tokens, ld) tensor with unit column stride")
    cos, sin = cos.contiguous(), sin.contiguous()
    t = qkv.shape[0]
    q = torch.empty(t, n_q_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty(t, n_k_heads, head_dim, dtype=torch.bfloat16, device=qkv.device)
    ld = qkv.stride(0) if t > 1 else qkv.shape[1]
    with torch.cuda.device(qkv.device):
        L.check(L.lib().fp8b200_rope_bf16(qkv.data_ptr(), t, ld, n_q_heads, n_k_heads, head_dim, seq,
                                          cos.data_ptr(), sin.data_ptr(), q.data_ptr(), k.data_ptr(),
                                          L.stream_of(qkv)), "rope")
    return q, k


def fp8_quantize(input):
    """amax-scaled e4m3 encode; returns (codes, inv_scale f32[1])
    (fp8_mps_native.py:101-120), with the scale computed on the device."""
    out, scales = quantize_fp8(input, torch.float8_e4m3fn)
    return out, scales[1:2]


# ----------------------------------------------------------------- fp4
def fp4_decode(packed: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
               scale=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed e2m1 pairs (uint8 or float4_e2m1fn_x2, shape (..., B)) ->
    out_dtype of shape (..., 2B), low nibble first, times `scale` in f32.
    `out` (contiguous, out_dtype, 2x the input's numel) is written in place
    when given."""
    if out_dtype not in _FLOAT:
        raise RuntimeError(f"fp4_decode: unsupported output dtype {out_dtype}")
    src = _on_cuda(packed)
    if src.element_size() != 1:
        raise RuntimeError("fp4_decode: input must hold packed bytes")
    src = src.contiguous()
    shape = tuple(src.shape[:-1]) + (src.shape[-1] * 2,) if src.dim() else (2,)
    if out is None:
        out = torch.empty(shape, dtype=out_dtype, device=src.device)
    else:
        _check_out(out, out_dtype, 2 * src.numel(), src.device, "fp4_decode")
    sc = None if scale is None else _scale_f32(scale, src.device)
    mode = L.SCALE_NONE if sc is None else L.SCALE_F32
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_decode_fp4(src.data_ptr(), src.numel(), out.data_ptr(),
                                           L.dtype_code(out_dtype), L.ptr(sc), mode,
                                           L.stream_of(src)), "fp4 decode")
    return out


def fp4_dequantize(input, scale):
    """Packed bytes -> 1-D f16 of 2*numel values times scale, with the
    reference's f16 arithmetic (fp8_mps_native.py:162-179)."""
    src = _on_cuda(input)
    if src.element_size() != 1:
        raise RuntimeError("fp4_dequantize: input must hold packed bytes")
    src = src.contiguous()
    out = torch.empty(src.numel() * 2, dtype=torch.float16, device=src.device)
    sc = _scale_f32(scale, src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_decode_fp4(src.data_ptr(), src.numel(), out.data_ptr(), L.F16,
                                           sc.data_ptr(), L.SCALE_F16_REF, L.stream_of(src)),
                "fp4 dequantize")
    return out


def fp4_encode(input):
    """float -> packed e2m1 pairs, 1-D uint8 [numel/2], the reference's
    nearest-of-8 thresholds (fp8_mps_native.py:182-197)."""
    src = _as_float_src(input)
    if src.numel() % 2:
        raise RuntimeError("FP4 x2 requires even number of elements")
    out = torch.empty(src.numel() // 2, dtype=torch.uint8, device=src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_encode_fp4(src.data_ptr(), L.dtype_code(src.dtype), out.data_ptr(),
                                           src.numel(), None, L.stream_of(src)), "fp4 encode")
    return out


def fp4_quantize(input):
    """amax-scaled (6/amax) FP4 encode; returns (packed, inv_scale f32[1])
    (fp8_mps_native.py:200-221)."""
    src = _as_float_src(input)
    if src.numel() % 2:
        raise RuntimeError("FP4 x2 requires even number of elements")
    out = torch.empty(src.numel() // 2, dtype=torch.uint8, device=src.device)
    scales = torch.empty(2, dtype=torch.float32, device=src.device)
    with torch.cuda.device(src.device):
        L.check(L.lib().fp8b200_quantize_fp4(src.data_ptr(), L.dtype_code(src.dtype), out.data_ptr(),
                                             src.numel(), scales.data_ptr(),
                                             _amax_scratch(src.device).data_ptr(),
                                             L.stream_of(src)), "fp4 quantize")
    return out, scales[1:2]


# ----------------------------------------------------------------- scaled GEMM
# Above LINEAR_DECODE_ONCE_MIN_M - 1 rows of x, fp8_linear decodes the weights
# once and runs the 16-bit GEMM instead of dequantising them on load inside the
# GEMM whenever the dequant-on-load kernel's 256 x 256 output tiles outnumber
# the device's CTA pairs (one pair per two SMs): that kernel is bound by each
# SM's TMA intake, so a second wave of its tiles costs more than one pass over
# the weights in a wider type. Measured on one B200 (us, dequant-on-load /
# decode once): 384 x 14336 x 4096 93.9 / 77.6 (112 tiles), 1024 x 6144 x 4096
# 93.9 / 60.2 (96 tiles); 1024 x 4096 x 4096 50.2 / 55.3 (64 tiles),
# 768 x 6144 x 4096 51.3 / 59.4 (72 tiles).
LINEAR_DECODE_ONCE_MIN_M = 257
_SM_COUNT: dict[int, int] = {}


def linear_decodes_once(M: int, N: int, device: torch.device) -> bool:
    """Whether fp8_linear takes the decode-once path for M rows of x and N
    output channels on `device` (see LINEAR_DECODE_ONCE_MIN_M)."""
    if M < LINEAR_DECODE_ONCE_MIN_M:
        return False
    idx = torch.device(device).index
    idx = torch.cuda.current_device() if idx is None else idx
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    tiles = -(-M // 256) * -(-N // 256)
    return tiles > _SM_COUNT[idx] // 2


def gemm_16bit(a: torch.Tensor, b_nk: torch.Tensor, scale_b: torch.Tensor, bias: torch.Tensor | None = None,
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """D = a @ b_nk^T * scale_b [+ bias] for bf16 or f16 a (M, K) and b_nk
    (N, K) of the same type on the tensor cores (CTA-pair tcgen05 kind::f16).
    scale_b: 1 value or N values."""
    if a.dtype not in (torch.bfloat16, torch.float16) or b_nk.dtype != a.dtype:
        raise RuntimeError("gemm_16bit: operands must both be bfloat16 or both float16")
    if a.dim() != 2 or b_nk.dim() != 2 or a.shape[1] != b_nk.shape[1]:
        raise RuntimeError("gemm_16bit: shapes must be (M, K) and (N, K)")
    M, K = a.shape
    N = b_nk.shape[0]
    dev = a.device
    odt = out_dtype or a.dtype

    def aligned(t):
        return t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0

    if not aligned(a) or not aligned(b_nk):
        kp = (K + 7) // 8 * 8
        if not aligned(a):
            a = torch.nn.functional.pad(a, (0, kp - K)) if kp != K else a.contiguous()
        if not aligned(b_nk):
            b_nk = torch.nn.functional.pad(b_nk, (0, kp - K)) if kp != K else b_nk.contiguous()
    sb = scale_b.to(device=dev, dtype=torch.float32).contiguous()
    if sb.numel() not in (1, N):
        raise RuntimeError(f"gemm_16bit: scale_b has {sb.numel()} values, expected 1 or {N}")
    if bias is not None:
        bias = bias.to(dev).contiguous()
    npad = (N + 7) // 8 * 8                 # 16-byte aligned output rows
    out = torch.empty((M, npad), dtype=odt, device=dev)
    with torch.cuda.device(dev):
        L.check(L.lib().fp8b200_gemm_16bit(
            a.data_ptr(), b_nk.data_ptr(), L.dtype_code(a.dtype), a.stride(0), b_nk.stride(0), M, N, K,
            sb.data_ptr(), L.SCALE_TENSOR if sb.numel() == 1 else L.SCALE_ROWWISE,
            None if bias is None else bias.data_ptr(), 0 if bias is None else L.dtype_code(bias.dtype),
            out.data_ptr(), L.dtype_code(odt), npad, L.stream_of(a)), "gemm_16bit")
    return out[:, :N]


def fp8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
               bias: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """y = x @ (weight * weight_scale)^T [+ bias] with float8 weights that are
    dequantised on load inside the GEMM (never written out in a wider type):
    the reference's dequantise-then-matmul path (fp8_mps_native.py:129-159)
    for float8 weights and bf16/f16 activations. x: (..., K) bf16 or f16;
    weight: (N, K) float8_e4m3fn / float8_e5m2 (rows contiguous along K);
    weight_scale: 1 value or N values (one per output channel); bias: N values.
    Returns (..., N) in out_dtype (default x.dtype)."""
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"fp8_linear: activations must be bfloat16 or float16, got {x.dtype}")
    if weight.dtype not in _FP8 or weight.dim() != 2:
        raise RuntimeError("fp8_linear: weight must be a 2-D float8_e4m3fn / float8_e5m2 tensor")
    N, K = weight.shape
    if x.shape[-1] != K:
        raise RuntimeError(f"fp8_linear: x has {x.shape[-1]} features, weight expects {K}")
    dev = x.device
    if weight.device != dev:
        raise RuntimeError("fp8_linear: x and weight on different devices")
    odt = out_dtype or x.dtype
    if odt not in (torch.float32, torch.bfloat16, torch.float16):
        raise RuntimeError(f"fp8_linear: unsupported output dtype {odt}")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
        if K % 8:  # row starts must stay 16-byte aligned: pad the row pitch
            xp = torch.zeros(x2.shape[0], (K + 7) // 8 * 8, dtype=x.dtype, device=dev)
            xp[:, :K] = x2
            x2 = xp
    w = weight
    if w.stride(1) != 1 or w.stride(0) % 16 or w.data_ptr() % 16:
        wp = torch.zeros(N, (K + 15) // 16 * 16, dtype=torch.uint8, device=dev)
        wp[:, :K] = weight.view(torch.uint8)
        w = wp.view(weight.dtype)
    ws = weight_scale.to(device=dev, dtype=torch.float32).contiguous()
    if ws.numel() not in (1, N):
        raise RuntimeError(f"fp8_linear: weight_scale has {ws.numel()} values, expected 1 or {N}")
    if bias is not None:
        bias = bias.to(dev).contiguous()
        if bias.numel() != N or bias.dtype not in _FLOAT:
            raise RuntimeError("fp8_linear: bias must hold N float values")
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=odt, device=dev)
    if (N * out.element_size()) % 16 == 0 and linear_decodes_once(M, N, dev):
        # more output tiles than CTA pairs: decode the weights once (exact; N*K values against
        # M*N*K products) and run the 16-bit CTA-pair GEMM with the scale in its epilogue
        wd = decode_fp8(w.view(torch.uint8), weight.dtype, x.dtype)
        with torch.cuda.device(dev):
            L.check(L.lib().fp8b200_gemm_16bit(
                x2.data_ptr(), wd.data_ptr(), L.dtype_code(x.dtype), x2.stride(0), wd.stride(0), M, N, K,
                ws.data_ptr(), L.SCALE_TENSOR if ws.numel() == 1 else L.SCALE_ROWWISE,
                None if bias is None else bias.data_ptr(), 0 if bias is None else L.dtype_code(bias.dtype),
                out.data_ptr(), L.dtype_code(odt), N, L.stream_of(x2)), "fp8_linear")
        return out.reshape(*x.shape[:-1], N)
    with torch.cuda.device(dev):
        L.check(L.lib().fp8b200_linear_fp8w(
            x2.data_ptr(), L.dtype_code(x.dtype), x2.stride(0), w.data_ptr(), L.dtype_code(weight.dtype), w.stride(0),
            M, N, K, ws.data_ptr(), L.SCALE_TENSOR if ws.numel() == 1 else L.SCALE_ROWWISE,
            None if bias is None else bias.data_ptr(), 0 if bias is None else L.dtype_code(bias.dtype),
            out.data_ptr(), L.dtype_code(odt), N, L.stream_of(x2)), "fp8_linear")
    return out.reshape(*x.shape[:-1], N)


def scaled_mm(a: torch.Tensor, b_nk: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
              bias: torch.Tensor | None = None, scale_result: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16,
              a_dtype: torch.dtype = torch.float8_e4m3fn,
              b_dtype: torch.dtype = torch.float8_e4m3fn,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """D = (A * scale_a) @ (B * scale_b)^T [+ bias] [* scale_result].

    a: (M, K) fp8 codes, rows contiguous; b_nk: (N, K) fp8 codes, rows
    contiguous (the bytes of torch._scaled_mm's column-major mat2). An
    operand whose dtype argument is torch.float4_e2m1fn_x2 holds packed FP4
    instead: (M, K/2) or (N, K/2) bytes, two values per byte.
    scale_a: 1 value or M values; scale_b: 1 value or N values (float32).
    """
    if a.dim() != 2 or b_nk.dim() != 2:
        raise RuntimeError("scaled_mm: inputs must be 2-D")
    M, K = a.shape
    N, Kb = b_nk.shape
    K *= 2 if a_dtype == torch.float4_e2m1fn_x2 else 1
    Kb *= 2 if b_dtype == torch.float4_e2m1fn_x2 else 1
    if Kb != K:
        raise RuntimeError(f"scaled_mm: K mismatch ({K} vs {Kb})")
    dev = a.device
    if b_nk.device != dev:
        raise RuntimeError("scaled_mm: operands on different devices")
    if a.stride(1) != 1 or b_nk.stride(1) != 1:
        raise RuntimeError("scaled_mm: operand rows must be contiguous along K")
    sa = scale_a.to(device=dev, dtype=torch.float32).contiguous()
    sb = scale_b.to(device=dev, dtype=torch.float32).contiguous()
    la = L.SCALE_TENSOR if sa.numel() == 1 else L.SCALE_ROWWISE
    lb = L.SCALE_TENSOR if sb.numel() == 1 else L.SCALE_ROWWISE
    if la == L.SCALE_ROWWISE and sa.numel() != M:
        raise RuntimeError(f"scaled_mm: scale_a has {sa.numel()} values, expected 1 or {M}")
    if lb == L.SCALE_ROWWISE and sb.numel() != N:
        raise RuntimeError(f"scaled_mm: scale_b has {sb.numel()} values, expected 1 or {N}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
    elif out.dtype != out_dtype or tuple(out.shape) != (M, N) or out.stride(1) != 1 or out.device != dev:
        raise RuntimeError("scaled_mm: `out` must be an (M, N) out_dtype tensor with contiguous rows")
    if bias is not None:
        bias = bias.to(dev).contiguous()
        if bias.numel() != N or bias.dtype not in _FLOAT:
            raise RuntimeError("scaled_mm: bias must hold N float values")
    sr = None if scale_result is None else _scale_f32(scale_result, dev)
    with torch.cuda.device(dev):
        L.check(L.lib().fp8b200_scaled_mm(
            a.data_ptr(), L.dtype_code(a_dtype), a.stride(0),
            b_nk.data_ptr(), L.dtype_code(b_dtype), b_nk.stride(0),
            M, N, K,
            sa.data_ptr(), la, sb.data_ptr(), lb,
            L.ptr(bias), L.dtype_code(bias.dtype) if bias is not None else 0,
            L.ptr(sr), out.data_ptr(), L.dtype_code(out_dtype), out.stride(0),
            L.stream_of(a)), "scaled_mm")
    return out


def fp8_scaled_mm(A, B, scale_a, scale_b):
    """A (M,K) e4m3 bytes, B (N,K) e4m3 bytes -> f32 (M,N)
    (fp8_mps_native.py:26-62; scales: one value or one per row/column)."""
    if A.dtype != torch.uint8 or B.dtype != torch.uint8:
        raise RuntimeError("fp8_scaled_mm expects uint8 operands")
    if not (A.is_contiguous() and B.is_contiguous()):
        raise RuntimeError("fp8_scaled_mm expects contiguous operands")
    A = _on_cuda(A)
    B = B.to(A.device)
    return scaled_mm(A, B, scale_a, scale_b, out_dtype=torch.float32)


def _gemm_operand(t: torch.Tensor, what: str):
    """(uint8 view, dtype) of a float4 / float8 GEMM operand: uint8 and
    float4_e2m1fn_x2 tensors are packed FP4 bytes, float8 tensors their codes."""
    if t.dim() != 2:
        raise RuntimeError(f"fp4_scaled_mm: {what} must be 2-D")
    if t.dtype in (torch.uint8, torch.float4_e2m1fn_x2):
        return t.view(torch.uint8), torch.float4_e2m1fn_x2
    if t.dtype in _FP8:
        return t.view(torch.uint8), t.dtype
    raise RuntimeError(f"fp4_scaled_mm: {what} must be packed float4 (uint8 / float4_e2m1fn_x2) or float8, "
                       f"got {t.dtype}")


def fp4_scaled_mm(A, B, scale_a, scale_b, out_dtype: torch.dtype = torch.float32):
    """GEMM on packed FP4 operands: (A * scale_a) @ (B * scale_b)^T.

    A: (M, K/2) packed FP4 bytes (the format fp4_encode / fp4_quantize write,
    element 2i in the low nibble); B: (N, K/2) packed FP4 bytes or (N, K)
    float8 codes. Scales: one value or one per row of A / column of the
    output. Float32 accumulation on the tensor cores (tcgen05 kind::f8f6f4),
    so the FP4 codes are multiplied as they are, never decoded to 16-bit.
    An addition to the reference, whose FP4 path (fp8_mps_native.py:162-221)
    ends at decoding."""
    a, adt = _gemm_operand(_on_cuda(A), "A")
    b, bdt = _gemm_operand(B, "B")
    b = b.to(a.device)
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise RuntimeError("fp4_scaled_mm: operand rows must be contiguous")
    return scaled_mm(a, b, torch.as_tensor(scale_a), torch.as_tensor(scale_b), out_dtype=out_dtype,
                     a_dtype=adt, b_dtype=bdt)


def fp8_scaled_mm_auto(A, B, scale_a, scale_b):
    """Shape-based kernel choice happens inside the library (fp8_mps_native.py:123-126)."""
    return fp8_scaled_mm(A.contiguous(), B.contiguous(), scale_a, scale_b)


def fp8_scaled_mm_fast(A, B, scale_a, scale_b):
    """The reference's decode + fp16 matmul path (fp8_mps_native.py:129-159);
    here the same tensor-core GEMM as every other size."""
    return fp8_scaled_mm(A.contiguous(), B.contiguous(), scale_a, scale_b)

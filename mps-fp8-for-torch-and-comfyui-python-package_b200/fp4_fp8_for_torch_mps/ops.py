"""torch.library registrations: aten overrides on the CUDA dispatch key and
the fp8_mps::* custom ops.

Mirrors the reference's plugin surface (ops.py:7-246), which registers on the
"MPS" key: the same three aten overrides (`_scaled_mm`, `_to_copy`,
`copy_`, the latter two with_keyset=True, allow_override=True) and the same
seven custom ops with identical schemas and fake (meta) implementations.
Here they register on "CUDA" and launch the sm_100a kernels of
libfp8_b200.so through fp8_mps_native.

Routing follows CPU PyTorch semantics (the arithmetic the reference's own
tests hold the device path to, tests/test_mps_vs_cpu.py:124-149): e5m2 is a
distinct format (the reference routes it through e4m3, ops.py:9-12), and
`_scaled_mm(out_dtype=None)` returns self.dtype as torch does.

Pass-through: every `_to_copy` / `copy_` case the kernels do not cover
(other dtypes, devices that are not sm_100) goes to PyTorch's own kernels by
redispatching with the CUDA key removed, exactly as the reference does with
the MPS key (ops.py:122-126, :165-166). `_scaled_mm` replaces PyTorch's CUDA
kernel outright; modes the B200 kernel does not implement raise instead of
falling back to cuBLASLt. Set FP8_B200_DISABLE_OVERRIDES=1 before import to
skip the aten overrides.
"""
from __future__ import annotations

import os
import warnings

from typing import Optional

import torch
import torch.library

_DK = torch._C.DispatchKey

_FP8_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2)
_FP4_DTYPES = (torch.float4_e2m1fn_x2,)
_SUB_BYTE_DTYPES = _FP8_DTYPES + _FP4_DTYPES
_FLOAT_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _is_fp8(dtype):
    return dtype in _FP8_DTYPES


def _is_fp4(dtype):
    return dtype in _FP4_DTYPES


def _is_sub_byte(dtype):
    return dtype in _SUB_BYTE_DTYPES


def _is_float(dtype):
    return dtype in _FLOAT_DTYPES


_sm100_cache: dict[int, bool] = {}


def _device_ok(dev: torch.device) -> bool:
    """True if `dev` is a CUDA device the sm_100a kernels can run on."""
    if dev.type != "cuda":
        return False
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ok = _sm100_cache.get(idx)
    if ok is None:
        ok = torch.cuda.get_device_capability(idx) == (10, 0)
        _sm100_cache[idx] = ok
    return ok


def _target_device(device, self_device: torch.device) -> torch.device:
    if device is None:
        return self_device
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


# ------------------------------------------------------------------ routing decisions
# Pure functions of (dtypes, device facts) so the table is testable without a GPU.
TO_COPY_ENCODE_FP8 = "encode_fp8"
TO_COPY_ENCODE_FP4 = "encode_fp4"
TO_COPY_DECODE_FP8 = "decode_fp8"
TO_COPY_DECODE_FP4 = "decode_fp4"
TO_COPY_FP8_TO_FP8 = "fp8_to_fp8"
TO_COPY_REINTERPRET = "reinterpret"
TO_COPY_PASS = "pass"


def route_to_copy(src_dtype, dst_dtype, src_on_kernel_device: bool, dst_on_cuda: bool) -> str:
    """Which path `_to_copy` takes for a CUDA source (reference ops.py:52-126)."""
    if not src_on_kernel_device or not dst_on_cuda:
        return TO_COPY_PASS
    if _is_float(src_dtype) and _is_fp8(dst_dtype):
        return TO_COPY_ENCODE_FP8            # ops.py:86-96
    if _is_float(src_dtype) and _is_fp4(dst_dtype):
        return TO_COPY_ENCODE_FP4            # ops.py:74-84
    if _is_fp8(src_dtype) and _is_float(dst_dtype):
        return TO_COPY_DECODE_FP8            # ops.py:113-120
    if _is_fp4(src_dtype) and _is_float(dst_dtype):
        return TO_COPY_DECODE_FP4            # ops.py:104-111
    if _is_fp8(src_dtype) and _is_fp8(dst_dtype) and src_dtype != dst_dtype:
        return TO_COPY_FP8_TO_FP8            # CPU torch converts values
    if _is_sub_byte(src_dtype) and _is_sub_byte(dst_dtype) and src_dtype != dst_dtype:
        return TO_COPY_REINTERPRET           # fp4 <-> fp8: raw bytes, ops.py:98-102
    return TO_COPY_PASS


COPY_RAW = "raw_bytes"
COPY_ENCODE_FP8 = "encode_fp8"
COPY_ENCODE_FP4 = "encode_fp4"
COPY_DECODE_FP8 = "decode_fp8"
COPY_FP8_TO_FP8 = "fp8_to_fp8"
COPY_PASS = "pass"


def route_copy(dst_dtype, src_dtype, dst_on_kernel_device: bool, src_on_cuda_or_cpu: bool) -> str:
    """Which path `copy_` takes when the destination is a CUDA tensor
    (reference ops.py:132-166)."""
    if not dst_on_kernel_device or not src_on_cuda_or_cpu:
        return COPY_PASS
    if _is_sub_byte(dst_dtype) and _is_sub_byte(src_dtype):
        if _is_fp8(dst_dtype) and _is_fp8(src_dtype) and dst_dtype != src_dtype:
            return COPY_FP8_TO_FP8
        return COPY_RAW                      # ops.py:137-143
    if _is_fp4(dst_dtype) and _is_float(src_dtype):
        return COPY_ENCODE_FP4               # ops.py:145-153
    if _is_fp8(dst_dtype) and _is_float(src_dtype):
        return COPY_ENCODE_FP8               # ops.py:155-163
    if _is_float(dst_dtype) and _is_fp8(src_dtype):
        return COPY_DECODE_FP8
    return COPY_PASS


# ------------------------------------------------------------------ helpers
def _native():
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


def _fp4_packed_shape(shape) -> tuple:
    if len(shape) >= 1 and shape[-1] % 2 == 0:
        return tuple(shape[:-1]) + (shape[-1] // 2,)
    n = 1
    for s in shape:
        n *= s
    if n % 2:
        raise RuntimeError("FP4 x2 requires even number of elements")
    return (n // 2,)


def _flat_dense(src: torch.Tensor, dtype: torch.dtype, memory_format):
    """(flat source, output, flat output) for an elementwise conversion.

    Contiguous inputs and dense non-contiguous ones (channels_last,
    transposes) under preserve_format convert in storage order into an output
    with the same strides, as torch's preserve_format does. Anything else is
    made contiguous first and the caller applies `memory_format` afterwards."""
    from torch._prims_common import is_non_overlapping_and_dense_or_false as dense
    mf = torch.preserve_format if memory_format is None else memory_format
    if mf == torch.preserve_format and not src.is_contiguous() and dense(src):
        out = torch.empty_strided(src.shape, src.stride(), dtype=dtype, device=src.device)
        n = src.numel()
        return (src.as_strided((n,), (1,), src.storage_offset()), out,
                out.as_strided((n,), (1,), out.storage_offset()))
    src = src.contiguous()
    out = torch.empty(src.shape, dtype=dtype, device=src.device)
    return src.reshape(-1), out, out.reshape(-1)


def _apply_memory_format(t: torch.Tensor, memory_format) -> torch.Tensor:
    if memory_format in (None, torch.preserve_format, torch.contiguous_format):
        return t
    return t.contiguous(memory_format=memory_format)


# ------------------------------------------------------------------ aten overrides
def check_scaled_mm_args(self, mat2, scale_a, scale_b, out_dtype=None):
    """Argument checks of the `_scaled_mm` override: the rank, stride and
    divisibility checks of PyTorch's meta function for the op
    (torch/_meta_registrations.py, `meta_scaled_mm`) with its messages, plus the
    scale-shape rules of its CUDA kernel. Returns (M, N, K, output dtype). Pure shape/dtype/stride logic: runs on any
    device, so the boundary's error behaviour is testable without a GPU. Modes the
    B200 kernels do not implement raise instead of falling back: float4_e2m1fn_x2
    operands, block-scaled (MX / NVFP4) scales and e5m2 x e5m2."""
    if self.dim() != 2 or mat2.dim() != 2:
        raise RuntimeError(f"Inputs must be 2D but got self.dim()={self.dim()} and mat2.dim()={mat2.dim()}")
    if not (_is_fp8(self.dtype) and _is_fp8(mat2.dtype)):
        raise RuntimeError(
            f"_scaled_mm on B200: operands must be float8_e4m3fn/float8_e5m2, got {self.dtype} and {mat2.dtype}")
    if self.dtype == torch.float8_e5m2 and mat2.dtype == torch.float8_e5m2:
        raise RuntimeError("Multiplication of two Float8_e5m2 matrices is not supported")
    M, K = self.shape
    K2, N = mat2.shape
    if K != K2:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({M}x{K} and {K2}x{N})")
    if M and K and not (self.stride(1) == 1 and self.stride(0) >= K):
        raise RuntimeError(f"self must be row_major, got stride {self.stride()}")
    if N and K and not (mat2.stride(0) == 1 and mat2.stride(1) >= K):
        raise RuntimeError(f"mat2 must be col_major, got stride {mat2.stride()}")
    if K % 16:
        raise RuntimeError(f"Expected self.size(1) to be divisible by 16, but got self.size(1)={K}")
    if K2 % 16 or N % 16:
        raise RuntimeError(f"Expected both dimensions of mat2 to be divisible by 16 but got {tuple(mat2.shape)}")
    if scale_a.dtype != torch.float32 or scale_b.dtype != torch.float32:
        raise RuntimeError("_scaled_mm: scale_a and scale_b must be float32 tensors")
    if scale_a.numel() == 1 and scale_b.numel() == 1:
        pass                                           # tensorwise
    elif (scale_a.dim() == 2 and scale_b.dim() == 2 and tuple(scale_a.shape) == (M, 1)
          and tuple(scale_b.shape) == (1, N)):
        if not (scale_a.is_contiguous() and scale_b.is_contiguous()):
            raise RuntimeError("Both scale_a and scale_b must be contiguous for rowwise scaling.")
    else:
        raise RuntimeError(
            "Invalid scaling configuration for the B200 kernels: tensorwise needs two scalar scales, "
            f"rowwise needs scale_a ({M}, 1) and scale_b (1, {N}); got {tuple(scale_a.shape)} and "
            f"{tuple(scale_b.shape)}")
    odt = self.dtype if out_dtype is None else out_dtype
    if odt not in _FLOAT_DTYPES + _FP8_DTYPES:
        raise RuntimeError(f"_scaled_mm: unsupported out_dtype {odt}")
    return M, N, K, odt


def _cuda_scaled_mm(self, mat2, scale_a, scale_b, bias=None, scale_result=None, out_dtype=None,
                    use_fast_accum=False):
    if not _device_ok(self.device):
        raise RuntimeError(
            f"_scaled_mm: the fp4_fp8_for_torch_mps override is registered but {self.device} is not "
            "an sm_100 (B200) device; set FP8_B200_DISABLE_OVERRIDES=1 to use PyTorch's kernel")
    M, N, K, odt = check_scaled_mm_args(self, mat2, scale_a, scale_b, out_dtype)
    if M == 0 or N == 0:
        return torch.empty((M, N), dtype=odt, device=self.device)
    if K == 0:
        out = torch.zeros((M, N), dtype=torch.float32, device=self.device)
        if bias is not None:
            out = out + bias.float()
        return out.to(odt)
    with torch.cuda.device(self.device):
        return _native().scaled_mm(self, mat2.t(), scale_a, scale_b, bias=bias, scale_result=scale_result,
                                   out_dtype=odt, a_dtype=self.dtype, b_dtype=mat2.dtype)


def _redispatch_to_copy(keyset, self, dtype, layout, device, pin_memory, non_blocking, memory_format):
    ks = keyset.remove(_DK.CUDA)
    return torch.ops.aten._to_copy.default.redispatch(
        ks, self, dtype=dtype, layout=layout, device=device, pin_memory=pin_memory,
        non_blocking=non_blocking, memory_format=memory_format)


def _cuda_to_copy(keyset, self, *, dtype=None, layout=None, device=None, pin_memory=None,
                  non_blocking=False, memory_format=None):
    target_dtype = dtype or self.dtype
    tdev = _target_device(device, self.device)
    strided = layout in (None, torch.strided) and self.layout == torch.strided
    route = route_to_copy(self.dtype, target_dtype, strided and _device_ok(self.device),
                          tdev.type == "cuda")
    if route == TO_COPY_PASS:
        return _redispatch_to_copy(keyset, self, dtype, layout, device, pin_memory, non_blocking,
                                   memory_format)
    nat = _native()
    with torch.cuda.device(self.device):
        if route == TO_COPY_ENCODE_FP8:
            flat_src, out, flat_out = _flat_dense(self, torch.uint8, memory_format)
            nat.encode_fp8(flat_src, target_dtype, out=flat_out)
            result = out.view(target_dtype)
        elif route == TO_COPY_ENCODE_FP4:
            src = self.contiguous()
            result = nat.fp4_encode(src).view(_fp4_packed_shape(src.shape)).view(target_dtype)
        elif route == TO_COPY_DECODE_FP8:
            flat_src, out, flat_out = _flat_dense(self.view(torch.uint8), target_dtype, memory_format)
            nat.decode_fp8(flat_src, self.dtype, target_dtype, out=flat_out)
            result = out
        elif route == TO_COPY_DECODE_FP4:
            result = nat.fp4_decode(self.view(torch.uint8), target_dtype)
        elif route == TO_COPY_FP8_TO_FP8:
            wide = nat.decode_fp8(self.view(torch.uint8).contiguous(), self.dtype, torch.float32)
            result = nat.encode_fp8(wide, target_dtype).view(target_dtype)
        else:  # TO_COPY_REINTERPRET
            result = self.contiguous().view(torch.uint8).clone().view(target_dtype)
    result = _apply_memory_format(result, memory_format)
    if result.device != tdev:
        result = result.to(tdev, non_blocking=non_blocking)
    if pin_memory:
        result = result.pin_memory()
    return result


def _cuda_copy_(keyset, self, src, non_blocking=False):
    route = route_copy(self.dtype, src.dtype,
                       self.layout == torch.strided and src.layout == torch.strided
                       and _device_ok(self.device),
                       src.device.type in ("cuda", "cpu"))
    ks = keyset.remove(_DK.CUDA)
    if route == COPY_PASS:
        return torch.ops.aten.copy_.default.redispatch(ks, self, src, non_blocking)
    nat = _native()
    with torch.cuda.device(self.device):
        if route == COPY_RAW:
            # 1-byte dtypes on both sides: byte views keep any strides, and a
            # uint8 copy_ passes straight through this override
            torch.ops.aten.copy_.default.redispatch(
                ks, self.view(torch.uint8), src.view(torch.uint8), non_blocking)
            return self
        # move the source to the destination device first (it is the smaller
        # side for a decode)
        if src.device != self.device:
            src = src.to(self.device, non_blocking=non_blocking)
        if route == COPY_ENCODE_FP4:
            enc = nat.fp4_encode(src.contiguous())
            if enc.numel() != self.numel():
                raise RuntimeError(
                    f"copy_: {src.numel()} float values do not pack into {self.numel()} float4_e2m1fn_x2 bytes")
            torch.ops.aten.copy_.default.redispatch(ks, self.view(torch.uint8), enc.view(self.shape),
                                                    non_blocking)
            return self
        if src.shape != self.shape:
            src = src.expand_as(self)
        if route == COPY_ENCODE_FP8:
            if self.is_contiguous():
                nat.encode_fp8(src, self.dtype, out=self.view(torch.uint8).reshape(-1))
            else:
                enc = nat.encode_fp8(src, self.dtype)
                torch.ops.aten.copy_.default.redispatch(ks, self.view(torch.uint8), enc, non_blocking)
            return self
        if route == COPY_DECODE_FP8:
            if self.is_contiguous():
                nat.decode_fp8(src.contiguous().view(torch.uint8), src.dtype, self.dtype,
                               out=self.reshape(-1))
            else:
                dec = nat.decode_fp8(src.contiguous().view(torch.uint8), src.dtype, self.dtype)
                torch.ops.aten.copy_.default.redispatch(ks, self, dec, non_blocking)
            return self
        # COPY_FP8_TO_FP8
        wide = nat.decode_fp8(src.contiguous().view(torch.uint8), src.dtype, torch.float32)
        enc = nat.encode_fp8(wide, self.dtype)
        torch.ops.aten.copy_.default.redispatch(ks, self.view(torch.uint8), enc, non_blocking)
        return self


_aten_lib = None


def _all_gpus_sm100() -> bool | None:
    """Compute capability of every visible GPU via NVML (no CUDA context is
    created, so forking after `import torch` stays safe). None if unknown."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            n = pynvml.nvmlDeviceGetCount()
            caps = [pynvml.nvmlDeviceGetCudaComputeCapability(pynvml.nvmlDeviceGetHandleByIndex(i))
                    for i in range(n)]
        finally:
            pynvml.nvmlShutdown()
        return n > 0 and all(tuple(c) == (10, 0) for c in caps)
    except Exception:
        return None


def register_aten_overrides() -> bool:
    """Register the CUDA-key aten overrides once. Returns True if registered.

    `_to_copy` and `copy_` pass through on devices that are not sm_100, so
    they register on any CUDA build with a GPU. `_scaled_mm` replaces
    PyTorch's CUDA kernel outright, so it registers only when every visible
    GPU is an sm_100 part."""
    global _aten_lib
    if _aten_lib is not None:
        return True
    if os.environ.get("FP8_B200_DISABLE_OVERRIDES", "0") not in ("", "0"):
        return False
    if torch.version.cuda is None or not torch.cuda.is_available():
        return False
    try:
        lib = torch.library.Library("aten", "IMPL")
        lib.impl("_to_copy", _cuda_to_copy, "CUDA", with_keyset=True, allow_override=True)
        lib.impl("copy_", _cuda_copy_, "CUDA", with_keyset=True, allow_override=True)
        sm100 = _all_gpus_sm100()
        if sm100 is None:
            sm100 = all(torch.cuda.get_device_capability(i) == (10, 0)
                        for i in range(torch.cuda.device_count()))
        if sm100:
            lib.impl("_scaled_mm", _cuda_scaled_mm, "CUDA", allow_override=True)
        else:
            warnings.warn("fp4_fp8_for_torch_mps: not every GPU is sm_100 (B200); "
                          "torch._scaled_mm keeps PyTorch's kernel")
    except Exception as e:  # never break `import torch`
        warnings.warn(f"fp4_fp8_for_torch_mps: aten overrides not registered: {e}")
        return False
    _aten_lib = lib
    return True


register_aten_overrides()


# ------------------------------------------------------------------ custom ops (ops.py:172-246)
@torch.library.custom_op("fp8_mps::scaled_mm", mutates_args=())
def fp8_scaled_mm(A: torch.Tensor, B: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor) -> torch.Tensor:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp8_scaled_mm_auto
    return fp8_scaled_mm_auto(A, B, scale_a, scale_b)


@fp8_scaled_mm.register_fake
def _(A, B, scale_a, scale_b):
    return A.new_empty((A.shape[0], B.shape[0]), dtype=torch.float32)


@torch.library.custom_op("fp8_mps::encode", mutates_args=())
def fp8_encode(input: torch.Tensor) -> torch.Tensor:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp8_encode as _encode
    return _encode(input)


@fp8_encode.register_fake
def _(input):
    return input.new_empty(input.shape, dtype=torch.uint8)


@torch.library.custom_op("fp8_mps::quantize", mutates_args=())
def fp8_quantize(input: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp8_quantize as _quantize
    q, s = _quantize(input)
    return q, s.clone()


@fp8_quantize.register_fake
def _(input):
    return (input.new_empty(input.shape, dtype=torch.uint8), input.new_empty((1,), dtype=torch.float32))


@torch.library.custom_op("fp8_mps::dequantize", mutates_args=())
def fp8_dequantize(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp8_dequantize as _dequantize
    return _dequantize(input, scale)


@fp8_dequantize.register_fake
def _(input, scale):
    return input.new_empty(input.shape, dtype=torch.float16)


@torch.library.custom_op("fp8_mps::fp4_encode", mutates_args=())
def fp4_encode(input: torch.Tensor) -> torch.Tensor:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp4_encode as _encode
    return _encode(input)


@fp4_encode.register_fake
def _(input):
    return input.new_empty(input.numel() // 2, dtype=torch.uint8)


@torch.library.custom_op("fp8_mps::fp4_quantize", mutates_args=())
def fp4_quantize(input: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp4_quantize as _quantize
    q, s = _quantize(input)
    return q, s.clone()


@fp4_quantize.register_fake
def _(input):
    return (input.new_empty(input.numel() // 2, dtype=torch.uint8), input.new_empty((1,), dtype=torch.float32))


@torch.library.custom_op("fp8_mps::fp8_linear", mutates_args=())
def fp8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
               bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x @ (weight * weight_scale)^T [+ bias], float8 weights dequantised on
    load (an addition to the reference's seven ops)."""
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp8_linear as _linear
    return _linear(x, weight, weight_scale, bias)


@fp8_linear.register_fake
def _(x, weight, weight_scale, bias=None):
    return x.new_empty(tuple(x.shape[:-1]) + (weight.shape[0],))


@torch.library.custom_op("fp8_mps::fp4_scaled_mm", mutates_args=())
def fp4_scaled_mm(A: torch.Tensor, B: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                  out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """(A * scale_a) @ (B * scale_b)^T on packed FP4 operands (A: (M, K/2)
    bytes; B: (N, K/2) bytes or (N, K) float8), float32 output by default
    like fp8_mps::scaled_mm (an addition to the reference's seven ops)."""
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp4_scaled_mm as _mm
    return _mm(A, B, scale_a, scale_b, out_dtype=out_dtype or torch.float32)


@fp4_scaled_mm.register_fake
def _(A, B, scale_a, scale_b, out_dtype=None):
    return A.new_empty((A.shape[0], B.shape[0]), dtype=out_dtype or torch.float32)


@torch.library.custom_op("fp8_mps::fp4_dequantize", mutates_args=())
def fp4_dequantize(input: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    from fp4_fp8_for_torch_mps.fp8_mps_native import fp4_dequantize as _dequantize
    return _dequantize(input, scale)


@fp4_dequantize.register_fake
def _(input, scale):
    return input.new_empty(input.numel() * 2, dtype=torch.float16)

"""CPU-side tests: C-ABI library exports, argument validation that runs
before any device work, routing tables, and package registration."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "mps-fp8-for-torch-and-comfyui-python-package_b200", "fp4_fp8_for_torch_mps",
                   "libfp8_b200.so")
HDR = os.path.join(ROOT, "include", "fp8_b200.h")


def declared_symbols():
    txt = open(HDR).read()
    return sorted(set(re.findall(r"\b(fp8b200_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "run __graft_entry__.build() first"
    lib = ctypes.CDLL(LIB)
    syms = declared_symbols()
    assert len(syms) >= 11
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_library_argument_validation():
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    assert lib.fp8b200_encode_fp8(None, 7, None, L.E4M3, 16, None, None) == -1
    assert b"source dtype" in lib.fp8b200_last_error()
    assert lib.fp8b200_decode_fp8(None, L.F32, None, L.F32, 16, None, 0, None) == -1
    assert lib.fp8b200_decode_fp4(None, -1, None, L.F32, None, 0, None) == -1
    assert lib.fp8b200_decode_fp4(None, 4, None, L.BF16, None, L.SCALE_F32, None) == -1
    assert b"scale pointer" in lib.fp8b200_last_error()
    assert lib.fp8b200_decode_fp8(None, L.E4M3, None, L.BF16, 4, 64, L.SCALE_F16_REF, None) == -1
    assert lib.fp8b200_encode_fp4(None, L.F32, None, 3, None, None) == -1
    # scaled_mm shape/stride rules are checked before the device
    args = dict(lda=64, ldb=64, M=8, N=16, K=64)

    def mm(**kw):
        a = dict(args, **kw)
        return lib.fp8b200_scaled_mm(16, L.E4M3, a["lda"], 16, L.E4M3, a["ldb"], a["M"], a["N"], a["K"],
                                     16, 0, 16, 0, None, 0, None, 16, L.BF16, a["N"], None)
    assert mm(K=40) == -1 and b"multiple of 16" in lib.fp8b200_last_error()
    assert mm(lda=32) == -1 and b"row strides" in lib.fp8b200_last_error()
    assert mm(M=0) == 0  # empty output: nothing to do
    # zero-length calls are valid no-ops
    assert lib.fp8b200_encode_fp8(None, L.F32, None, L.E4M3, 0, None, None) == 0
    assert lib.fp8b200_decode_fp4(None, 0, None, L.F32, None, 0, None) == 0


def test_library_reports_missing_device():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    rc = lib.fp8b200_decode_fp8(16, L.E4M3, 16, L.F32, 16, None, 0, None)
    assert rc == -3


def test_package_registers_custom_ops():
    import fp4_fp8_for_torch_mps  # noqa: F401
    for name in ("scaled_mm", "encode", "quantize", "dequantize", "fp4_encode", "fp4_quantize",
                 "fp4_dequantize"):
        assert hasattr(torch.ops.fp8_mps, name), name


def test_fake_impls_match_reference_schemas():
    import fp4_fp8_for_torch_mps  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        a = torch.empty(8, 32, dtype=torch.uint8)
        b = torch.empty(16, 32, dtype=torch.uint8)
        s = torch.empty(1)
        assert torch.ops.fp8_mps.scaled_mm(a, b, s, s).shape == (8, 16)
        x = torch.empty(4, 6)
        assert torch.ops.fp8_mps.encode(x).dtype == torch.uint8
        q, sc = torch.ops.fp8_mps.quantize(x)
        assert q.shape == (4, 6) and sc.shape == (1,)
        assert torch.ops.fp8_mps.dequantize(q, sc).dtype == torch.float16
        assert torch.ops.fp8_mps.fp4_encode(x).shape == (12,)
        p, sc2 = torch.ops.fp8_mps.fp4_quantize(x)
        assert p.shape == (12,) and sc2.shape == (1,)
        assert torch.ops.fp8_mps.fp4_dequantize(p, sc2).shape == (24,)
        xb = torch.empty(2, 3, 32, dtype=torch.bfloat16)
        w8 = torch.empty(16, 32, dtype=torch.float8_e4m3fn)
        assert torch.ops.fp8_mps.fp8_linear(xb, w8, s).shape == (2, 3, 16)   # addition to the seven


def test_no_aten_overrides_without_cuda():
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    from fp4_fp8_for_torch_mps import ops
    assert ops._aten_lib is None
    # CPU conversions are untouched
    assert torch.tensor([1.0]).to(torch.float8_e4m3fn).view(torch.uint8).item() == 0x38


E4, E5, F4 = torch.float8_e4m3fn, torch.float8_e5m2, torch.float4_e2m1fn_x2
F32, BF, H = torch.float32, torch.bfloat16, torch.float16


@pytest.mark.parametrize("src,dst,want", [
    (F32, E4, "encode_fp8"), (BF, E5, "encode_fp8"), (H, E4, "encode_fp8"),
    (F32, F4, "encode_fp4"), (E4, F32, "decode_fp8"), (E5, BF, "decode_fp8"),
    (F4, H, "decode_fp4"), (E4, E5, "fp8_to_fp8"), (E4, F4, "reinterpret"),
    (E4, E4, "pass"), (F32, H, "pass"), (torch.int32, E4, "pass"), (E4, torch.int8, "pass"),
])
def test_to_copy_routing(src, dst, want):
    from fp4_fp8_for_torch_mps.ops import route_to_copy
    assert route_to_copy(src, dst, True, True) == want
    assert route_to_copy(src, dst, False, True) == "pass"   # not an sm_100 device
    assert route_to_copy(src, dst, True, False) == "pass"   # result wanted on the CPU


@pytest.mark.parametrize("dst,src,want", [
    (E4, F32, "encode_fp8"), (E5, BF, "encode_fp8"), (F4, F32, "encode_fp4"),
    (F32, E4, "decode_fp8"), (BF, E5, "decode_fp8"), (E4, E4, "raw_bytes"),
    (F4, F4, "raw_bytes"), (F4, E4, "raw_bytes"), (E5, E4, "fp8_to_fp8"),
    (F32, BF, "pass"), (F32, F4, "pass"),
])
def test_copy_routing(dst, src, want):
    from fp4_fp8_for_torch_mps.ops import route_copy
    assert route_copy(dst, src, True, True) == want
    assert route_copy(dst, src, False, True) == "pass"


def test_fp4_packed_shape():
    from fp4_fp8_for_torch_mps.ops import _fp4_packed_shape
    assert _fp4_packed_shape((4, 8)) == (4, 4)
    assert _fp4_packed_shape((3, 5, 2)) == (3, 5, 1)
    assert _fp4_packed_shape((2, 3)) == (3,)
    with pytest.raises(RuntimeError):
        _fp4_packed_shape((3,))


def test_redispatch_mechanism_on_cpu_key():
    """The overrides hand unsupported cases back with `keyset.remove(<backend>)`
    (reference ops.py:122-126). Exercise the same mechanism on the CPU key in a
    child process so the global registration does not leak into this one."""
    import subprocess
    import sys
    code = r'''
import torch
lib = torch.library.Library("aten", "IMPL")
seen = []
def to_copy(keyset, self, *, dtype=None, layout=None, device=None, pin_memory=None, non_blocking=False, memory_format=None):
    seen.append("to_copy")
    return torch.ops.aten._to_copy.default.redispatch(keyset.remove(torch._C.DispatchKey.CPU), self,
        dtype=dtype, layout=layout, device=device, pin_memory=pin_memory, non_blocking=non_blocking,
        memory_format=memory_format)
def copy_(keyset, self, src, non_blocking=False):
    seen.append("copy_")
    return torch.ops.aten.copy_.default.redispatch(keyset.remove(torch._C.DispatchKey.CPU), self, src, non_blocking)
lib.impl("_to_copy", to_copy, "CPU", with_keyset=True, allow_override=True)
lib.impl("copy_", copy_, "CPU", with_keyset=True, allow_override=True)
y = torch.tensor([1.0, 500.0]).to(torch.float8_e4m3fn)
assert y.view(torch.uint8).tolist() == [0x38, 0x7F], y
z = torch.empty(2, dtype=torch.float8_e4m3fn); z.copy_(torch.tensor([2.0, -0.0]))
assert z.view(torch.uint8).tolist() == [0x40, 0x80]
assert seen[:2] == ["to_copy", "copy_"], seen
print("ok")
'''
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]

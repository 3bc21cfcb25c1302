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


def test_binding_declares_every_entry_point_with_arguments():
    """Every C entry point that takes arguments has ctypes argtypes in the
    package's binding: an undeclared one would pass 64-bit pointers and
    streams as truncated C ints."""
    from fp4_fp8_for_torch_mps import _lib
    L = _lib.lib()
    txt = open(HDR).read()
    decls = re.findall(r"^(?:int|const char \*|uint64_t)\s*(fp8b200_[a-z0-9_]+)\s*\(([^)]*)\);", txt, re.M)
    assert len(decls) >= 11
    for name, args in decls:
        if args.strip() in ("", "void"):
            continue
        fn = getattr(L, name)
        assert fn.argtypes is not None, name
        assert len(fn.argtypes) == len(args.split(",")), name


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


def _fp8_pair(M, N, K, da=E4, db=E4):
    a = torch.zeros(M, K, dtype=torch.uint8).view(da)
    b = torch.zeros(N, K, dtype=torch.uint8).view(db)
    return a, b


def test_scaled_mm_argument_checks_accept():
    """The `_scaled_mm` override's argument checks, run on CPU tensors: the
    accepted modes (tensorwise and rowwise scales, mixed e4m3/e5m2, fp8 or
    16/32-bit output, views with padded row strides)."""
    from fp4_fp8_for_torch_mps.ops import check_scaled_mm_args
    s = torch.tensor(1.0)
    a, b = _fp8_pair(32, 48, 64)
    assert check_scaled_mm_args(a, b.t(), s, s) == (32, 48, 64, E4)
    assert check_scaled_mm_args(a, b.t(), s, s, BF) == (32, 48, 64, BF)
    assert check_scaled_mm_args(a.view(E5), b.t(), s, s, F32)[3] == F32
    assert check_scaled_mm_args(a, b.view(E5).t(), torch.ones(32, 1), torch.ones(1, 48), H)[3] == H
    wide_a, wide_b = _fp8_pair(32, 48, 128)
    assert check_scaled_mm_args(wide_a[:, 16:80], wide_b[:, 32:96].t(), s, s, BF)[:3] == (32, 48, 64)
    e0, e1 = _fp8_pair(0, 16, 32)
    assert check_scaled_mm_args(e0, e1.t(), s, s, BF)[:3] == (0, 16, 32)


_REJECT_WHY = {
    "fp4_operands": "operands must be float8", "int8_operands": "operands must be float8",
    "bf16_operands": "operands must be float8", "e5m2_x_e5m2": "two Float8_e5m2",
    "3d": "must be 2D", "k_mismatch": "cannot be multiplied", "mat2_row_major": "col_major",
    "self_col_major": "row_major", "k_not_16": "self.size\\(1\\) to be divisible by 16",
    "n_not_16": "mat2 to be divisible by 16", "f16_scales": "must be float32",
    "blockwise_scales": "Invalid scaling configuration", "mx_scales": "must be float32",
    "rowwise_transposed": "Invalid scaling configuration", "rowwise_noncontiguous": "contiguous",
    "int_out": "unsupported out_dtype",
}


@pytest.mark.parametrize("case", sorted(_REJECT_WHY))
def test_scaled_mm_argument_checks_reject(case):
    """Every unsupported call raises RuntimeError, for its own reason, before any
    device work: the stride/divisibility rules PyTorch's meta function enforces,
    and the modes the B200 kernels do not implement (float4_e2m1fn_x2 operands,
    block scales, e5m2 x e5m2), which raise instead of falling back to a library
    kernel."""
    from fp4_fp8_for_torch_mps.ops import check_scaled_mm_args
    s = torch.tensor(1.0)
    a, b = _fp8_pair(32, 48, 64)
    args = {
        "fp4_operands": (a.view(F4), b.view(F4).t(), s, s),
        "int8_operands": (a.view(torch.int8), b.view(torch.int8).t(), s, s),
        "bf16_operands": (torch.zeros(32, 64, dtype=BF), torch.zeros(48, 64, dtype=BF).t(), s, s),
        "e5m2_x_e5m2": (a.view(E5), b.view(E5).t(), s, s),
        "3d": (a.unsqueeze(0), b.t(), s, s),
        "k_mismatch": (a, _fp8_pair(32, 48, 80)[1].t(), s, s),
        "mat2_row_major": (a, torch.zeros(64, 48, dtype=torch.uint8).view(E4), s, s),
        "self_col_major": (torch.zeros(64, 32, dtype=torch.uint8).view(E4).t(), b.t(), s, s),
        "k_not_16": (a[:, :40], b[:, :40].t(), s, s),
        "n_not_16": (a, _fp8_pair(32, 40, 64)[1].t(), s, s),
        "f16_scales": (a, b.t(), s.half(), s.half()),
        "blockwise_scales": (a, b.t(), torch.ones(32, 2), s),
        "mx_scales": (a, b.t(), torch.ones(32, 2).to(torch.float8_e8m0fnu),
                      torch.ones(48, 2).to(torch.float8_e8m0fnu)),
        "rowwise_transposed": (a, b.t(), torch.ones(1, 32), torch.ones(48, 1)),
        "rowwise_noncontiguous": (a, b.t(), torch.ones(32, 2)[:, :1], torch.ones(1, 48)),
        "int_out": (a, b.t(), s, s, torch.int32),
    }
    with pytest.raises(RuntimeError, match=_REJECT_WHY[case]):
        check_scaled_mm_args(*args[case])


@pytest.mark.parametrize("M,N,want", [
    (256, 14336, False),    # at most 256 rows: never decoded once
    (257, 14336, True),     # 2 x 56 = 112 tiles of 256 x 256 > 74 CTA pairs
    (320, 14336, True),
    (1024, 4096, False),    # 4 x 16 = 64 tiles: one wave of the dequant-on-load kernel
    (768, 6144, False),     # 3 x 24 = 72 tiles
    (1024, 6144, True),     # 4 x 24 = 96 tiles
    (16384, 256, False),    # 64 x 1 = 64 tiles: one wave
    (19200, 256, True),     # 75 x 1 = 75 tiles > 74
])
def test_linear_decode_once_rule(monkeypatch, M, N, want):
    """fp8_linear's choice between dequant-on-load and decode-once + 16-bit GEMM, for a
    148-SM device (74 CTA pairs), without touching a GPU."""
    import fp4_fp8_for_torch_mps.fp8_mps_native as nat
    monkeypatch.setattr(nat, "_SM_COUNT", {0: 148})
    assert nat.linear_decodes_once(M, N, torch.device("cuda", 0)) == want

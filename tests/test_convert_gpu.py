"""Device parity of the conversion kernels (called through the C ABI via the
package launchers and the aten overrides) against the CPU oracle, CPU
PyTorch and the golden fixtures. Bit-exact everywhere: these are
byte/bit-pattern conversions."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

FP8 = {0: torch.float8_e4m3fn, 1: torch.float8_e5m2}
OUT = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}
UINT = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}
NPU = {torch.float32: np.uint32, torch.bfloat16: np.uint16, torch.float16: np.uint16}
SCALES = {"037": 0.37, "1": 1.0, "3": 3.0}


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.view(UINT[t.dtype]).numpy().view(NPU[t.dtype])


@pytest.fixture(scope="module")
def nat(device):
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


# ---------------------------------------------------------------- decode
@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("odt", [0, 1, 2])
def test_decode_all_codes(nat, golden, fmt, odt):
    codes = torch.arange(256, dtype=torch.uint8, device="cuda")
    out = nat.decode_fp8(codes, FP8[fmt], OUT[odt])
    assert np.array_equal(bits(out), golden[f"decode_f{fmt}_o{odt}"])
    out2 = codes.view(FP8[fmt]).to(OUT[odt])          # aten route: .to() on the device
    assert np.array_equal(bits(out2), golden[f"decode_f{fmt}_o{odt}"])
    dst = torch.empty(256, dtype=OUT[odt], device="cuda")
    dst.copy_(codes.view(FP8[fmt]))                     # aten route: copy_
    assert np.array_equal(bits(dst), golden[f"decode_f{fmt}_o{odt}"])


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 255, 4097, 1000003, 16777216 + 4096 + 48 + 5])
@pytest.mark.parametrize("offset", [0, 1, 3, 16])
def test_decode_ragged_and_unaligned(nat, n, offset):
    g = torch.Generator().manual_seed(n + offset)
    host = torch.randint(0, 256, (n + offset,), dtype=torch.uint8, generator=g)
    dev = host.cuda()[offset:]
    for fmt in (0, 1):
        for odt in (0, 1, 2):
            out = nat.decode_fp8(dev, FP8[fmt], OUT[odt])
            ref = O.decode_fp8(host[offset:].numpy(), fmt, odt)
            assert np.array_equal(bits(out), ref), (fmt, odt)


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("odt", [0, 1, 2])
@pytest.mark.parametrize("sc", list(SCALES))
def test_decode_scaled_f32(nat, fmt, odt, sc):
    codes = torch.arange(256, dtype=torch.uint8, device="cuda").repeat(41)
    out = bits(nat.decode_fp8(codes, FP8[fmt], OUT[odt], scale=torch.tensor([SCALES[sc]])))
    ref = O.decode_fp8(codes.cpu().numpy(), fmt, odt, scale=SCALES[sc])
    assert np.array_equal(out, ref)


@pytest.mark.parametrize("sc", list(SCALES))
def test_fp8_dequantize_reference_semantics(nat, golden, sc):
    codes = torch.arange(256, dtype=torch.uint8, device="cuda")
    out = nat.fp8_dequantize(codes, torch.tensor([SCALES[sc]]))
    assert out.dtype == torch.float16 and out.shape == (256,)
    assert np.array_equal(bits(out), golden[f"deqref_f0_s{sc}"])
    out2 = torch.ops.fp8_mps.dequantize(codes, torch.tensor([SCALES[sc]], device="cuda"))
    assert np.array_equal(bits(out2), golden[f"deqref_f0_s{sc}"])


# ---------------------------------------------------------------- encode
@pytest.mark.parametrize("fmt", [0, 1])
def test_encode_every_f32_bit_pattern(nat, fmt):
    """All 2^32 float32 bit patterns, in 2^28 chunks, against CPU PyTorch."""
    chunk = 1 << 28
    out = torch.empty(chunk, dtype=torch.uint8, device="cuda")
    for lo in range(0, 1 << 32, chunk):
        x = torch.arange(lo, lo + chunk, dtype=torch.int64, device="cuda").to(torch.int32).view(torch.float32)
        nat.encode_fp8(x, FP8[fmt], out=out)
        del x
        xc = torch.arange(lo, lo + chunk, dtype=torch.int64).to(torch.int32).view(torch.float32)
        ref = xc.to(FP8[fmt]).view(torch.uint8)
        got = out.cpu()
        if not torch.equal(got, ref):
            bad = (got != ref).nonzero()[0].item()
            pytest.fail(f"fmt {fmt}: pattern {lo + bad:#010x}: got {got[bad].item():#04x} "
                        f"want {ref[bad].item():#04x}")


@pytest.mark.parametrize("src", ["bf16", "f16"])
@pytest.mark.parametrize("fmt", [0, 1])
def test_encode_every_16bit_pattern(nat, golden, src, fmt):
    dt = torch.bfloat16 if src == "bf16" else torch.float16
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(dt).cuda()
    out = nat.encode_fp8(x, FP8[fmt])
    assert np.array_equal(out.cpu().numpy(), golden[f"encode_{src}_f{fmt}"])
    out2 = x.to(FP8[fmt]).view(torch.uint8)
    assert np.array_equal(out2.cpu().numpy(), golden[f"encode_{src}_f{fmt}"])


@pytest.mark.parametrize("fmt", [0, 1])
def test_encode_planted_edges_and_reference_known_answers(nat, golden, fmt):
    x = torch.from_numpy(golden["edge_f32"].view(np.int32).copy()).view(torch.float32).cuda()
    assert np.array_equal(nat.encode_fp8(x, FP8[fmt]).cpu().numpy(), golden[f"edge_f32_f{fmt}"])
    if fmt == 0:
        for k in ("exact", "mid", "five"):
            v = torch.from_numpy(golden[f"kat_{k}_f32"].view(np.int32).copy()).view(torch.float32).cuda()
            assert np.array_equal(torch.ops.fp8_mps.encode(v).cpu().numpy(), golden[f"kat_{k}_e4m3"]), k


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 1000003, 4096 * 444 * 3 + 16 * 7 + 9])
@pytest.mark.parametrize("offset", [0, 1, 8])
@pytest.mark.parametrize("sdt", [0, 1, 2])
def test_encode_ragged_and_unaligned(nat, n, offset, sdt):
    g = torch.Generator().manual_seed(7 * n + offset)
    x = (torch.randn(n + offset, generator=g) * 300).to(OUT[sdt])
    dev = x.cuda()[offset:]
    for fmt in (0, 1):
        out = nat.encode_fp8(dev, FP8[fmt])
        ref = O.encode_fp8(bits(x[offset:]), sdt, fmt)
        assert np.array_equal(out.cpu().numpy(), ref), fmt


@pytest.mark.parametrize("fmt", [0, 1])
def test_fp8_roundtrip_workload(nat, fmt):
    """The FP8 round-trip workload (4096x4096 f32, N(0,1)*64, planted edges):
    encode via .to(), decode back to every float dtype, bit-exact."""
    from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
    x = fp8_roundtrip_input()
    enc = x.cuda().to(FP8[fmt])
    ref = O.encode_fp8(x.view(torch.int32).numpy().view(np.uint32), 0, fmt, threads=8)
    assert np.array_equal(enc.view(torch.uint8).cpu().numpy(), ref)
    for odt in (0, 1, 2):
        dec = enc.to(OUT[odt])
        assert np.array_equal(bits(dec), O.decode_fp8(ref, fmt, odt, threads=8)), odt
    for sdt in (1, 2):  # from bf16/f16 casts of the same data
        xs = x.to(OUT[sdt])
        e2 = xs.cuda().to(FP8[fmt]).view(torch.uint8).cpu().numpy()
        assert np.array_equal(e2, O.encode_fp8(bits(xs), sdt, fmt, threads=8)), sdt


def test_aten_routes_layouts_and_devices(nat):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 3, 8, 5, generator=g) * 40
    xd = x.cuda().to(memory_format=torch.channels_last)
    e = xd.to(torch.float8_e4m3fn)                      # preserve_format keeps channels_last
    assert e.is_contiguous(memory_format=torch.channels_last)
    assert torch.equal(e.contiguous().view(torch.uint8).cpu(), x.to(torch.float8_e4m3fn).view(torch.uint8))
    t = x.cuda().transpose(1, 3)                        # dense non-contiguous
    assert torch.equal(t.to(torch.float8_e5m2).contiguous().view(torch.uint8).cpu(),
                       x.transpose(1, 3).to(torch.float8_e5m2).contiguous().view(torch.uint8))
    s = x.cuda()[:, :, ::2]                             # non-dense slice
    assert torch.equal(s.to(torch.float8_e4m3fn).view(torch.uint8).cpu(),
                       x[:, :, ::2].to(torch.float8_e4m3fn).view(torch.uint8))
    c = x.to("cuda", dtype=torch.float8_e4m3fn)         # CPU float -> CUDA fp8 (copy_ route)
    assert torch.equal(c.view(torch.uint8).cpu(), x.to(torch.float8_e4m3fn).view(torch.uint8))
    f = x.to(torch.float8_e4m3fn).to("cuda")            # raw bytes CPU -> CUDA
    assert torch.equal(f.view(torch.uint8).cpu(), x.to(torch.float8_e4m3fn).view(torch.uint8))
    d = c.to(torch.float8_e5m2)                         # fp8 -> fp8 converts values, as CPU torch
    assert torch.equal(d.view(torch.uint8).cpu(),
                       x.to(torch.float8_e4m3fn).to(torch.float8_e5m2).view(torch.uint8))
    dst = torch.empty(2, 3, 8, 5, dtype=torch.float8_e4m3fn, device="cuda")
    dst.copy_(x)                                        # copy_ from CPU float
    assert torch.equal(dst.view(torch.uint8).cpu(), x.to(torch.float8_e4m3fn).view(torch.uint8))
    y = x.cuda()
    assert y.to(torch.float16).dtype == torch.float16   # untouched ops still work
    assert y.to("cpu").device.type == "cpu"


# ---------------------------------------------------------------- quantize
@pytest.mark.parametrize("sdt", [0, 1, 2])
@pytest.mark.parametrize("n", [1, 4096, 1 << 20, (1 << 20) + 7])
def test_quantize_matches_reference_formula(nat, sdt, n):
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 5).to(OUT[sdt])
    q, inv = nat.fp8_quantize(x.cuda())
    xf = x.float()
    amax = xf.abs().max().item()
    scale = 448.0 / amax if amax > 0 else 1.0
    ref = O.encode_fp8_scaled(xf.numpy(), scale, 0)
    assert np.array_equal(q.cpu().numpy(), ref)
    assert inv.item() == np.float32(1.0 / scale)
    q2, s2 = torch.ops.fp8_mps.quantize(x.cuda())
    assert torch.equal(q2.cpu(), q.cpu()) and s2.shape == (1,)


def test_quantize_zero_input_and_repeat(nat):
    q, inv = nat.fp8_quantize(torch.zeros(1000, device="cuda"))
    assert int(q.sum().item()) == 0 and inv.item() == 1.0
    # the amax scratch is cleared by every call: a large tensor then a small one
    nat.fp8_quantize(torch.full((4096,), 1000.0, device="cuda"))
    q, inv = nat.fp8_quantize(torch.full((16,), 2.0, device="cuda"))
    assert inv.item() == np.float32(1.0 / (448.0 / 2.0))


@pytest.mark.parametrize("sdt", [0, 1, 2])
@pytest.mark.parametrize("offset", [1, 2, 8])
def test_quantize_unaligned_views(nat, sdt, offset):
    """Per-tensor fp8 and FP4 quantize of views that start off the 16-byte
    boundary: the element-wise amax, scale and encode kernels instead of the
    bulk ones, same results as the oracle."""
    n = 300002
    x = (torch.randn(n + offset, generator=torch.Generator().manual_seed(offset)) * 7).to(OUT[sdt])
    dev = x.cuda()[offset:]
    xf = x[offset:].float().numpy()
    amax = float(np.max(np.abs(xf)))
    q, sc = nat.quantize_fp8(dev, torch.float8_e4m3fn)
    assert sc[0].item() == np.float32(448.0 / amax)
    assert np.array_equal(q.cpu().numpy(), O.encode_fp8_scaled(xf, 448.0 / amax, 0))
    enc, inv = torch.ops.fp8_mps.fp4_quantize(dev)
    assert inv.item() == np.float32(1.0 / (6.0 / amax))
    assert np.array_equal(enc.cpu().numpy(), O.fp4_encode_ref(xf, 6.0 / amax))


@pytest.mark.parametrize("sdt", [0, 1])
@pytest.mark.parametrize("n", [4096 * 300 + 3, 1 << 22, (1 << 24) + 24])
def test_quantize_amax_position(nat, sdt, n):
    """The amax reduction finds a lone maximum wherever it sits: first
    element, middle, the last vectorised unit, the scalar tail."""
    base = (torch.rand(n, generator=torch.Generator().manual_seed(n)) - 0.5).to(OUT[sdt])
    per_unit = 8 if sdt == 0 else 16
    for pos in (0, n // 2, (n // per_unit - 1) * per_unit, n - 1):
        for v in (1000.0, -1000.0):
            x = base.clone()
            x[pos] = v
            q, sc = nat.quantize_fp8(x.cuda(), torch.float8_e4m3fn)
            assert sc[0].item() == np.float32(448.0 / 1000.0), (pos, v)
            assert q.view(-1)[pos].item() == (0x7E if v > 0 else 0xFE), (pos, v)


@pytest.mark.parametrize("case", ["randn_e4m3", "randn_e5m2", "planted_e4m3"])
def test_quantize_full_size(nat, case):
    """Per-tensor quantize at the 4096x4096 f32 workload size: thousands of
    chunks per launch, several per CTA, walked last-to-first by the encoder.
    Every element against the oracle; the planted input (NaN, inf, every
    code and midpoint) has a NaN amax, so its scale is 1."""
    from fp4_fp8_for_torch_mps.workloads import fp8_roundtrip_input
    fmt = 1 if case.endswith("e5m2") else 0
    if case.startswith("planted"):
        x = fp8_roundtrip_input(seed=3)
    else:
        x = torch.randn(4096, 4096, generator=torch.Generator().manual_seed(11)) * 64
    q, sc = nat.quantize_fp8(x.cuda(), FP8[fmt])
    xf = x.reshape(-1).numpy()
    amax = float(np.max(np.abs(xf)))
    scale = (57344.0 if fmt else 448.0) / amax if amax > 0 else 1.0
    assert sc[0].item() == np.float32(scale) and sc[1].item() == np.float32(1.0 / scale)
    assert np.array_equal(q.reshape(-1).cpu().numpy(), O.encode_fp8_scaled(xf, scale, fmt))


# ---------------------------------------------------------------- fp4
@pytest.mark.parametrize("odt", [0, 1, 2])
@pytest.mark.parametrize("sc", list(SCALES))
def test_fp4_decode_all_bytes(nat, golden, odt, sc):
    b = torch.arange(256, dtype=torch.uint8, device="cuda")
    out = nat.fp4_decode(b, OUT[odt], scale=torch.tensor([SCALES[sc]]))
    assert out.shape == (512,)
    assert np.array_equal(bits(out), golden[f"fp4_s{sc}_o{odt}"])


@pytest.mark.parametrize("sc", list(SCALES))
def test_fp4_dequantize_reference_op(nat, golden, sc):
    b = torch.arange(256, dtype=torch.uint8, device="cuda")
    out = torch.ops.fp8_mps.fp4_dequantize(b, torch.tensor([SCALES[sc]], device="cuda"))
    assert out.dtype == torch.float16 and out.shape == (512,)
    assert np.array_equal(bits(out), golden[f"fp4ref_s{sc}"])


@pytest.mark.parametrize("odt", [0, 1])
def test_fp4_decode_workload_full_size(nat, odt):
    """The FP4 decode workload: 16384x8192 bytes (exhaustive 256-byte prefix),
    x 0.37, to bf16 and f32, bit-exact against the oracle."""
    from fp4_fp8_for_torch_mps.workloads import fp4_decode_input
    x = fp4_decode_input()
    out = nat.fp4_decode(x.cuda().view(torch.float4_e2m1fn_x2), OUT[odt], scale=torch.tensor([0.37]))
    assert out.shape == (16384, 16384)
    ref = O.fp4_decode(x.numpy(), odt, 0.37, threads=8)
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("n", [0, 1, 15, 17, 1000003, 4096 * 296 * 5 + 16 * 3 + 11])
@pytest.mark.parametrize("offset", [0, 1, 16])
def test_fp4_decode_ragged_unaligned(nat, n, offset):
    g = torch.Generator().manual_seed(n)
    host = torch.randint(0, 256, (n + offset,), dtype=torch.uint8, generator=g)
    for odt in (0, 1, 2):
        out = nat.fp4_decode(host.cuda()[offset:], OUT[odt], scale=torch.tensor([1.5]))
        assert np.array_equal(bits(out), O.fp4_decode(host[offset:].numpy(), odt, 1.5)), odt


def test_fp4_aten_routes(nat):
    x = torch.tensor([[0.5, 1.0, 2.0, 3.0], [-1.0, -4.0, 0.0, 6.0]], device="cuda")
    f4 = x.to(torch.float4_e2m1fn_x2)
    assert f4.dtype == torch.float4_e2m1fn_x2 and f4.shape == (2, 2)
    back = f4.to(torch.float32)
    assert back.shape == (2, 4) and torch.equal(back.cpu(), x.cpu())
    cpu4 = torch.zeros(4, dtype=torch.uint8).view(torch.float4_e2m1fn_x2)
    assert torch.equal(cpu4.to("cuda").view(torch.uint8).cpu(), cpu4.view(torch.uint8))
    dst = torch.empty(2, 2, dtype=torch.float4_e2m1fn_x2, device="cuda")
    dst.copy_(f4)
    assert torch.equal(dst.view(torch.uint8), f4.view(torch.uint8))


@pytest.mark.parametrize("n", [2, 30, 32, 34, 100002, 4096 * 300 + 4098])
@pytest.mark.parametrize("sdt", [0, 1, 2])
def test_fp4_encode_reference_thresholds(nat, n, sdt):
    special = np.array([0.0, -0.0, 0.24, 0.25, 0.74, 0.75, 1.25, 1.74, 1.75, 2.49, 2.5, 3.49, 3.5,
                        4.99, 5.0, 100.0, -100.0, -0.001, np.nan, -np.inf, 6.0, -6.0], np.float32)
    vals = (np.random.default_rng(n).standard_normal(n) * 3).astype(np.float32)
    vals[: min(n, special.size)] = special[: min(n, special.size)]
    x = torch.from_numpy(vals).to(OUT[sdt])
    enc = torch.ops.fp8_mps.fp4_encode(x.cuda()).cpu().numpy()
    assert np.array_equal(enc, O.fp4_encode_ref(x.float().numpy()))


@pytest.mark.parametrize("n", [4098, (1 << 20) + 6])
@pytest.mark.parametrize("sdt", [0, 1, 2])
def test_fp4_quantize_matches_reference_formula(nat, n, sdt):
    x = (torch.randn(n, generator=torch.Generator().manual_seed(5)) * 3).to(OUT[sdt])
    enc, inv = torch.ops.fp8_mps.fp4_quantize(x.cuda())
    xf = x.float()
    amax = xf.abs().max().item()
    scale = 6.0 / amax
    assert np.array_equal(enc.cpu().numpy(), O.fp4_encode_ref(xf.numpy(), scale))
    assert inv.item() == np.float32(1.0 / scale) and enc.shape == (n // 2,)


def test_fp4_quantize_full_size(nat):
    """Per-tensor FP4 quantize of 8192x8192 bf16 (several chunks per CTA,
    walked last-to-first by the encoder), every byte against the oracle."""
    x = (torch.randn(8192, 8192, generator=torch.Generator().manual_seed(12)) * 3).to(torch.bfloat16)
    enc, inv = torch.ops.fp8_mps.fp4_quantize(x.cuda())
    xf = x.float().reshape(-1).numpy()
    scale = 6.0 / float(np.max(np.abs(xf)))
    assert inv.item() == np.float32(1.0 / scale)
    assert np.array_equal(enc.cpu().numpy(), O.fp4_encode_ref(xf, scale))


@pytest.mark.parametrize("sdt", [1, 2])
def test_fp4_encode_every_16bit_pattern(nat, sdt):
    """All 65536 bf16 / f16 bit patterns (NaNs, infs, signed zeros,
    subnormals), unscaled and scaled, against the reference thresholds."""
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(OUT[sdt])
    for scale in (None, 0.37):
        dev = x.cuda()
        out = torch.empty(32768, dtype=torch.uint8, device="cuda")
        sc = None if scale is None else torch.tensor([scale], dtype=torch.float32, device="cuda")
        from fp4_fp8_for_torch_mps import _lib as L
        L.check(L.lib().fp8b200_encode_fp4(dev.data_ptr(), sdt, out.data_ptr(), 65536,
                                           None if sc is None else sc.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream), "fp4 encode")
        assert np.array_equal(out.cpu().numpy(), O.fp4_encode_ref(x.float().numpy(), scale)), scale


def test_fp4_encode_every_f32_pattern(nat):
    """All 2^32 float bit patterns, in 16 slices, against the reference
    thresholds (the bulk encoder converts with cvt.rn.satfinite.e2m1x2 and
    falls back to the thresholds for the inputs where the two differ)."""
    out = torch.empty(1 << 27, dtype=torch.uint8, device="cuda")
    from fp4_fp8_for_torch_mps import _lib as L
    for k in range(16):
        lo = k << 28
        bits = np.arange(lo, lo + (1 << 28), dtype=np.uint64).astype(np.uint32)
        dev = torch.arange(lo, lo + (1 << 28), dtype=torch.int64, device="cuda").to(torch.int32)
        L.check(L.lib().fp8b200_encode_fp4(dev.data_ptr(), 0, out.data_ptr(), 1 << 28, None,
                                           torch.cuda.current_stream().cuda_stream), "fp4 encode")
        assert np.array_equal(out.cpu().numpy(), O.fp4_encode_ref(bits.view(np.float32))), hex(lo)


def test_fp4_encode_f32_near_every_threshold(nat):
    """f32 values within 4096 ulps of each threshold (0.25 ... 5) and of the
    e2m1 values, both signs, plus 2^22 random bit patterns."""
    marks = np.array([0.25, 0.5, 0.75, 1.0, 1.25, 1.5, 1.75, 2.0, 2.5, 3.0, 3.5, 4.0, 5.0, 6.0, 8.0], np.float32)
    near = (marks.view(np.uint32)[:, None] + np.arange(-4096, 4096, dtype=np.int64)[None, :]).astype(np.uint32)
    rnd = np.random.default_rng(9).integers(0, 1 << 32, size=1 << 22, dtype=np.uint64).astype(np.uint32)
    bits = np.concatenate([near.reshape(-1), near.reshape(-1) | np.uint32(0x80000000), rnd])
    bits = bits[: bits.size // 2 * 2]
    x = torch.from_numpy(bits.view(np.int32).copy()).view(torch.float32)
    enc = torch.ops.fp8_mps.fp4_encode(x.cuda()).cpu().numpy()
    assert np.array_equal(enc, O.fp4_encode_ref(bits.view(np.float32)))


# ---------------------------------------------------------------- per-row quantize
@pytest.mark.parametrize("rows,cols", [(1, 16), (3, 17), (64, 4096), (37, 14336), (5, 1000), (2, 70000),
                                       (300, 512), (1000, 2048), (9, 4080), (17, 1024), (40, 4112)])
@pytest.mark.parametrize("sdt", [0, 1, 2])
@pytest.mark.parametrize("fmt", [0, 1])
def test_quantize_rows(nat, rows, cols, sdt, fmt):
    g = torch.Generator().manual_seed(rows * cols + sdt)
    x = (torch.randn(rows, cols, generator=g) * torch.rand(rows, 1, generator=g) * 50).to(OUT[sdt])
    if rows > 2:
        x[1] = 0                                  # all-zero row -> scale 1
        x[2, cols // 2] = float("nan")            # NaN row -> scale 1, NaN code
    if rows > 5:
        x[3, cols - 1] = float("-inf")            # inf row -> scale 0, NaN / zero codes
        x[4] = 0
        x[4, 0] = 1e-40 if sdt != 2 else 6e-8     # tiny amax -> scale overflows to inf
        x[5, 1] = 60000.0                          # large amax among ordinary values
    codes, inv = nat.quantize_rows_fp8(x.cuda(), FP8[fmt])
    assert codes.dtype == FP8[fmt] and codes.shape == (rows, cols) and inv.shape == (rows, 1)
    fmax = 448.0 if fmt == 0 else 57344.0
    xf = x.float().numpy()
    got = codes.view(torch.uint8).cpu().numpy()
    gi = inv.cpu().numpy().reshape(-1)
    for r in range(rows):
        amax = np.float64(np.max(np.abs(xf[r])))
        sd = fmax / amax if amax > 0 else 1.0
        with np.errstate(divide="ignore"):        # inf row: scale 0, inverse inf
            assert gi[r] == np.float32(1.0 / sd), r
        assert np.array_equal(got[r], O.encode_fp8_scaled(xf[r], np.float32(sd), fmt)), r


def test_quantize_rows_feeds_rowwise_scaled_mm(nat):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(256, 512, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(384, 512, generator=g) * 0.02).cuda()
    wq, ws = nat.quantize_fp8(w)
    xq, xs = nat.quantize_rows_fp8(x)
    y = torch._scaled_mm(xq, wq.view(torch.float8_e4m3fn).t(), xs, ws[1:2].expand(1, 384).contiguous(),
                         out_dtype=torch.bfloat16)
    ref = x.float() @ w.float().t()
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 0.05

"""Device parity of the GEMM on packed FP4 (float4_e2m1fn_x2) operands —
fp8b200_scaled_mm with FP8B200_E2M1 operands, the launcher fp4_scaled_mm and
the custom op fp8_mps::fp4_scaled_mm — against the float64 oracle.

Tolerance, FP4 x FP4: every e2m1 value is a multiple of 0.5 with |v| <= 6, so
each product is a multiple of 0.25 of magnitude <= 36 and every partial sum
over K <= 2^16 is an integer multiple of 0.25 below 2^22 · 0.25 · 36 <
2^24 · 0.25: the float32 accumulation is exact in any order. The only
rounding is the epilogue's, so the bar is

    |out - r| <= ulp_out(|r|)        (one output ulp, no accumulation term)

Mixed FP4 x float8 products need the float8 tolerance of
tests/test_scaled_mm_gpu.py: |out - r| <= ulp_out(|r|) + 2^-20 * S.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

E4, E5 = torch.float8_e4m3fn, torch.float8_e5m2
FP4 = torch.float4_e2m1fn_x2
ACC_TOL = 2.0 ** -20


def ulp(x, dtype):
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(ax)) - mant)


def check(out, ref, S, acc_tol, what):
    o = out.float().cpu().double().numpy()
    err = np.abs(o - ref)
    tol = ulp(ref, out.dtype) + acc_tol * S
    bad = err > tol
    if bad.any():
        i = tuple(np.argwhere(bad)[0])
        pytest.fail(f"{what}: {bad.sum()} of {bad.size} outside tolerance; first at {i}: "
                    f"out {o[i]!r} ref {ref[i]!r} tol {tol[i]!r}")
    return float((err / ulp(ref, out.dtype)).max())


@pytest.fixture(scope="module")
def nat(device):
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


@pytest.fixture(params=[1, 2, 3, 4], ids=["single_cta", "cta_pair", "small_m", "cta_pair_wide"])
def path(request, nat):
    from fp4_fp8_for_torch_mps import _lib as L
    L.check(L.lib().fp8b200_gemm_set_path(request.param), "gemm path")
    yield request.param
    L.check(L.lib().fp8b200_gemm_set_path(0), "gemm path")


def rand_fp4(rows, k, gen):
    """Packed FP4 bytes, every byte value equally likely (all 16 codes in both nibbles)."""
    return torch.randint(0, 256, (rows, k // 2), dtype=torch.uint8, generator=gen)


def rand_fp8(shape, dtype, gen, scale=100.0):
    return (torch.randn(*shape, generator=gen) * scale).clamp(-440, 440).to(dtype)


SHAPES = [(1, 16, 128), (16, 128, 256), (17, 48, 128), (128, 256, 128), (129, 272, 384),
          (300, 528, 1024), (256, 512, 4096), (1000, 1008, 2048)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("rowwise", [False, True])
def test_fp4_x_fp4(nat, path, M, N, K, rowwise):
    g = torch.Generator().manual_seed(M * 5 + N * 3 + K)
    a, b = rand_fp4(M, K, g), rand_fp4(N, K, g)
    if rowwise:
        sa = torch.rand(M, 1, generator=g) * 0.5 + 0.01
        sb = torch.rand(1, N, generator=g) * 0.5 + 0.01
    else:
        sa, sb = torch.tensor(0.37), torch.tensor(1.25)
    out = nat.scaled_mm(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16,
                        a_dtype=FP4, b_dtype=FP4)
    ref, S = O.scaled_mm_ref(a.numpy(), b.numpy(), sa.numpy().reshape(-1), sb.numpy().reshape(-1),
                             fmt_a=O.FP4, fmt_b=O.FP4)
    check(out, ref, S, 0.0, f"fp4 x fp4 {M}x{N}x{K} rowwise={rowwise}")


def test_every_code_pair(nat, path):
    """Row i of A is the FP4 code i (all 16 codes), column j of B the code j:
    out[i, j] = K * v_i * v_j for all 256 code pairs, f32 output (exact)."""
    K = 256
    a = torch.arange(16, dtype=torch.uint8).mul(17).reshape(16, 1).expand(16, K // 2).contiguous()
    b = torch.arange(16, dtype=torch.uint8).mul(17).reshape(16, 1).expand(16, K // 2).contiguous()
    b = b.repeat(2, 1)  # N = 32 (two copies) so every kernel accepts the shape
    out = nat.scaled_mm(a.cuda(), b.cuda(), torch.tensor(1.0).cuda(), torch.tensor(1.0).cuda(),
                        out_dtype=torch.float32, a_dtype=FP4, b_dtype=FP4).cpu().numpy()
    v = O.fp4_values().astype(np.float64)
    expect = K * np.outer(v, np.concatenate([v, v]))
    assert np.array_equal(out.astype(np.float64), expect)


@pytest.mark.parametrize("fmts", [(FP4, E4), (E4, FP4), (FP4, E5), (E5, FP4)],
                         ids=["fp4_e4m3", "e4m3_fp4", "fp4_e5m2", "e5m2_fp4"])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_mixed_fp4_fp8(nat, path, fmts, out_dtype):
    M, N, K = 200, 320, 512
    g = torch.Generator().manual_seed(23)
    fa, fb = fmts

    def make(rows, fmt):
        if fmt == FP4:
            return rand_fp4(rows, K, g), O.FP4
        return rand_fp8((rows, K), fmt, g, 4.0 if fmt == E4 else 100.0).view(torch.uint8), \
            (O.E4M3 if fmt == E4 else O.E5M2)

    (a, oa), (b, ob) = make(M, fa), make(N, fb)
    sa = torch.rand(M, 1, generator=g) * 0.1 + 1e-3
    sb = torch.tensor(0.05)
    out = nat.scaled_mm(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), out_dtype=out_dtype, a_dtype=fa, b_dtype=fb)
    ref, S = O.scaled_mm_ref(a.numpy(), b.numpy(), sa.numpy().reshape(-1), sb.numpy().reshape(-1),
                             fmt_a=oa, fmt_b=ob)
    check(out, ref, S, ACC_TOL, f"{fa} x {fb} -> {out_dtype}")


def test_bias_and_scale_result(nat):
    M, N, K = 256, 512, 1024
    g = torch.Generator().manual_seed(5)
    a, b = rand_fp4(M, K, g), rand_fp4(N, K, g)
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    sr = torch.tensor([0.5])
    out = nat.scaled_mm(a.cuda(), b.cuda(), torch.tensor(0.25).cuda(), torch.tensor(0.75).cuda(),
                        bias=bias.cuda(), scale_result=sr.cuda(), out_dtype=torch.float32,
                        a_dtype=FP4, b_dtype=FP4)
    ref, S = O.scaled_mm_ref(a.numpy(), b.numpy(), 0.25, 0.75, fmt_a=O.FP4, fmt_b=O.FP4,
                             bias=bias.float().numpy())
    ref = ref * 0.5
    check(out, ref, S, 0.0, "bias + scale_result")


def test_custom_op_from_fp4_quantize(nat):
    """The end-to-end FP4 path: fp8_mps::fp4_quantize both operands (the
    reference's FP4 producer), then fp8_mps::fp4_scaled_mm with the returned
    inverse scales; checked against the oracle's product of the packed codes."""
    M, N, K = 384, 1024, 2048
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M, K, generator=g).cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).cuda()
    qx, sx = torch.ops.fp8_mps.fp4_quantize(x)
    qw, sw = torch.ops.fp8_mps.fp4_quantize(w)
    qx, qw = qx.reshape(M, K // 2), qw.reshape(N, K // 2)
    out = torch.ops.fp8_mps.fp4_scaled_mm(qx, qw.view(FP4), sx, sw)
    assert out.shape == (M, N) and out.dtype == torch.float32
    ref, S = O.scaled_mm_ref(qx.cpu().numpy(), qw.cpu().numpy(), sx.item(), sw.item(),
                             fmt_a=O.FP4, fmt_b=O.FP4)
    check(out, ref, S, 0.0, "fp4_quantize -> fp4_scaled_mm")
    # the float4 product approximates the float product of the inputs
    rel = (out - x @ w.t()).norm() / (x @ w.t()).norm()
    assert rel.item() < 0.25
    bf = torch.ops.fp8_mps.fp4_scaled_mm(qx, qw, sx, sw, out_dtype=torch.bfloat16)
    assert bf.dtype == torch.bfloat16
    check(bf, ref, S, 0.0, "bf16 out")


def test_large_fp4_rows_sample(nat):
    """8192 x 8192 x 8192 FP4 x FP4 (per-tensor, bf16 out) on the default
    kernel choice: 256 seeded rows x all columns against the oracle, exact
    accumulation, so within one bf16 ulp."""
    M = N = K = 8192
    g = torch.Generator().manual_seed(0)
    a, b = rand_fp4(M, K, g), rand_fp4(N, K, g)
    out = nat.scaled_mm(a.cuda(), b.cuda(), torch.tensor(0.01).cuda(), torch.tensor(0.02).cuda(),
                        out_dtype=torch.bfloat16, a_dtype=FP4, b_dtype=FP4)
    rows = np.sort(np.random.default_rng(0).choice(M, 256, replace=False))
    ref, S = O.scaled_mm_ref(a.numpy(), b.numpy(), 0.01, 0.02, fmt_a=O.FP4, fmt_b=O.FP4, rows=rows)
    worst = check(out[torch.from_numpy(rows).cuda()], ref, S, 0.0, "8192^3 fp4")
    assert worst <= 1.0


def test_invalid_fp4_calls(nat):
    from fp4_fp8_for_torch_mps import _lib as L
    a = torch.zeros(64, 48, dtype=torch.uint8, device="cuda")  # K = 96: not a multiple of 128
    b = torch.zeros(64, 48, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 128"):
        nat.scaled_mm(a, b, torch.tensor(1.0), torch.tensor(1.0), a_dtype=FP4, b_dtype=FP4)
    buf = torch.zeros(64 * 64 + 16, dtype=torch.uint8, device="cuda")
    a16 = buf[16:].view(64, 64)  # 16-byte but not 32-byte aligned base
    s = torch.ones(1, device="cuda")
    out = torch.empty(64, 64, device="cuda")
    rc = L.lib().fp8b200_scaled_mm(a16.data_ptr(), L.E2M1, 64, a16.data_ptr(), L.E2M1, 64, 64, 64, 128,
                                   s.data_ptr(), 0, s.data_ptr(), 0, None, 0, None, out.data_ptr(), L.F32, 64,
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == -1 and b"32-byte" in L.lib().fp8b200_last_error()


@pytest.mark.parametrize("M,N,K", [(256, 480, 256), (512, 1000, 1024), (300, 2048, 4096), (1024, 8192, 2048)])
def test_block_scaled_path_matches_byte_padded_path(nat, M, N, K):
    """FP4 x FP4 on the 256x480 CTA-pair kernel runs as tcgen05 kind::mxf4 (packed operands,
    unit block scales); the 256x256 kernel (path 2) as kind::f8f6f4 on byte-padded operands.
    Both accumulate exactly, so their outputs are identical, and equal the oracle within
    one output ulp."""
    from fp4_fp8_for_torch_mps import _lib as L
    g = torch.Generator().manual_seed(M + N + K)
    a, b = rand_fp4(M, K, g), rand_fp4(N, K, g)
    sa = torch.rand(M, 1, generator=g) * 0.5 + 0.01
    sb = torch.tensor(0.125)
    outs = {}
    try:
        for path in (4, 2):
            L.check(L.lib().fp8b200_gemm_set_path(path), "gemm path")
            outs[path] = nat.scaled_mm(a.cuda(), b.cuda(), sa.cuda(), sb.cuda(), out_dtype=torch.float32,
                                       a_dtype=FP4, b_dtype=FP4)
            torch.cuda.synchronize()
    finally:
        L.check(L.lib().fp8b200_gemm_set_path(0), "gemm path")
    assert torch.equal(outs[4], outs[2])
    rows = np.arange(0, M, max(1, M // 64))
    ref, S = O.scaled_mm_ref(a.numpy(), b.numpy(), sa.numpy().reshape(-1), 0.125, fmt_a=O.FP4, fmt_b=O.FP4,
                             rows=rows)
    check(outs[4][torch.from_numpy(rows).cuda()], ref, S, 0.0, f"mxf4 {M}x{N}x{K}")

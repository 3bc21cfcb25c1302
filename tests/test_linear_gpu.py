"""Device parity of the float8-weight linear with dequant-on-load
(fp8b200_linear_fp8w, fp8_mps::fp8_linear) against a float64 reference
x @ (decode(w) * s)^T + bias.

Tolerance (the GEMM tests' bound): |out - r| <= ulp_out(|r|) + 2^-20 * S with
S = sum_k |x_k| |w_k s| (+ |bias| 2^-4 when a bias is added): one output ulp
plus the float32 accumulation bound. The products x_k * w_k are exact (the
weights enter the tensor cores unrounded), so this is the same bar as the
fp8 x fp8 GEMM.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

E4, E5 = torch.float8_e4m3fn, torch.float8_e5m2
FMT = {E4: O.E4M3, E5: O.E5M2}
ACC_TOL = 2.0 ** -20


@pytest.fixture(scope="module")
def nat(device):
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


def ulp(x, dtype):
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    u = 2.0 ** (np.floor(np.log2(ax)) - mant)
    if dtype == torch.float16:
        u = np.maximum(u, 2.0 ** -24)
    return u


def reference(x, w, scale, bias=None):
    xv = x.float().cpu().double().numpy()
    wv = O.fp8_table_f64(FMT[w.dtype])[w.view(torch.uint8).cpu().numpy()]
    sv = scale.float().cpu().double().numpy().reshape(1, -1)
    W = wv * sv.reshape(-1, 1) if sv.size > 1 else wv * sv.item()
    r = xv @ W.T
    S = np.abs(xv) @ np.abs(W).T
    if bias is not None:
        bv = bias.float().cpu().double().numpy().reshape(1, -1)
        r = r + bv
        S = S + np.abs(bv) * 2.0 ** -4
    return r, S


def check(out, r, S, what):
    o = out.float().cpu().double().numpy()
    tol = ulp(r, out.dtype) + ACC_TOL * S
    bad = np.abs(o - r) > tol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"


def rand_w(shape, dtype, gen):
    w = (torch.randn(*shape, generator=gen) * 30).clamp(-400, 400).to(dtype)
    return w


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (17, 300, 200), (128, 256, 64), (129, 512, 72),
                                   (300, 528, 1040), (1000, 1008, 2000), (64, 4096, 4096)])
def test_shapes(nat, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), E4, g)
    s = torch.tensor(0.0123)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    r, S = reference(x, w, s)
    check(out, r, S, f"{M}x{N}x{K}")


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bias_dt", [None, torch.float32, torch.bfloat16])
def test_dtypes_scales_bias(nat, xdt, wdt, odt, bias_dt):
    M, N, K = 200, 320, 384
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(M, K, generator=g) * 2).to(xdt)
    w = rand_w((N, K), wdt, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3          # per output channel
    bias = None if bias_dt is None else (torch.randn(N, generator=g) * 5).to(bias_dt)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), None if bias is None else bias.cuda(), out_dtype=odt)
    assert out.dtype == odt
    r, S = reference(x, w, s, bias)
    check(out, r, S, f"{xdt} {wdt} {odt} bias={bias_dt}")


@pytest.mark.parametrize("wdt", [E4, E5])
def test_every_finite_weight_code(nat, wdt):
    """Each of the finite codes appears in every column position of K: the
    conversion inside shared memory is exact for all of them (a one-hot x
    row picks out single weight values)."""
    codes = torch.arange(256, dtype=torch.uint8)
    vals = codes.view(wdt).float()
    finite = codes[torch.isfinite(vals)]
    K = 128
    w = finite.repeat(256 * K // finite.numel() + 1)[: 256 * K].reshape(256, K).view(wdt)
    x = torch.eye(K, dtype=torch.bfloat16)                 # row i selects column i of every weight row
    out = nat.fp8_linear(x.cuda(), w.cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32)
    want = w.float().T                                     # (K, 256): exact values
    assert torch.equal(out.cpu(), want)


def test_nan_weight_propagates(nat):
    x = torch.ones(4, 64, dtype=torch.bfloat16)
    w = torch.zeros(256, 64, dtype=torch.uint8)
    w[3, 5] = 0x7F                                          # e4m3 NaN
    out = nat.fp8_linear(x.cuda(), w.view(E4).cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32).cpu()
    assert torch.isnan(out[:, 3]).all() and not torch.isnan(out[:, [0, 1, 2, 4]]).any()


def test_leading_dims_custom_op_and_unaligned(nat):
    """(..., K) activations, the fp8_mps::fp8_linear op, and K not a multiple
    of 8 (the launcher pads the row pitch)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 5, 100, generator=g).to(torch.bfloat16)
    w = rand_w((64, 100), E4, g)
    s = torch.tensor(0.02)
    out = torch.ops.fp8_mps.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    assert out.shape == (2, 5, 64)
    r, S = reference(x.reshape(-1, 100), w, s)
    check(out.reshape(-1, 64), r, S, "leading dims")


def test_rejects_bad_input(nat):
    x = torch.zeros(4, 32, device="cuda")
    w = torch.zeros(8, 32, dtype=E4, device="cuda")
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        nat.fp8_linear(x, w, torch.tensor(1.0))
    with pytest.raises(RuntimeError, match="weight_scale"):
        nat.fp8_linear(x.bfloat16(), w, torch.ones(3))


# ---------------------------------------------------------------- 16 < M <= 256 with many output channels
@pytest.mark.parametrize("M,N,K", [(17, 14336, 256), (100, 9600, 384), (256, 10240, 128), (200, 14336, 1040)])
@pytest.mark.parametrize("wdt", [E4, E5])
def test_mid_rows_wide_output(nat, M, N, K, wdt):
    """16 < M <= 256 and N wide enough that the CTA-pair dequant-on-load kernel's column
    tiles fill half the GPU: that kernel serves these calls; per-channel scales, bias."""
    g = torch.Generator().manual_seed(M * 3 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), wdt, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), bias.cuda())
    r, S = reference(x, w, s, bias.float())
    check(out, r, S, f"{M}x{N}x{K} {wdt}")


# ---------------------------------------------------------------- many rows: decode once + 16-bit GEMM
@pytest.mark.parametrize("M,N,K,once", [(1024, 6144, 256, True), (2048, 4864, 512, True), (1500, 5000, 333, True),
                                        (300, 14336, 192, True), (1024, 512, 256, False), (1100, 100, 64, False),
                                        (1500, 776, 333, False)])
@pytest.mark.parametrize("wdt", [E4, E5])
def test_many_rows_path(nat, M, N, K, once, wdt):
    """More than 256 rows: weights decoded once and the 16-bit CTA-pair GEMM when the
    dequant-on-load kernel's 256 x 256 tiles outnumber the CTA pairs, else that kernel
    (N = 100: output rows not 16-byte aligned, dequant-on-load kernel at any size)."""
    assert nat.linear_decodes_once(M, N, torch.device("cuda")) == once
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), wdt, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = torch.randn(N, generator=g)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), bias.cuda())
    r, S = reference(x, w, s, bias)
    check(out, r, S, f"{M}x{N}x{K} {wdt}")


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(256, 512, 64), (300, 520, 200), (1024, 1536, 1024)])
def test_gemm_16bit(nat, dt, odt, M, N, K):
    g = torch.Generator().manual_seed(M * N + K)
    a = torch.randn(M, K, generator=g).to(dt)
    b = torch.randn(N, K, generator=g).to(dt)
    s = torch.rand(N, generator=g) + 0.5
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    out = nat.gemm_16bit(a.cuda(), b.cuda(), s.cuda(), bias.cuda(), out_dtype=odt)
    av, bv = a.double().numpy(), b.double().numpy()
    sv, bb = s.double().numpy(), bias.float().double().numpy()
    r = (av @ bv.T) * sv[None, :] + bb[None, :]
    S = (np.abs(av) @ np.abs(bv).T) * sv[None, :] + np.abs(bb)[None, :] * 2.0 ** -4
    check(out, r, S, f"gemm_16bit {dt} {odt} {M}x{N}x{K}")


# ---------------------------------------------------------------- M <= 16, K % 128 == 0: register-converted path
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 14336, 4096), (3, 4096, 14336), (5, 300, 256),
                                   (16, 64, 128), (8, 1000, 1408), (2, 65, 2048)])
def test_few_rows_shapes(nat, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), E4, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    r, S = reference(x, w, s)
    check(out, r, S, f"few rows {M}x{N}x{K}")


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bias_dt", [None, torch.float16])
def test_few_rows_dtypes_scales_bias(nat, xdt, wdt, odt, bias_dt):
    M, N, K = 7, 200, 384
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(M, K, generator=g) * 2).to(xdt)
    w = rand_w((N, K), wdt, g)
    s = torch.tensor(0.0071) if bias_dt is None else torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = None if bias_dt is None else (torch.randn(N, generator=g) * 5).to(bias_dt)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), None if bias is None else bias.cuda(), out_dtype=odt)
    r, S = reference(x, w, s, bias)
    check(out, r, S, f"few rows {xdt} {wdt} {odt} bias={bias_dt}")


@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
def test_few_rows_every_finite_weight_code(nat, wdt, xdt):
    """Every finite code in every k position, picked out exactly by one-hot x
    rows, 16 rows at a time: the in-register conversion is exact."""
    codes = torch.arange(256, dtype=torch.uint8)
    finite = codes[torch.isfinite(codes.view(wdt).float())]
    K = 128
    w = finite.repeat(256 * K // finite.numel() + 1)[: 256 * K].reshape(256, K).view(wdt)
    eye = torch.eye(K, dtype=xdt)
    for k0 in range(0, K, 16):
        out = nat.fp8_linear(eye[k0:k0 + 16].cuda(), w.cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32)
        assert torch.equal(out.cpu(), w.float().T[k0:k0 + 16]), k0


def test_few_rows_nan_weight_propagates(nat):
    x = torch.ones(4, 128, dtype=torch.bfloat16)
    w = torch.zeros(256, 128, dtype=torch.uint8)
    w[3, 5] = 0x7F                                          # e4m3 NaN
    out = nat.fp8_linear(x.cuda(), w.view(E4).cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32).cpu()
    assert torch.isnan(out[:, 3]).all() and not torch.isnan(out[:, [0, 1, 2, 4]]).any()


def test_few_rows_matches_tensor_core_path(nat):
    """The register-converted path and the tcgen05 small-M path (forced) agree
    within the tolerance on the same inputs."""
    from fp4_fp8_for_torch_mps import _lib as L
    g = torch.Generator().manual_seed(21)
    x = torch.randn(9, 2048, generator=g).to(torch.bfloat16)
    w = rand_w((1536, 2048), E4, g)
    s = torch.rand(1536, generator=g) * 0.01 + 1e-3
    r, S = reference(x, w, s)
    a = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    L.lib().fp8b200_gemm_set_path(3)
    try:
        b = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    finally:
        L.lib().fp8b200_gemm_set_path(0)
    check(a, r, S, "register-converted")
    check(b, r, S, "tcgen05 small-M")


def test_few_rows_repeated_calls_are_stable(nat):
    """Back-to-back calls on the same inputs (a stage of the weight ring is
    refilled while other warps may still be reading the previous tile) give
    identical outputs within the tolerance, every time."""
    g = torch.Generator().manual_seed(5)
    M, N, K = 16, 14336, 4096
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), E4, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    r, S = reference(x, w, s)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    outs = [nat.fp8_linear(xd, wd, sd) for _ in range(12)]
    for i, o in enumerate(outs):
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16)), i
    check(outs[0], r, S, "repeated few-row calls")


def test_few_rows_bounded_wait_times_out_and_context_survives(nat):
    """The warp-level kernel's consumers wait for weight tiles that never
    arrive (the test hook stops the producer before its first load): they give
    up after 50 ms with the status word set, the call returns, and the next
    call on the same context is correct."""
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(4, 1024, generator=g).to(torch.bfloat16).cuda()
    w = rand_w((512, 1024), E4, g).cuda()
    s = torch.tensor(0.01).cuda()
    L.gemm_status(reset=True)
    try:
        lib.fp8b200_debug_gemm(1, 50_000_000)
        nat.fp8_linear(x, w, s)
        status = L.gemm_status(reset=True)
    finally:
        lib.fp8b200_debug_gemm(0, 0)
    assert status & 0x80000000, hex(status)
    out = nat.fp8_linear(x, w, s)
    torch.cuda.synchronize()
    assert L.gemm_status() == 0
    r, S = reference(x.cpu(), w.cpu(), s.cpu())
    check(out, r, S, "after timeout")


@pytest.mark.parametrize("M,N,K", [(16, 9600, 256), (9, 11008, 512), (1, 14336, 128), (5, 9473, 384)])
@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
def test_few_rows_112_channel_ctas(nat, M, N, K, wdt, xdt):
    """Shapes whose 64-channel CTAs would fill the SMs unevenly (more CTAs than SMs, fewer than two per
    SM) run 112-channel CTAs, one per SM: per-channel scales, bias, a ragged last CTA (N = 9473)."""
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).to(xdt)
    w = rand_w((N, K), wdt, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = torch.randn(N, generator=g).to(torch.bfloat16)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), bias.cuda(), out_dtype=torch.float32)
    r, S = reference(x, w, s, bias.float())
    check(out, r, S, f"112-channel CTAs {M}x{N}x{K} {wdt} {xdt}")


@pytest.mark.parametrize("wdt", [E4, E5])
def test_few_rows_112_channel_ctas_every_finite_code(nat, wdt):
    """Every finite code in every k position of the 112-row weight tiles, picked out by one-hot rows."""
    codes = torch.arange(256, dtype=torch.uint8)
    finite = codes[torch.isfinite(codes.view(wdt).float())]
    N, K = 9600, 128
    w = finite.repeat(N * K // finite.numel() + 1)[: N * K].reshape(N, K).view(wdt)
    eye = torch.eye(K, dtype=torch.bfloat16)
    for k0 in range(0, K, 16):
        out = nat.fp8_linear(eye[k0:k0 + 16].cuda(), w.cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32)
        assert torch.equal(out.cpu(), w.float().T[k0:k0 + 16]), k0


# ---------------------------------------------------------------- 16 < M <= 64, K % 128 == 0: four or eight 8-row x tiles
@pytest.mark.parametrize("M,N,K", [(17, 1000, 1408), (32, 14336, 4096), (33, 4096, 256), (48, 300, 256),
                                   (64, 4096, 4096), (64, 9600, 512), (40, 65, 2048), (24, 4096, 14336)])
def test_few_rows_up_to_64_shapes(nat, M, N, K):
    g = torch.Generator().manual_seed(M * 5 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), E4, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    r, S = reference(x, w, s)
    check(out, r, S, f"up to 64 rows {M}x{N}x{K}")


@pytest.mark.parametrize("M", [29, 64])
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("odt", [torch.float32, torch.bfloat16])
def test_few_rows_up_to_64_dtypes_scales_bias(nat, M, xdt, wdt, odt):
    N, K = 392, 640
    g = torch.Generator().manual_seed(13 + M)
    x = (torch.randn(M, K, generator=g) * 2).to(xdt)
    w = rand_w((N, K), wdt, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    bias = (torch.randn(N, generator=g) * 5).to(torch.float16)
    out = nat.fp8_linear(x.cuda(), w.cuda(), s.cuda(), bias.cuda(), out_dtype=odt)
    r, S = reference(x, w, s, bias)
    check(out, r, S, f"up to 64 rows {M} {xdt} {wdt} {odt}")


@pytest.mark.parametrize("wdt", [E4, E5])
@pytest.mark.parametrize("rows", [32, 64])
def test_few_rows_up_to_64_every_finite_weight_code(nat, wdt, rows):
    """Every finite code in every k position, picked out by `rows` one-hot x rows at a time."""
    codes = torch.arange(256, dtype=torch.uint8)
    finite = codes[torch.isfinite(codes.view(wdt).float())]
    K = 128
    w = finite.repeat(256 * K // finite.numel() + 1)[: 256 * K].reshape(256, K).view(wdt)
    eye = torch.eye(K, dtype=torch.bfloat16)
    for k0 in range(0, K, rows):
        out = nat.fp8_linear(eye[k0:k0 + rows].cuda(), w.cuda(), torch.tensor(1.0).cuda(), out_dtype=torch.float32)
        assert torch.equal(out.cpu(), w.float().T[k0:k0 + rows]), k0


def test_few_rows_64_repeated_calls_are_stable(nat):
    g = torch.Generator().manual_seed(8)
    M, N, K = 64, 14336, 4096
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = rand_w((N, K), E4, g)
    s = torch.rand(N, generator=g) * 0.01 + 1e-3
    r, S = reference(x, w, s)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    outs = [nat.fp8_linear(xd, wd, sd) for _ in range(8)]
    for i, o in enumerate(outs):
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16)), i
    check(outs[0], r, S, "repeated 64-row calls")

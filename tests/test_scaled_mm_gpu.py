"""Device parity of the tcgen05 FP8 GEMM (through the C ABI via the package
launcher, torch._scaled_mm and fp8_mps::scaled_mm) against the float64
dequantised oracle.

Tolerance (written once here, used by every case): for an output element
with float64 reference r and magnitude sum S = sum_k |a_k sa| |b_k sb|,

    |out - r| <= ulp_out(|r|) + 2^-20 * S

ulp_out is the spacing of the output type at |r| (bf16: 2^(e-7), f16: 2^(e-10),
f32: 2^(e-23)); the second term bounds the float32 accumulation error over K,
which also covers outputs near zero where cancellation makes ulp(r) tiny. For
bf16 this is the "within 1 bf16 ulp of an fp32-accumulated dequantised
reference" bar.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

E4, E5 = torch.float8_e4m3fn, torch.float8_e5m2
FMT = {E4: O.E4M3, E5: O.E5M2}
ACC_TOL = 2.0 ** -20


def ulp(x, dtype):
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[dtype]
    ax = np.maximum(np.abs(x), 2.0 ** -126)
    u = 2.0 ** (np.floor(np.log2(ax)) - mant)
    if dtype == torch.float16:
        u = np.maximum(u, 2.0 ** -24)
    return u


def check_close(out: torch.Tensor, ref: np.ndarray, S: np.ndarray, what=""):
    o = out.float().cpu().double().numpy()
    err = np.abs(o - ref)
    tol = ulp(ref, out.dtype) + ACC_TOL * S
    bad = err > tol
    if bad.any():
        i = np.argwhere(bad)[0]
        pytest.fail(f"{what}: {bad.sum()} of {bad.size} outside tolerance; first at {tuple(i)}: "
                    f"out {o[tuple(i)]!r} ref {ref[tuple(i)]!r} tol {tol[tuple(i)]!r}")
    return float((err / np.maximum(np.abs(ref), 1e-30)).max())


@pytest.fixture(scope="module")
def nat(device):
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


@pytest.fixture(params=[1, 2, 3, 4], ids=["single_cta", "cta_pair", "small_m", "cta_pair_wide"])
def path(request, nat):
    """Run the test on the single-CTA, the CTA-pair (256x256 and 256x512
    tiles) and the small-M kernel."""
    from fp4_fp8_for_torch_mps import _lib as L
    L.check(L.lib().fp8b200_gemm_set_path(request.param), "gemm path")
    yield request.param
    L.check(L.lib().fp8b200_gemm_set_path(0), "gemm path")


def codes(t):
    return t.view(torch.uint8).cpu().numpy()


def rand_fp8(shape, dtype, gen, scale=100.0):
    return (torch.randn(*shape, generator=gen) * scale).clamp(-440, 440).to(dtype)


# ---------------------------------------------------------------- golden cases
@pytest.mark.parametrize("case", [0, 1, 2])
def test_golden_cpu_scaled_mm_cases(nat, golden, case):
    a = torch.from_numpy(golden[f"mm{case}_a"]).view(E4)
    b = torch.from_numpy(golden[f"mm{case}_b"]).view(E4)
    sa = torch.tensor(golden[f"mm{case}_sa"][0])
    sb = torch.tensor(golden[f"mm{case}_sb"][0])
    M, K = a.shape
    N = b.shape[0]
    if K % 16 or N % 16:
        pytest.skip("shape not accepted by torch._scaled_mm on CUDA")
    out = torch._scaled_mm(a.cuda(), b.cuda().t(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), sa.item(), sb.item())
    check_close(out, ref, S, f"golden case {case}")
    cpu = (golden[f"mm{case}_bf16"].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    o = out.float().cpu().double().numpy()
    assert np.all(np.abs(o - cpu) <= 2 * ulp(cpu, torch.bfloat16) + ACC_TOL * S)


# ---------------------------------------------------------------- shapes, dtypes, epilogues
SHAPES = [(1, 16, 16), (1, 256, 512), (17, 48, 64), (64, 128, 256), (128, 256, 128),
          (129, 272, 144), (300, 528, 1040), (256, 512, 4096), (1000, 1008, 2000)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("rowwise", [False, True])
def test_shapes_bf16(nat, path, M, N, K, rowwise):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a = rand_fp8((M, K), E4, g)
    b = rand_fp8((N, K), E4, g)
    if rowwise:
        sa = torch.rand(M, 1, generator=g) * 0.01 + 1e-3
        sb = torch.rand(1, N, generator=g) * 0.01 + 1e-3
    else:
        sa, sb = torch.tensor(0.0123), torch.tensor(0.0456)
    out = torch._scaled_mm(a.cuda(), b.cuda().t(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16)
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    ref, S = O.scaled_mm_ref(codes(a), codes(b), sa.numpy().reshape(-1), sb.numpy().reshape(-1))
    check_close(out, ref, S, f"{M}x{N}x{K} rowwise={rowwise}")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fmts", [(E4, E4), (E4, E5), (E5, E4)])
@pytest.mark.parametrize("bias_dtype", [None, torch.float32, torch.bfloat16])
def test_dtypes_and_bias(nat, path, out_dtype, fmts, bias_dtype):
    M, N, K = 200, 320, 384
    g = torch.Generator().manual_seed(11)
    a = rand_fp8((M, K), fmts[0], g, 20.0)
    b = rand_fp8((N, K), fmts[1], g, 20.0)
    sa, sb = torch.tensor(0.05), torch.tensor(0.02)
    bias = None if bias_dtype is None else (torch.randn(N, generator=g) * 10).to(bias_dtype)
    out = torch._scaled_mm(a.cuda(), b.cuda().t(), sa.cuda(), sb.cuda(),
                           bias=None if bias is None else bias.cuda(), out_dtype=out_dtype)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), sa.item(), sb.item(), FMT[fmts[0]], FMT[fmts[1]],
                             bias=None if bias is None else bias.float().numpy())
    if bias is not None:
        S = S + np.abs(bias.float().numpy()).reshape(1, -1) * 2.0 ** -4
    check_close(out, ref, S, f"{out_dtype} {fmts} bias={bias_dtype}")


def test_fp8_output_and_scale_result(nat, path):
    """out_dtype=None returns self.dtype (fp8), as torch._scaled_mm does."""
    M, N, K = 128, 256, 256
    g = torch.Generator().manual_seed(5)
    a = rand_fp8((M, K), E4, g, 10.0)
    b = rand_fp8((N, K), E4, g, 10.0)
    sa, sb, sr = torch.tensor(0.01), torch.tensor(0.01), torch.tensor(0.5)
    out = torch._scaled_mm(a.cuda(), b.cuda().t(), sa.cuda(), sb.cuda(), scale_result=sr.cuda())
    assert out.dtype == E4
    ref, S = O.scaled_mm_ref(codes(a), codes(b), sa.item(), sb.item())
    ref = ref * 0.5
    dec = out.float().cpu().double().numpy()
    e4_ulp = np.maximum(2.0 ** (np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -6))) - 3), 2.0 ** -9)
    ok = np.isnan(dec) & (np.abs(ref) > 448) | (np.abs(dec - ref) <= e4_ulp * 0.5 + ACC_TOL * S)
    assert ok.all(), (dec[~ok][:5], ref[~ok][:5])


def test_strided_operands_and_output(nat, path):
    """Row strides larger than K (views into wider buffers) on both operands."""
    M, N, K = 256, 256, 256
    g = torch.Generator().manual_seed(9)
    abuf = rand_fp8((M, K + 64), E4, g)
    bbuf = rand_fp8((N, K + 128), E4, g)
    a, b = abuf.cuda()[:, 16:16 + K], bbuf.cuda()[:, 32:32 + K]
    out = nat.scaled_mm(a, b, torch.tensor(0.01), torch.tensor(0.02), out_dtype=torch.bfloat16)
    ref, S = O.scaled_mm_ref(codes(abuf)[:, 16:16 + K], codes(bbuf)[:, 32:32 + K], 0.01, 0.02)
    check_close(out, ref, S, "strided")


@pytest.mark.parametrize("force", [0, 4], ids=["by_shape", "wide_requested"])
@pytest.mark.parametrize("case", ["fp8_out_n1000", "bf16_ldd_odd"])
def test_unaligned_output_rows(nat, force, case):
    """Output rows that are not 16-byte aligned (fp8 output with N % 16 != 0, a bf16
    output with an odd row stride) go to a kernel with plain stores even where the
    256x512 kernel (which stores through a tensor map) would be chosen by shape or
    requested."""
    from fp4_fp8_for_torch_mps import _lib as L
    M, N, K = 512, 1000, 256
    g = torch.Generator().manual_seed(21)
    a = rand_fp8((M, K), E4, g).cuda()
    b = rand_fp8((N, K), E4, g).cuda()
    sa, sb = torch.tensor(0.01), torch.tensor(0.02)
    L.check(L.lib().fp8b200_gemm_set_path(force), "gemm path")
    try:
        if case == "fp8_out_n1000":
            out = nat.scaled_mm(a, b, sa, sb, out_dtype=torch.float32)
            o8 = nat.scaled_mm(a, b, sa, sb, out_dtype=torch.float8_e4m3fn, scale_result=torch.tensor([1 / 16.0]))
            torch.cuda.synchronize()
            ref8 = (out.cpu() / 16.0).to(torch.float8_e4m3fn)
            diff = (o8.cpu().float() - ref8.float()).abs()
            # one e4m3 step at most (the f32 output and the fp8 epilogue round independently)
            assert bool((diff <= ref8.float().abs() * 0.125 + 2.0 ** -9).all())
        else:
            buf = torch.empty(M, N + 1, dtype=torch.bfloat16, device="cuda")
            out = nat.scaled_mm(a, b, sa, sb, out_dtype=torch.bfloat16, out=buf[:, :N])
            torch.cuda.synchronize()
        ref, S = O.scaled_mm_ref(codes(a), codes(b), 0.01, 0.02)
        check_close(out, ref, S, f"unaligned output ({case}, path {force})")
    finally:
        L.check(L.lib().fp8b200_gemm_set_path(0), "gemm path")


def test_invalid_calls_raise(nat):
    a = torch.zeros(32, 64, dtype=torch.uint8, device="cuda").view(E4)
    b = torch.zeros(48, 64, dtype=torch.uint8, device="cuda").view(E4)
    s = torch.tensor(1.0, device="cuda")
    with pytest.raises(RuntimeError):
        torch._scaled_mm(a, b, s, s)                       # mat2 not column-major
    with pytest.raises(RuntimeError):
        torch._scaled_mm(a.view(E5), b.view(E5).t(), s, s)  # e5m2 x e5m2
    with pytest.raises(RuntimeError):
        torch._scaled_mm(a.view(torch.float4_e2m1fn_x2), b.view(torch.float4_e2m1fn_x2).t(), s, s)  # fp4
    with pytest.raises(RuntimeError):
        torch._scaled_mm(a, b.t(), torch.ones(32, 2, device="cuda"), s)  # blockwise-like scales
    with pytest.raises(RuntimeError):
        torch._scaled_mm(a[:, :40], b[:, :40].t(), s, s)  # K not multiple of 16


# ---------------------------------------------------------------- reference op surface
def test_reference_custom_ops_accuracy(nat):
    """tests/test_fp8_metal.py:52-93 / test_integration.py:125-138 of the
    reference (rel RMSE < 15%), plus the oracle bound."""
    for M, K, N in ((64, 256, 128), (1, 512, 256), (16, 32, 24), (32, 64, 48)):
        g = torch.Generator().manual_seed(M + K + N)
        A = torch.randn(M, K, generator=g)
        B = torch.randn(N, K, generator=g)
        Aq, As = torch.ops.fp8_mps.quantize(A.cuda())
        Bq, Bs = torch.ops.fp8_mps.quantize(B.cuda())
        if K % 16:
            continue
        r = torch.ops.fp8_mps.scaled_mm(Aq, Bq, As, Bs).cpu()
        assert r.shape == (M, N) and r.dtype == torch.float32
        ref = A @ B.T
        rel = torch.sqrt(((r - ref) ** 2).mean()) / torch.sqrt((ref ** 2).mean())
        assert rel < 0.15
        oref, S = O.scaled_mm_ref(Aq.cpu().numpy(), Bq.cpu().numpy(), As.item(), Bs.item())
        check_close(r, oref, S, f"custom op {M}x{K}x{N}")


# ---------------------------------------------------------------- full-size workloads
def ulp_stats(out, ref, S):
    """Error in bf16 ulps of the float64 reference: the largest over the
    outputs whose float32 accumulation bound (2^-20 S) is below half an ulp
    (no cancellation), and the fraction of all outputs above one ulp."""
    o = out.float().cpu().double().numpy()
    u = ulp(ref, torch.bfloat16)
    e = np.abs(o - ref) / u
    well = ACC_TOL * S <= 0.5 * u
    return float(e[well].max()), float(well.mean()), float((e > 1.0).mean())


@pytest.mark.parametrize("size", [4096, 8192, 16384])
def test_per_tensor_workload(nat, size):
    """Default kernel choice (the CTA-pair kernels at these sizes), 256 seeded
    rows x all columns. Beyond the tolerance: every well-conditioned output is
    within one bf16 ulp of the float64 reference, and at most 1e-3 of all
    outputs (those near zero, where the float32 sum's own rounding exceeds an
    output ulp) are above one ulp."""
    from fp4_fp8_for_torch_mps.workloads import scaled_mm_operands
    aq, bq, sa, sb = scaled_mm_operands(size, size, size)
    out = torch._scaled_mm(aq.cuda(), bq.cuda().t(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16)
    rows = np.sort(np.random.default_rng(size).choice(size, 256, replace=False))
    ref, S = O.scaled_mm_ref(codes(aq), codes(bq), sa.item(), sb.item(), rows=rows)
    sel = out[torch.from_numpy(rows).cuda()]
    check_close(sel, ref, S, f"{size}^3 per-tensor")
    worst_well, frac_well, over = ulp_stats(sel, ref, S)
    assert frac_well > 0.9 and worst_well <= 1.0 and over <= 1e-3, (worst_well, frac_well, over)


@pytest.mark.parametrize("shape", [(16384, 4096, 4096), (16384, 14336, 4096), (16384, 4096, 14336)])
def test_rowwise_workload(nat, shape):
    from fp4_fp8_for_torch_mps.workloads import rowwise_operands
    M, N, K = shape
    aq, wq, sa, sw = rowwise_operands(M, N, K)
    out = torch._scaled_mm(aq.cuda(), wq.cuda().t(), sa.cuda(), sw.cuda(), out_dtype=torch.bfloat16)
    rows = np.sort(np.random.default_rng(N).choice(M, 256, replace=False))
    ref, S = O.scaled_mm_ref(codes(aq), codes(wq), sa.numpy().reshape(-1), sw.numpy().reshape(-1), rows=rows)
    sel = out[torch.from_numpy(rows).cuda()]
    check_close(sel, ref, S, f"rowwise {shape}")
    worst_well, frac_well, over = ulp_stats(sel, ref, S)
    assert frac_well > 0.9 and worst_well <= 1.0 and over <= 1e-3, (worst_well, frac_well, over)


# ---------------------------------------------------------------- small M (split-K clusters)
@pytest.mark.parametrize("M", [1, 2, 16, 33, 64, 200, 256])
@pytest.mark.parametrize("N,K", [(1024, 8192), (4096, 4096), (6144, 4096), (4096, 14336)])
def test_small_m_split_k(nat, M, N, K):
    """Decode-sized activations against Llama-shaped weights on the default
    (by shape) path: few column tiles, so K is split over clusters of up to 8
    CTAs and reduced through distributed shared memory. Rowwise scales."""
    g = torch.Generator().manual_seed(M * 13 + N + K)
    a = rand_fp8((M, K), E4, g, 30.0)
    b = rand_fp8((N, K), E4, g, 30.0)
    sa = torch.rand(M, 1, generator=g) * 0.01 + 1e-3
    sb = torch.rand(1, N, generator=g) * 0.01 + 1e-3
    out = torch._scaled_mm(a.cuda(), b.cuda().t(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), sa.numpy().reshape(-1), sb.numpy().reshape(-1))
    check_close(out, ref, S, f"{M}x{N}x{K}")


def test_small_m_matches_other_kernels_closely(nat):
    """The small-M kernel (split-K, DSMEM reduction) and the single-CTA kernel
    agree to within the accumulation-order tolerance on the same inputs."""
    from fp4_fp8_for_torch_mps import _lib as L
    g = torch.Generator().manual_seed(77)
    a = rand_fp8((48, 8192), E4, g, 30.0).cuda()
    b = rand_fp8((2048, 8192), E4, g, 30.0).cuda()
    s = torch.tensor(0.003)
    outs = []
    for path_id in (3, 1):
        L.check(L.lib().fp8b200_gemm_set_path(path_id), "gemm path")
        try:
            outs.append(nat.scaled_mm(a, b, s, s, out_dtype=torch.float32))
        finally:
            L.lib().fp8b200_gemm_set_path(0)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), 0.003, 0.003)
    d = (outs[0] - outs[1]).abs().cpu().double().numpy()
    assert np.all(d <= 2 * ACC_TOL * S + 2 * ulp(ref, torch.float32))


# ---------------------------------------------------------------- failure detection
def test_bounded_wait_times_out_and_context_survives(nat, path):
    """A wait that nothing will satisfy (the producer is told never to fill the
    first stage) gives up after 50 ms with a status word; the next GEMM on the
    same context is correct."""
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(1)
    a = rand_fp8((256, 256), E4, g).cuda()
    b = rand_fp8((256, 256), E4, g).cuda()
    s = torch.tensor(0.01)
    L.gemm_status(reset=True)
    try:
        lib.fp8b200_debug_gemm(1, 50_000_000)
        nat.scaled_mm(a, b, s, s, out_dtype=torch.bfloat16)
        status = L.gemm_status(reset=True)
    finally:
        lib.fp8b200_debug_gemm(0, 0)
    assert status & 0x80000000, hex(status)
    out = nat.scaled_mm(a, b, s, s, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert L.gemm_status() == 0
    ref, S = O.scaled_mm_ref(codes(a), codes(b), 0.01, 0.01)
    check_close(out, ref, S, "after timeout")


def test_timeout_does_not_leak_into_later_launches(nat, path):
    """A launch that timed out leaves its record in the status word, but the
    next launches, run without a reset, are complete and correct: the word is
    scoped to the launch that wrote it. The record stays readable until a
    reset."""
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(2)
    a = rand_fp8((300, 512), E4, g).cuda()
    b = rand_fp8((272, 512), E4, g).cuda()
    s = torch.tensor(0.02)
    L.gemm_status(reset=True)
    try:
        lib.fp8b200_debug_gemm(1, 50_000_000)
        nat.scaled_mm(a, b, s, s, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
    finally:
        lib.fp8b200_debug_gemm(0, 0)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), 0.02, 0.02)
    for _ in range(3):
        out = nat.scaled_mm(a, b, s, s, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        check_close(out, ref, S, "launch after an unread timeout")
    status = L.gemm_status(reset=True)
    assert status & 0x80000000, hex(status)
    assert L.gemm_status() == 0


def test_debug_hooks_are_per_thread(nat):
    """A test hook set on one host thread (a forced kernel path, a skipped
    load) does not reach launches from another thread."""
    import threading
    from fp4_fp8_for_torch_mps import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(4)
    a = rand_fp8((256, 256), E4, g).cuda()
    b = rand_fp8((256, 256), E4, g).cuda()
    s = torch.tensor(0.01)
    ref, S = O.scaled_mm_ref(codes(a), codes(b), 0.01, 0.01)
    L.gemm_status(reset=True)
    lib.fp8b200_debug_gemm(1, 50_000_000)
    lib.fp8b200_gemm_set_path(3)
    result = {}

    def other():
        torch.cuda.set_device(0)
        out = nat.scaled_mm(a, b, s, s, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        result["out"] = out
    try:
        t = threading.Thread(target=other)
        t.start()
        t.join()
    finally:
        lib.fp8b200_debug_gemm(0, 0)
        lib.fp8b200_gemm_set_path(0)
    assert L.gemm_status() == 0
    check_close(result["out"], ref, S, "other thread")


def test_single_cta_kernel_at_8192(nat):
    from fp4_fp8_for_torch_mps import _lib as L
    from fp4_fp8_for_torch_mps.workloads import scaled_mm_operands
    aq, bq, sa, sb = scaled_mm_operands(8192, 8192, 8192, seed=3)
    L.check(L.lib().fp8b200_gemm_set_path(1), "gemm path")
    try:
        out = torch._scaled_mm(aq.cuda(), bq.cuda().t(), sa.cuda(), sb.cuda(), out_dtype=torch.bfloat16)
    finally:
        L.lib().fp8b200_gemm_set_path(0)
    rows = np.sort(np.random.default_rng(1).choice(8192, 64, replace=False))
    ref, S = O.scaled_mm_ref(codes(aq), codes(bq), sa.item(), sb.item(), rows=rows)
    check_close(out[torch.from_numpy(rows).cuda()], ref, S, "8192^3 single-CTA")

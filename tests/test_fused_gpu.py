"""Device parity of the fused SiLU-gate + per-row quantisation kernel
(fp8b200_silu_mul_quantize_rows_fp8) against the unfused path it replaces:
PyTorch's bf16 F.silu(g) * u on the same GPU, then quantize_rows_fp8.
Codes and inverse scales must be bit-identical."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

FP8 = (torch.float8_e4m3fn, torch.float8_e5m2)


@pytest.fixture(scope="module")
def nat(device):
    from fp4_fp8_for_torch_mps import fp8_mps_native
    return fp8_mps_native


def unfused(nat, gu, fmt):
    g, u = gu.chunk(2, dim=1)
    return nat.quantize_rows_fp8(F.silu(g) * u, fmt)


def assert_same(a, b):
    (qa, sa), (qb, sb) = a, b
    assert qa.shape == qb.shape and sa.shape == sb.shape
    assert torch.equal(qa.view(torch.uint8), qb.view(torch.uint8))
    assert torch.equal(sa.view(torch.int32), sb.view(torch.int32))


@pytest.mark.parametrize("fmt", FP8)
@pytest.mark.parametrize("rows,f", [(0, 64), (1, 1), (3, 7), (5, 8), (17, 1000), (257, 14336), (2, 24577),
                                    (3, 38912), (2, 38920), (1000, 4096), (7, 2048 * 3 + 8), (600, 14336)])
def test_matches_unfused(nat, fmt, rows, f):
    g = torch.Generator(device="cuda").manual_seed(rows * 131 + f)
    gu = (torch.randn(rows, 2 * f, generator=g, device="cuda") * 3).to(torch.bfloat16)
    assert_same(nat.silu_mul_quantize_rows_fp8(gu, fmt), unfused(nat, gu, fmt))


@pytest.mark.parametrize("fmt", FP8)
def test_every_bf16_gate_value(nat, fmt):
    """All 65536 bf16 patterns as g (NaNs, infs, denormals included) in one
    row of F = 65536 (128 KiB of shared memory), against three u rows."""
    g = torch.arange(65536, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16)
    for u in (torch.ones_like(g), -torch.full_like(g, 0.75),
              torch.randn(65536, generator=torch.Generator(device="cuda").manual_seed(1),
                          device="cuda").to(torch.bfloat16)):
        gu = torch.cat([g, u])[None]
        assert_same(nat.silu_mul_quantize_rows_fp8(gu, fmt), unfused(nat, gu, fmt))


@pytest.mark.parametrize("fmt", FP8)
def test_every_bf16_gate_value_in_short_rows(nat, fmt):
    """All 65536 bf16 patterns as g in 4 rows of F = 16384 (vectorised
    path), against random u."""
    g = torch.arange(65536, dtype=torch.int32, device="cuda").to(torch.int16).view(torch.bfloat16).reshape(4, -1)
    u = torch.randn(4, 16384, generator=torch.Generator(device="cuda").manual_seed(5), device="cuda").to(torch.bfloat16)
    gu = torch.cat([g, u], dim=1)
    assert_same(nat.silu_mul_quantize_rows_fp8(gu, fmt), unfused(nat, gu, fmt))


def test_row_lengths_up_and_down(nat):
    """Alternating large and small rows: every launch still gets the shared
    memory it needs (the per-kernel limit only rises)."""
    gen = torch.Generator(device="cuda").manual_seed(6)
    for f in (24576, 1000, 24576, 64, 38912, 8, 24576):
        gu = (torch.randn(9, 2 * f, generator=gen, device="cuda") * 2).to(torch.bfloat16)
        assert_same(nat.silu_mul_quantize_rows_fp8(gu), unfused(nat, gu, torch.float8_e4m3fn))


@pytest.mark.parametrize("fmt", FP8)
def test_special_rows(nat, fmt):
    """Rows that are all zero (scale 1), hold a NaN or an inf (amax NaN/inf),
    or have one large value among tiny ones."""
    f = 40
    gu = torch.randn(6, 2 * f, generator=torch.Generator(device="cuda").manual_seed(2),
                     device="cuda").to(torch.bfloat16)
    gu[0] = 0
    gu[1, 3] = float("nan")
    gu[2, f + 5] = float("inf")
    gu[3, 7] = float("-inf")
    gu[4] *= 1e-30
    gu[4, 9], gu[4, f + 9] = 30.0, 1000.0
    gu[5, :f] = 80.0          # silu saturates to g
    gu[5, 2], gu[5, f + 2] = float("inf"), 0.0     # inf * 0 -> NaN
    gu[5, 3], gu[5, f + 3] = float("-inf"), 2.0    # silu(-inf) is NaN
    assert_same(nat.silu_mul_quantize_rows_fp8(gu, fmt), unfused(nat, gu, fmt))


def test_strided_rows(nat):
    """A row stride wider than 2F (a column slice of a wider projection) and
    an unaligned base (odd element offset) takes the scalar path."""
    base = (torch.randn(33, 304, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
            ).to(torch.bfloat16)
    for off in (0, 1, 8):
        gu = base[:, off:off + 256]
        assert gu.stride(0) == 304
        assert_same(nat.silu_mul_quantize_rows_fp8(gu), unfused(nat, gu.contiguous(), torch.float8_e4m3fn))


def test_rejects_bad_input(nat):
    x = torch.zeros(4, 6, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="bfloat16"):
        nat.silu_mul_quantize_rows_fp8(x)
    with pytest.raises(RuntimeError, match="bfloat16"):
        nat.silu_mul_quantize_rows_fp8(torch.zeros(4, 5, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError, match="row limit"):
        nat.silu_mul_quantize_rows_fp8(torch.zeros(1, 2 * 102401, dtype=torch.bfloat16, device="cuda"))


def test_llama_mlp_fused_equals_unfused(device):
    """One Llama-shaped layer gives bit-identical hidden states with the
    fused and the unfused MLP activation."""
    from fp4_fp8_for_torch_mps import workloads as W
    stack = W.Fp8LlamaStack("cuda", layers=1, seed=0)
    x = W.llama_input(1, 256).cuda()
    out = {}
    for fused in (True, False):
        stack.layers[0].fused = fused
        out[fused] = stack.forward(x, 1, 256)
    assert torch.equal(out[True].view(torch.int16), out[False].view(torch.int16))


@pytest.mark.parametrize("tokens,seq,nq,nk,hd", [(1, 1, 1, 1, 16), (7, 3, 2, 1, 32), (4096, 2048, 32, 8, 128),
                                                 (33, 33, 4, 0, 64)])
def test_rope_matches_pytorch(nat, tokens, seq, nq, nk, hd):
    """The rotary kernel equals PyTorch's bf16 expression bit for bit (values
    spanning small, large and zero, plus NaN/inf planted)."""
    from fp4_fp8_for_torch_mps import workloads as W
    g = torch.Generator(device="cuda").manual_seed(tokens + hd)
    ld = (nq + 2 * nk) * hd
    qkv = (torch.randn(tokens, ld, generator=g, device="cuda") * 4).to(torch.bfloat16)
    qkv[0, :3] = torch.tensor([0.0, float("inf"), float("nan")])
    ang = torch.rand(seq, hd // 2, generator=g, device="cuda") * 100
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
    q, k = nat.rope_bf16(qkv, cos, sin, nq, nk, hd, seq)
    pos = torch.arange(tokens, device="cuda") % seq
    c4, s4 = cos[pos][:, None, :], sin[pos][:, None, :]
    ref_q = W._rope(qkv[:, :nq * hd].reshape(tokens, nq, hd), c4, s4)
    assert torch.equal(q.view(torch.int16), ref_q.contiguous().view(torch.int16))
    if nk:
        ref_k = W._rope(qkv[:, nq * hd:(nq + nk) * hd].reshape(tokens, nk, hd), c4, s4)
        assert torch.equal(k.view(torch.int16), ref_k.contiguous().view(torch.int16))


def test_rope_rejects_bad_input(nat):
    qkv = torch.zeros(4, 96, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        nat.rope_bf16(qkv, c, c, 2, 2, 24, 4)

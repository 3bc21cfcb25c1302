"""Seeded synthetic inputs for the benchmark workloads of this path.

Every input is generated on the CPU with torch.Generator().manual_seed(seed)
so that each GPU (and the CPU baseline) sees identical data. There is no
external dataset: the shapes and value distributions are those of the
workloads the package is measured on.

  fp8_roundtrip   4096x4096 float32, N(0,1)*64, planted edge values first
  fp4_decode      16384x8192 packed FP4 bytes, uniform, arange(256) prefix,
                  per-tensor scale 0.37
  scaled_mm       per-tensor e4m3 operands quantised from N(0,1) with
                  scale = amax/448 (M=N=K in {4096, 8192, 16384})
  scaled_mm_rowwise  rowwise e4m3: activations N(0,1) per-row, weights
                  N(0,0.02) per-column, LLM shapes
  fp4_scaled_mm   packed FP4 operands, uniform bytes, per-tensor scales
"""
from __future__ import annotations

import numpy as np
import torch

FP4_DECODE_SHAPE = (16384, 8192)
FP4_DECODE_SCALE = 0.37
FP8_ROUNDTRIP_SHAPE = (4096, 4096)
SCALED_MM_SIZES = (4096, 8192, 16384)
ROWWISE_SHAPES = ((16384, 4096, 4096), (16384, 14336, 4096), (16384, 4096, 14336))


def planted_f32_edges() -> np.ndarray:
    """Edge values as float32 bit patterns: signed zeros, NaNs (quiet,
    signalling, both signs), infs, every finite e4m3fn and e5m2 value, every
    midpoint between adjacent distinct values and its f32 neighbours, the
    overflow boundaries, the 2^-10 / 2^-17 ties and f32 denormals."""
    out = [np.array([0.0, -0.0, np.inf, -np.inf], np.float32).view(np.uint32),
           np.array([0x7FC00000, 0xFFC00000, 0x7F800001, 0xFFBFFFFF, 0x7FFFFFFF], np.uint32)]
    for dt in (torch.float8_e4m3fn, torch.float8_e5m2):
        allv = torch.arange(256, dtype=torch.uint8).view(dt).to(torch.float64)
        fin = allv[torch.isfinite(allv)]
        uniq = torch.unique(fin)
        mids = (uniq[:-1] + uniq[1:]) / 2
        for t in (fin, mids):
            out.append(t.to(torch.float32).numpy().view(np.uint32))
        m32 = mids.to(torch.float32).numpy().view(np.uint32).astype(np.int64)
        for d in (-1, 1):
            nb = m32 + np.where(m32 & 0x80000000, -d, d)
            out.append((nb & 0xFFFFFFFF).astype(np.uint32))
    edges = [448.0, 464.0, 463.99, 464.01, 479.99, 480.0, 500.0, 57344.0, 61439.0, 61440.0,
             61441.0, 65504.0, 65536.0, 2.0 ** -10, 1.5 * 2.0 ** -10, 2.0 ** -9, 2.0 ** -17,
             1.5 * 2.0 ** -17, 2.0 ** -16, 2.0 ** -6, 2.0 ** -14, 3.4e38]
    e = np.array(edges, np.float32)
    out.append(np.concatenate([e, -e]).view(np.uint32))
    out.append(np.array([1, 2, 0x007FFFFF, 0x00400000, 0x80000001, 0x807FFFFF], np.uint32))
    return np.concatenate(out).astype(np.uint32)


def fp8_roundtrip_input(seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*FP8_ROUNDTRIP_SHAPE, generator=g) * 64
    e = torch.from_numpy(planted_f32_edges().view(np.int32).copy())
    x.view(-1).view(torch.int32)[: e.numel()] = e
    return x


def fp4_decode_input(seed: int = 0, rows: int | None = None) -> torch.Tensor:
    r, c = FP4_DECODE_SHAPE
    r = r if rows is None else rows
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, 256, (r, c), dtype=torch.uint8, generator=g)
    x.view(-1)[:256] = torch.arange(256, dtype=torch.uint8)
    return x


def quantize_per_tensor(x: torch.Tensor):
    """e4m3 codes and f32 scale with scale = amax/448 (x ~= codes * scale)."""
    s = (x.abs().max() / 448.0).to(torch.float32)
    return (x / s).to(torch.float8_e4m3fn), s.reshape(())


def scaled_mm_operands(m: int, n: int, k: int, seed: int = 0):
    """Per-tensor workload: A (M,K) e4m3, B as (N,K) e4m3 rows (mat2 = B.t()),
    f32 scalar scales."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    aq, sa = quantize_per_tensor(a)
    del a
    b = torch.randn(n, k, generator=g)
    bq, sb = quantize_per_tensor(b)
    return aq, bq, sa, sb


def rowwise_operands(m: int, n: int, k: int, seed: int = 0):
    """Rowwise workload: activations N(0,1) quantised per row (scale_a (M,1)),
    weights N(0,0.02) quantised per output column (scale_b (1,N))."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    sa = (a.abs().amax(dim=1, keepdim=True) / 448.0).float()
    aq = (a / sa).to(torch.float8_e4m3fn)
    del a
    w = torch.randn(n, k, generator=g) * 0.02
    sw = (w.abs().amax(dim=1, keepdim=True) / 448.0).float()
    wq = (w / sw).to(torch.float8_e4m3fn)
    return aq, wq, sa, sw.reshape(1, n)


def fp4_gemm_operands(m: int, n: int, k: int, seed: int = 0):
    """Packed FP4 GEMM operands: A (M, K/2) and B (N, K/2) bytes uniform over
    all 256 patterns (every e2m1 code in both nibbles, like the FP4 decode
    input), per-tensor f32 scales 0.01 and 0.02."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(0, 256, (m, k // 2), dtype=torch.uint8, generator=g)
    b = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)
    return a, b, torch.tensor(0.01), torch.tensor(0.02)


# ---------------------------------------------------------------------------
# FP8 weight-only inference stack: Llama-3-8B-shaped layers with random
# weights. Every linear is torch._scaled_mm on e4m3 weights (per-tensor fp32
# scale, broadcast per output column) and per-token e4m3 activations; the
# MLP's SiLU(g) * u is fused with its per-token quantisation and the rotary
# embedding is one kernel (both bit-identical to the PyTorch expressions);
# norms and attention (SDPA) stay in bf16 PyTorch.

LLAMA = dict(hidden=4096, intermediate=14336, heads=32, kv_heads=8, head_dim=128, layers=32,
             rope_theta=500000.0, eps=1e-5)


class Fp8LlamaLayer:
    """One decoder layer. Weights are generated on `device` from a seeded
    CUDA generator (deterministic) and quantised to e4m3 per tensor."""

    def __init__(self, device, gen: torch.Generator, cfg=LLAMA):
        from . import fp8_mps_native as nat
        h, f = cfg["hidden"], cfg["intermediate"]
        kvd = cfg["kv_heads"] * cfg["head_dim"]
        self.cfg = cfg
        self.nat = nat

        def qw(n, k):
            w = torch.randn(n, k, generator=gen, device=device, dtype=torch.bfloat16) * 0.02
            q, s = nat.quantize_fp8(w)          # s = [scale, 1/scale]
            return q.view(torch.float8_e4m3fn), s[1:2].clone()

        wq, sq = qw(h, h)
        wk, sk = qw(kvd, h)
        wv, sv = qw(kvd, h)
        self.w_qkv = torch.cat([wq, wk, wv])    # (h + 2*kvd, h) rows = output features
        self.s_qkv = torch.cat([sq.expand(h), sk.expand(kvd), sv.expand(kvd)]).reshape(1, -1).contiguous()
        self.w_o, so = qw(h, h)
        self.s_o = so.expand(h).reshape(1, -1).contiguous()
        wg, sg = qw(f, h)
        wu, su = qw(f, h)
        self.w_gu = torch.cat([wg, wu])
        self.s_gu = torch.cat([sg.expand(f), su.expand(f)]).reshape(1, -1).contiguous()
        self.w_d, sd = qw(h, f)
        self.s_d = sd.expand(h).reshape(1, -1).contiguous()
        self.n1 = torch.ones(h, device=device, dtype=torch.bfloat16)
        self.n2 = torch.ones(h, device=device, dtype=torch.bfloat16)

    gemm_events = None  # set to a list to record (start, end) CUDA events around each GEMM
    fused = True        # one kernel each for rotary embedding and for SiLU(g) * u + per-token quantisation

    def linear(self, x2d, w, sw):
        return self.linear_q(*self.nat.quantize_rows_fp8(x2d), w, sw)

    def linear_q(self, xq, xs, w, sw):
        if self.gemm_events is None:
            return torch._scaled_mm(xq, w.t(), xs, sw, out_dtype=torch.bfloat16)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        y = torch._scaled_mm(xq, w.t(), xs, sw, out_dtype=torch.bfloat16)
        e1.record()
        self.gemm_events.append((e0, e1, 2.0 * xq.shape[0] * xq.shape[1] * w.shape[0]))
        return y

    def forward(self, x, cos, sin, batch, seq):
        import torch.nn.functional as F
        c = self.cfg
        h, hd, nh, nkv = c["hidden"], c["head_dim"], c["heads"], c["kv_heads"]
        t = x.shape[0]
        r = F.rms_norm(x, (h,), self.n1, c["eps"])
        qkv = self.linear(r, self.w_qkv, self.s_qkv)
        q, k, v = qkv.split([h, nkv * hd, nkv * hd], dim=1)
        v = v.view(batch, seq, nkv, hd)
        if self.fused:
            q, k = self.nat.rope_bf16(qkv, cos, sin, nh, nkv, hd, seq)
            q, k = q.view(batch, seq, nh, hd), k.view(batch, seq, nkv, hd)
        else:
            q, k = _rope(q.view(batch, seq, nh, hd), cos, sin), _rope(k.view(batch, seq, nkv, hd), cos, sin)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=True, enable_gqa=True)
        a = a.transpose(1, 2).reshape(t, h)
        x = x + self.linear(a, self.w_o, self.s_o)
        r = F.rms_norm(x, (h,), self.n2, c["eps"])
        gu = self.linear(r, self.w_gu, self.s_gu)
        if self.fused:
            y = self.linear_q(*self.nat.silu_mul_quantize_rows_fp8(gu), self.w_d, self.s_d)
        else:
            g, u = gu.chunk(2, dim=1)
            y = self.linear(F.silu(g) * u, self.w_d, self.s_d)
        x = x + y
        return x

    def gemm_flops(self, tokens: int) -> float:
        c = self.cfg
        h, f, kvd = c["hidden"], c["intermediate"], c["kv_heads"] * c["head_dim"]
        return 2.0 * tokens * h * (h + 2 * kvd + h + 2 * f) + 2.0 * tokens * f * h


def _rope(x, cos, sin):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rope_tables(seq: int, device, cfg=LLAMA):
    hd = cfg["head_dim"]
    inv = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
    ang = torch.arange(seq, device=device, dtype=torch.float32)[:, None] * inv[None, :]
    cos = ang.cos().to(torch.bfloat16)[None, :, None, :]
    sin = ang.sin().to(torch.bfloat16)[None, :, None, :]
    return cos, sin


class Fp8LlamaStack:
    """`layers` decoder layers over a batch of `batch` x `seq` tokens."""

    def __init__(self, device, layers: int = LLAMA["layers"], seed: int = 0):
        gen = torch.Generator(device=device).manual_seed(seed)
        self.layers = [Fp8LlamaLayer(device, gen) for _ in range(layers)]
        self.device = device

    def forward(self, x, batch, seq):
        cos, sin = rope_tables(seq, x.device)
        for layer in self.layers:
            x = layer.forward(x, cos, sin, batch, seq)
        return x

    def gemm_flops(self, tokens: int) -> float:
        return sum(l.gemm_flops(tokens) for l in self.layers)


def llama_input(batch: int, seq: int, seed: int = 0) -> torch.Tensor:
    """Hidden states N(0,1) bf16, (batch*seq, hidden), generated on the CPU."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch * seq, LLAMA["hidden"], generator=g).to(torch.bfloat16)

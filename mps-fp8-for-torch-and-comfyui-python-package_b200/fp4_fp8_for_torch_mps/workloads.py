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

"""Generate the golden fixtures in tests/golden/ (run in a container that has
the reference tree mounted; the GPU box only reads the committed outputs).

    python tests/golden/gen_golden.py [--reference-root PATH]

Every table is produced by CPU PyTorch (the arithmetic the reference's own
tests compare the device path against: tests/test_mps_vs_cpu.py:124-149,
tests/test_integration.py:59-90) or read from the reference's test modules:

* FP4_SPEC, the nibble -> value table, from tests/test_fp4.py:14-20 (imported).
* The reference's pure-Python e4m3 spec encoder from
  tests/test_fp8_correctness.py:29-55 (imported), evaluated on its own
  special values (:72-87); kept to document where that spec differs from
  CPU torch (saturation at 448), not as a parity target.
* The exhaustive encode known answers of tests/test_mps_vs_cpu.py:124-149:
  every finite e4m3 value and the 125 midpoints between positive codes.

Output: tests/golden/golden.npz (bit patterns as unsigned integers).
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
FP8 = {0: torch.float8_e4m3fn, 1: torch.float8_e5m2}
OUT = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}
UINT = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}
NPU = {torch.float32: np.uint32, torch.bfloat16: np.uint16, torch.float16: np.uint16}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(UINT[t.dtype]).numpy().view(NPU[t.dtype]).copy()


def load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def f32_edge_values() -> np.ndarray:
    """The planted edge values of the FP8 round-trip workload."""
    sys.path.insert(0, os.path.join(ROOT, "mps-fp8-for-torch-and-comfyui-python-package_b200"))
    from fp4_fp8_for_torch_mps.workloads import planted_f32_edges
    return planted_f32_edges()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default="/root/reference")
    args = ap.parse_args()
    rt = os.path.join(args.reference_root, "tests")
    sys.path.insert(0, rt)                      # their modules import `conftest`
    fp4_mod = load_module(os.path.join(rt, "test_fp4.py"), "ref_test_fp4")
    corr_mod = load_module(os.path.join(rt, "test_fp8_correctness.py"), "ref_test_fp8_correctness")

    g: dict[str, np.ndarray] = {}
    codes = torch.arange(256, dtype=torch.uint8)

    # 1. decode tables: every code x {e4m3, e5m2} x {f32, bf16, f16}
    for f, dt in FP8.items():
        for o, odt in OUT.items():
            g[f"decode_f{f}_o{o}"] = bits(codes.view(dt).to(odt))
            # a single-element conversion takes CPU torch's scalar path; keep it
            # too so a path disagreement would show up in the fixture tests
            g[f"decode1_f{f}_o{o}"] = np.concatenate(
                [bits(codes[i:i + 1].view(dt).to(odt)) for i in range(256)])

    # 2. encode of every bf16 and f16 bit pattern
    all16 = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    for name, sdt in (("bf16", torch.bfloat16), ("f16", torch.float16)):
        x = all16.view(sdt)
        for f, dt in FP8.items():
            g[f"encode_{name}_f{f}"] = x.to(dt).view(torch.uint8).numpy().copy()

    # 3. planted f32 edge values and their encodings
    edge = f32_edge_values()
    g["edge_f32"] = edge
    xe = torch.from_numpy(edge.view(np.int32).copy()).view(torch.float32)
    for f, dt in FP8.items():
        g[f"edge_f32_f{f}"] = xe.to(dt).view(torch.uint8).numpy().copy()

    # 4. reference known answers (tests/test_mps_vs_cpu.py:124-149, :107-117)
    allf = codes.view(torch.float8_e4m3fn).to(torch.float32)
    exact = allf[~allf.isnan()]
    pos = allf[1:127]
    mids = (pos[:-1] + pos[1:]) / 2
    g["kat_exact_f32"] = bits(exact)
    g["kat_exact_e4m3"] = exact.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    g["kat_mid_f32"] = bits(mids)
    g["kat_mid_e4m3"] = mids.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    five = torch.tensor([0.5, 1.0, 2.0, 10.0, 100.0])
    g["kat_five_f32"] = bits(five)
    g["kat_five_e4m3"] = five.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()

    # 5. FP4 table from the reference test module and the reference spec encoder
    spec = fp4_mod.FP4_SPEC
    g["fp4_spec_f32"] = np.array([spec[i] for i in range(16)], np.float32).view(np.uint32)
    special = [0.0, 0.001953125, 0.013671875, 0.015625, 1.0, 448.0, 500.0]
    g["refspec_special_f32"] = np.array(special, np.float32).view(np.uint32)
    g["refspec_special_code"] = np.array([corr_mod.fp8_e4m3fn_encode_spec(v) for v in special], np.uint8)
    g["refspec_special_torch"] = torch.tensor(special).to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()

    # 6. FP4 decode x scale with CPU torch: value table (f32) gathered per
    #    nibble, one f32 product, cast to the output dtype.
    lut = torch.tensor([spec[i] for i in range(16)], dtype=torch.float32)
    b = torch.arange(256, dtype=torch.uint8)
    pair = torch.stack([lut[(b & 15).long()], lut[(b >> 4).long()]], dim=1).reshape(-1)
    for sc_name, sc in (("037", 0.37), ("1", 1.0), ("3", 3.0)):
        prod = pair * torch.tensor(sc, dtype=torch.float32)
        for o, odt in OUT.items():
            g[f"fp4_s{sc_name}_o{o}"] = bits(prod.to(odt))
        # reference op semantics: f16 table times the scale rounded to f16
        ref16 = pair.to(torch.float16) * torch.tensor([sc]).to(torch.float16)
        g[f"fp4ref_s{sc_name}"] = bits(ref16)

    # 7. fp8_mps::dequantize semantics (fp8_mps_native.py:65-82) with CPU torch
    for f, dt in FP8.items():
        for sc_name, sc in (("037", 0.37), ("1", 1.0), ("3", 3.0)):
            h = codes.view(dt).to(torch.float16) * torch.tensor([sc]).to(torch.float16)
            g[f"deqref_f{f}_s{sc_name}"] = bits(h)
            # f32-scale decode (one f32 product, one rounding)
            p = codes.view(dt).to(torch.float32) * torch.tensor(sc, dtype=torch.float32)
            for o, odt in OUT.items():
                g[f"deqs_f{f}_s{sc_name}_o{o}"] = bits(p.to(odt))

    # 8. small torch._scaled_mm cases on CPU (per-tensor scales only on CPU)
    gen = torch.Generator().manual_seed(1234)
    for case, (M, N, K) in enumerate(((64, 96, 128), (32, 48, 64), (17, 32, 32))):
        a = torch.randn(M, K, generator=gen) * 2
        bb = torch.randn(N, K, generator=gen)
        sa = a.abs().max() / 448
        sb = bb.abs().max() / 448
        aq = (a / sa).to(torch.float8_e4m3fn)
        bq = (bb / sb).to(torch.float8_e4m3fn)
        for oname, odt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
            c = torch._scaled_mm(aq, bq.t(), sa.reshape(()).float(), sb.reshape(()).float(),
                                 out_dtype=odt)
            g[f"mm{case}_{oname}"] = bits(c)
        g[f"mm{case}_a"] = aq.view(torch.uint8).numpy().copy()
        g[f"mm{case}_b"] = bq.view(torch.uint8).numpy().copy()
        g[f"mm{case}_sa"] = np.array([sa.item()], np.float32)
        g[f"mm{case}_sb"] = np.array([sb.item()], np.float32)

    g["torch_version"] = np.frombuffer(torch.__version__.encode(), np.uint8).copy()
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **g)
    print(f"wrote {path}: {len(g)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()

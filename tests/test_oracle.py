"""Pin the CPU oracle (oracle/fp8_oracle.c) against CPU PyTorch and the
reference's own known answers before any device result is compared with it."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

FP8 = {0: torch.float8_e4m3fn, 1: torch.float8_e5m2}


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("odt", [0, 1, 2])
def test_decode_tables_match_golden(golden, fmt, odt):
    mine = O.decode_fp8(np.arange(256, dtype=np.uint8), fmt, odt)
    assert np.array_equal(mine, golden[f"decode_f{fmt}_o{odt}"])
    assert np.array_equal(mine, golden[f"decode1_f{fmt}_o{odt}"])


@pytest.mark.parametrize("src", ["bf16", "f16"])
@pytest.mark.parametrize("fmt", [0, 1])
def test_encode_all_16bit_patterns(golden, src, fmt):
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    mine = O.encode_fp8(pats, 1 if src == "bf16" else 2, fmt)
    assert np.array_equal(mine, golden[f"encode_{src}_f{fmt}"])


@pytest.mark.parametrize("fmt", [0, 1])
def test_encode_planted_edges(golden, fmt):
    mine = O.encode_fp8(golden["edge_f32"], 0, fmt)
    assert np.array_equal(mine, golden[f"edge_f32_f{fmt}"])


def test_reference_known_answers(golden):
    # tests/test_mps_vs_cpu.py:124-149 and :107-117 of the reference
    for k in ("exact", "mid", "five"):
        mine = O.encode_fp8(golden[f"kat_{k}_f32"], 0, 0)
        assert np.array_equal(mine, golden[f"kat_{k}_e4m3"]), k
    assert golden["kat_exact_f32"].size == 254 and golden["kat_mid_f32"].size == 125


def test_fp4_table_matches_reference_spec(golden):
    assert np.array_equal(O.fp4_values().view(np.uint32), golden["fp4_spec_f32"])


@pytest.mark.parametrize("sc", ["037", "1", "3"])
@pytest.mark.parametrize("odt", [0, 1, 2])
def test_fp4_decode_scaled(golden, sc, odt):
    scale = {"037": 0.37, "1": 1.0, "3": 3.0}[sc]
    mine = O.fp4_decode(np.arange(256, dtype=np.uint8), odt, scale)
    assert np.array_equal(mine, golden[f"fp4_s{sc}_o{odt}"])


@pytest.mark.parametrize("sc", ["037", "1", "3"])
def test_fp4_dequant_reference_op(golden, sc):
    scale = {"037": 0.37, "1": 1.0, "3": 3.0}[sc]
    mine = O.fp4_dequant_ref_f16(np.arange(256, dtype=np.uint8), scale)
    assert np.array_equal(mine, golden[f"fp4ref_s{sc}"])


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("sc", ["037", "1", "3"])
def test_fp8_dequant_semantics(golden, fmt, sc):
    scale = {"037": 0.37, "1": 1.0, "3": 3.0}[sc]
    codes = np.arange(256, dtype=np.uint8)
    assert np.array_equal(O.dequant_ref_f16(codes, fmt, scale), golden[f"deqref_f{fmt}_s{sc}"])
    for odt in (0, 1, 2):
        mine = O.decode_fp8(codes, fmt, odt, scale=scale)
        ref = golden[f"deqs_f{fmt}_s{sc}_o{odt}"]
        if odt == 1:
            # CPU torch's vectorised f32->bf16 cast writes NaN as 0xFFFF while
            # its scalar cast and its fp8->bf16 conversion write 0x7FC0; the
            # scaled decode follows the latter, so compare NaN-ness there.
            nan_ref = (ref & 0x7FFF) > 0x7F80
            assert np.array_equal(nan_ref, (mine & 0x7FFF) > 0x7F80)
            assert np.all(mine[nan_ref] == 0x7FC0)
            assert np.array_equal(mine[~nan_ref], ref[~nan_ref])
        else:
            assert np.array_equal(mine, ref), odt


def test_reference_spec_divergence_is_documented(golden):
    """The reference's Python spec and shader saturate 500.0 to 0x7E; CPU
    torch (the parity target) gives NaN 0x7F. Everything else agrees."""
    code = golden["refspec_special_code"]
    tor = golden["refspec_special_torch"]
    assert np.array_equal(code[:-1], tor[:-1])
    assert code[-1] == 0x7E and tor[-1] == 0x7F
    shader = O.refshader_e4m3(golden["refspec_special_f32"].view(np.float32))
    assert np.array_equal(shader, code)


def test_fp4_encode_reference_thresholds():
    """The reference FP4 encoder's ties (tests/test_fp4.py:80-107 accept
    either neighbour at midpoints and clamp to +-6)."""
    v = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 100.0, -100.0, 0.001, -0.001, -0.0], np.float32)
    packed = O.fp4_encode_ref(v)
    lo, hi = packed & 15, packed >> 4
    codes = np.stack([lo, hi], 1).reshape(-1)
    vals = O.fp4_values()[codes]
    assert list(vals[:7]) == [0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert vals[7] == 6.0 and vals[8] == -6.0 and vals[9] == 0.0 and vals[10] == 0.0
    assert codes[11] == 0  # -0.0 encodes as +0


@pytest.mark.parametrize("case", [0, 1, 2])
def test_scaled_mm_reference_vs_cpu_torch(golden, case):
    a, b = golden[f"mm{case}_a"], golden[f"mm{case}_b"]
    sa, sb = golden[f"mm{case}_sa"][0], golden[f"mm{case}_sb"][0]
    ref, S = O.scaled_mm_ref(a, b, sa, sb)
    c32 = golden[f"mm{case}_f32"].view(np.float32).astype(np.float64)
    # CPU torch accumulates in f32: agreement to a few f32 ulps of the magnitude sum
    assert np.all(np.abs(c32 - ref) <= 2.0 ** -20 * S + 1e-30)
    cbf = (golden[f"mm{case}_bf16"].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert np.all(np.abs(cbf - ref) <= O.bf16_ulp(ref) + 2.0 ** -20 * S)


def test_encode_sweep_sampled_f32():
    """A strided sample of the 2^32 f32 patterns (the full sweep runs in the
    GPU tests, and was run once against CPU torch when the oracle was written)."""
    bases = [0, 0x3F800000, 0x43E00000, 0x47600000, 0x7F7F0000, 0xC3E00000]
    bases += [int(x) for x in np.random.default_rng(0).integers(0, 2**32 - (1 << 20), 8, dtype=np.uint64)]
    for base in bases:
        base = min(base, 2**32 - (1 << 20))
        bits_t = torch.arange(base, base + (1 << 20), dtype=torch.int64).to(torch.int32)
        for fmt, dt in FP8.items():
            ref = bits_t.view(torch.float32).to(dt).view(torch.uint8).numpy()
            mine = O.encode_range(base, base + (1 << 20), fmt)
            assert np.array_equal(ref, mine), (hex(base), fmt)

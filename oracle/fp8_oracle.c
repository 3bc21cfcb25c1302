/*
 * ORACLE — test infrastructure only. Nothing in the product links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py use it, and only as the checker or the timed CPU baseline.
 *
 * A scalar CPU restatement of the arithmetic on the FP8/FP4 conversion path
 * that the plugin intercepts (tensor.to / tensor.copy_ / fp8_mps::* ops).
 *
 * Provenance of the semantics restated here
 * -----------------------------------------
 * The reference plugin (fp4-fp8-for-torch-mps) does its conversions on the GPU
 * and its own tests pin the result to CPU PyTorch byte for byte:
 *   tests/test_mps_vs_cpu.py:124-149  encode of every finite e4m3 value and of
 *                                     the midpoints between positive codes ==
 *                                     CPU `.to(torch.float8_e4m3fn)`
 *   tests/test_mps_vs_cpu.py:59-75    decode of all 256 codes == CPU path
 *   tests/test_integration.py:67-77   `.to(float32)` of arange(256) == CPU
 * CPU PyTorch is therefore the arithmetic this path must reproduce. That code
 * is a third-party dependency absent from the reference tree: torch 2.10.0 as
 * pinned in uv.lock:514-515 (torch>=2.9 in pyproject.toml:11); this image
 * carries torch 2.11.0 whose c10 headers hold the same algorithms:
 *   torch/headeronly/util/Float8_e4m3fn.h:67  fp8e4m3fn_to_fp32_value
 *   torch/headeronly/util/Float8_e4m3fn.h:170 fp8e4m3fn_from_fp32_value
 *   torch/headeronly/util/Float8_e5m2.h:56    fp8e5m2_to_fp32_value
 *   torch/headeronly/util/Float8_e5m2.h:77    fp8e5m2_from_fp32_value
 *   torch/headeronly/util/Half.h:118,261      x86 F16C half<->float
 *   torch/headeronly/util/BFloat16.h:100      round_to_nearest_even
 * The published algorithm (IEEE-style round-to-nearest-even onto the e4m3fn /
 * e5m2 grids, e4m3fn overflow to NaN, e5m2 overflow to inf) is restated below
 * in an independent formulation (generic integer RNE onto a (E,M) grid), not
 * transcribed from those headers. NaN payload rules follow what the x86 build
 * of CPU torch produces (F16C conversions quiet NaNs and keep their payload;
 * BFloat16 maps every NaN to 0x7FC0).
 *
 * FP4 (float4_e2m1fn_x2): CPU torch has no conversion. The value table follows
 * the reference shader (shaders/fp8_matmul.metal:77-85) and its test table
 * (tests/test_fp4.py:14-20, -0.0 at nibble 0b1000); element 2i is the low
 * nibble and 2i+1 the high nibble (fp8_matmul.metal:259-260,
 * tests/test_fp4.py:44-50). The reference launcher multiplies by the scale in
 * fp16 (fp8_mps_native.py:177-178); that is orc_fp4_dequant_ref_f16.
 *
 * Pinned against: the exhaustive CPU-torch tables and the reference's known
 * answers in tests/golden/ (see tests/test_oracle.py), and once against CPU
 * torch on all 2^32 float32 bit patterns for both fp8 formats.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stddef.h>

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* Generic round-to-nearest-even of a non-negative finite f32 (bits `a`) onto
 * a binary grid with `mbits` stored mantissa bits and smallest normal
 * exponent `emin`. Returns the magnitude code (exponent field << mbits |
 * mantissa) of the nearest grid point, which may exceed the format's range;
 * the caller applies the overflow policy. */
static uint32_t rne_code(uint32_t a, int mbits, int emin)
{
    uint32_t ef = a >> 23, frac = a & 0x7FFFFFu;
    uint64_t m; int e;                 /* value = m * 2^e, m integer */
    if (ef == 0) { m = frac; e = -149; }
    else         { m = frac | 0x800000u; e = (int)ef - 150; }
    if (m == 0) return 0;
    /* binade of the value: 2^E <= value < 2^(E+1) */
    int msb = 63 - __builtin_clzll(m);
    int E = msb + e;
    int qexp = (E < emin ? emin : E) - mbits;   /* grid spacing 2^qexp */
    int shift = qexp - e;
    uint64_t q;
    if (shift <= 0) {
        q = m << (-shift);
    } else if (shift >= 40) {
        q = 0;                          /* far below half a quantum */
    } else {
        q = m >> shift;
        uint64_t rem = m & ((1ull << shift) - 1), half = 1ull << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
    }
    if (q == 0) return 0;
    if (qexp == emin - mbits && q <= (1ull << mbits))
        return (uint32_t)q;             /* subnormal (or rounds up to min normal) */
    /* normal: q in [2^mbits, 2^(mbits+1)], carry into the exponent is implied */
    int efield = qexp + mbits - emin + 1;
    return (uint32_t)(((uint64_t)efield << mbits) + (q - (1ull << mbits)));
}

/* f32 -> float8_e4m3fn byte (CPU torch semantics: RNE; anything rounding past
 * 448, inf and NaN -> 0x7F | sign). */
uint8_t orc_e4m3_from_f32_bits(uint32_t bits)
{
    uint32_t s = (bits >> 24) & 0x80u, a = bits & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint8_t)(s | 0x7F);
    uint32_t c = rne_code(a, 3, -6);
    if (c > 0x7E) c = 0x7F;
    return (uint8_t)(s | c);
}

/* f32 -> float8_e5m2 byte (RNE; rounding past 57344 and inf -> 0x7C | sign;
 * NaN -> 0x7F | sign). */
uint8_t orc_e5m2_from_f32_bits(uint32_t bits)
{
    uint32_t s = (bits >> 24) & 0x80u, a = bits & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint8_t)(s | 0x7F);
    if (a == 0x7F800000u) return (uint8_t)(s | 0x7C);
    uint32_t c = rne_code(a, 2, -14);
    if (c > 0x7B) c = 0x7C;
    return (uint8_t)(s | c);
}

/* ------------------------------------------------------------------------ */
/* float32 -> float16 and bfloat16 bit patterns as CPU torch computes them. */
uint16_t orc_f16_from_f32_bits(uint32_t bits)
{
    uint32_t s = (bits >> 16) & 0x8000u, a = bits & 0x7FFFFFFFu;
    if (a > 0x7F800000u)                 /* NaN: quiet, keep top payload bits */
        return (uint16_t)(s | 0x7C00u | 0x200u | ((a & 0x7FFFFFu) >> 13));
    if (a == 0x7F800000u) return (uint16_t)(s | 0x7C00u);
    uint32_t c = rne_code(a, 10, -14);
    if (c >= 0x7C00u) c = 0x7C00u;       /* overflow -> inf */
    return (uint16_t)(s | c);
}

uint16_t orc_bf16_from_f32_bits(uint32_t bits)
{
    uint32_t a = bits & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7FC0u; /* every NaN, sign dropped */
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7FFFu + lsb) >> 16);
}

uint32_t orc_f32_from_f16_bits(uint16_t h)
{
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, f = h & 0x3FFu;
    if (e == 0x1F) return f ? (s | 0x7FC00000u | (f << 13)) : (s | 0x7F800000u);
    if (e == 0) {
        if (f == 0) return s;
        double v = ldexp((double)f, -24);
        return s | f2u((float)v);
    }
    return s | ((e + 112u) << 23) | (f << 13);
}

uint32_t orc_f32_from_bf16_bits(uint16_t b) { return (uint32_t)b << 16; }

/* ------------------------------------------------------------------------ */
/* fp8 byte -> float32 bits (CPU torch semantics, NaN payloads included). */
uint32_t orc_f32_from_e4m3(uint8_t c)
{
    uint32_t s = (uint32_t)(c & 0x80u) << 24, mag = c & 0x7Fu;
    if (mag == 0x7F) return s | 0x7FF00000u;
    uint32_t ef = mag >> 3, mf = mag & 7u;
    double v = ef ? ldexp((double)(8 + mf), (int)ef - 10) : ldexp((double)mf, -9);
    return s | f2u((float)v);
}

uint32_t orc_f32_from_e5m2(uint8_t c)
{
    uint32_t s = (uint32_t)(c & 0x80u) << 24, mag = c & 0x7Fu;
    uint32_t ef = mag >> 2, mf = mag & 3u;
    if (ef == 0x1F) return mf ? (s | 0x7FC00000u | (mf << 21)) : (s | 0x7F800000u);
    double v = ef ? ldexp((double)(4 + mf), (int)ef - 17) : ldexp((double)mf, -16);
    return s | f2u((float)v);
}

/* ------------------------------------------------------------------------ */
/* Array drivers. fmt: 0 = e4m3fn, 1 = e5m2.  src dtype: 0 = f32, 1 = bf16,
 * 2 = f16 (raw bit patterns).  Encoding from a 16-bit type widens exactly to
 * f32 first, as CPU torch does. */
static uint32_t widen(const void *src, int sdt, size_t i)
{
    if (sdt == 0) return ((const uint32_t *)src)[i];
    if (sdt == 1) return orc_f32_from_bf16_bits(((const uint16_t *)src)[i]);
    return orc_f32_from_f16_bits(((const uint16_t *)src)[i]);
}

void orc_encode_fp8(const void *src, int sdt, uint8_t *dst, size_t n, int fmt)
{
    for (size_t i = 0; i < n; i++) {
        uint32_t b = widen(src, sdt, i);
        dst[i] = fmt ? orc_e5m2_from_f32_bits(b) : orc_e4m3_from_f32_bits(b);
    }
}

/* scaled encode, as the reference quantize does it (fp8_mps_native.py:110):
 * the f32 product x*scale is rounded to f32 before encoding. */
void orc_encode_fp8_scaled(const float *src, uint8_t *dst, size_t n, int fmt, float scale)
{
    for (size_t i = 0; i < n; i++) {
        float v = src[i] * scale;
        uint32_t b = f2u(v);
        dst[i] = fmt ? orc_e5m2_from_f32_bits(b) : orc_e4m3_from_f32_bits(b);
    }
}

/* out dtype: 0 = f32, 1 = bf16, 2 = f16 */
void orc_decode_fp8(const uint8_t *src, int fmt, void *dst, int odt, size_t n)
{
    for (size_t i = 0; i < n; i++) {
        uint32_t b = fmt ? orc_f32_from_e5m2(src[i]) : orc_f32_from_e4m3(src[i]);
        if (odt == 0)      ((uint32_t *)dst)[i] = b;
        else if (odt == 1) ((uint16_t *)dst)[i] = orc_bf16_from_f32_bits(b);
        else               ((uint16_t *)dst)[i] = orc_f16_from_f32_bits(b);
    }
}

/* f32 product rounded once to f32 (x86 mulss semantics, NaN operand kept). */
static uint32_t mul_f32(uint32_t vb, float s)
{
    if ((vb & 0x7FFFFFFFu) > 0x7F800000u) return vb;
    return f2u(u2f(vb) * s);
}

static void store(void *dst, int odt, size_t i, uint32_t b)
{
    if (odt == 0)      ((uint32_t *)dst)[i] = b;
    else if (odt == 1) ((uint16_t *)dst)[i] = orc_bf16_from_f32_bits(b);
    else               ((uint16_t *)dst)[i] = orc_f16_from_f32_bits(b);
}

/* decode x f32 scale -> out dtype (one f32 product, one rounding to out). */
void orc_decode_fp8_scaled(const uint8_t *src, int fmt, void *dst, int odt, size_t n, float scale)
{
    for (size_t i = 0; i < n; i++) {
        uint32_t b = fmt ? orc_f32_from_e5m2(src[i]) : orc_f32_from_e4m3(src[i]);
        store(dst, odt, i, mul_f32(b, scale));
    }
}

/* fp8_mps::dequantize semantics (fp8_mps_native.py:65-82): decode to f16,
 * multiply by the scale rounded to f16, product rounded to f16. */
void orc_dequant_ref_f16(const uint8_t *src, int fmt, uint16_t *dst, size_t n, float scale)
{
    float s16 = u2f(orc_f32_from_f16_bits(orc_f16_from_f32_bits(f2u(scale))));
    for (size_t i = 0; i < n; i++) {
        uint32_t b = fmt ? orc_f32_from_e5m2(src[i]) : orc_f32_from_e4m3(src[i]);
        uint32_t h = orc_f16_from_f32_bits(b);
        uint32_t hb = orc_f32_from_f16_bits((uint16_t)h);
        dst[i] = orc_f16_from_f32_bits(mul_f32(hb, s16));
    }
}

/* ------------------------------------------------------------------------ */
/* FP4 e2m1 nibble values (fp8_matmul.metal:77-85, tests/test_fp4.py:14-20). */
static const float fp4_values[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

float orc_fp4_value(int nibble) { return fp4_values[nibble & 15]; }

/* packed bytes -> 2*n outputs, low nibble first, times an f32 scale:
 * out = round_out(round_f32(value * scale)). */
void orc_fp4_decode(const uint8_t *src, size_t nbytes, void *dst, int odt, float scale)
{
    for (size_t i = 0; i < nbytes; i++) {
        uint8_t b = src[i];
        float lo = (float)((double)fp4_values[b & 15] * (double)scale);
        float hi = (float)((double)fp4_values[b >> 4] * (double)scale);
        store(dst, odt, 2 * i, f2u(lo));
        store(dst, odt, 2 * i + 1, f2u(hi));
    }
}

/* fp8_mps::fp4_dequantize semantics (fp8_mps_native.py:162-179): f16 values
 * times the scale rounded to f16, product rounded to f16. */
void orc_fp4_dequant_ref_f16(const uint8_t *src, size_t nbytes, uint16_t *dst, float scale)
{
    float s16 = u2f(orc_f32_from_f16_bits(orc_f16_from_f32_bits(f2u(scale))));
    for (size_t i = 0; i < nbytes; i++) {
        uint8_t b = src[i];
        dst[2 * i]     = orc_f16_from_f32_bits(f2u(fp4_values[b & 15] * s16));
        dst[2 * i + 1] = orc_f16_from_f32_bits(f2u(fp4_values[b >> 4] * s16));
    }
}

/* ------------------------------------------------------------------------ */
/* The reference shader's own encoders, restated to document where the
 * reference diverges from CPU torch (fp8_matmul.metal:88-102, :105-142).
 * The FP4 one is also the parity target of fp8_mps::fp4_encode, which keeps
 * the reference's thresholds. */
uint8_t orc_refshader_e4m3(float val)
{
    uint32_t raw = f2u(val), sign = raw >> 31;
    float a = fabsf(val);
    if (a >= 448.0f) return (uint8_t)((sign << 7) | 0x7E);
    if (a < (1.0f / 512.0f)) return (uint8_t)(sign << 7);
    uint32_t bits = f2u(a);
    int ex = (int)((bits >> 23) & 0xFF) - 127;
    uint32_t man = bits & 0x7FFFFF;
    if (ex < -6) {
        uint32_t m = (uint32_t)nearbyintf(a * 512.0f);
        if (m >= 8) return (uint8_t)((sign << 7) | 0x08);
        return (uint8_t)((sign << 7) | m);
    }
    uint32_t tr = man & 0xFFFFF, half = 1u << 19, m = man >> 20;
    if (tr > half || (tr == half && (m & 1))) m++;
    int fe = ex + 7;
    if (m > 7) { m = 0; fe++; }
    if (fe < 1) fe = 1;
    if (fe > 15) fe = 15;
    if (fe == 15 && m == 7) m = 6;
    return (uint8_t)((sign << 7) | (uint32_t)(fe << 3) | m);
}

uint8_t orc_refshader_fp4(float val)
{
    uint32_t sign = 0;
    if (val < 0.0f) { sign = 1; val = -val; }
    uint32_t code;
    if (val < 0.25f) code = 0;
    else if (val < 0.75f) code = 1;
    else if (val < 1.25f) code = 2;
    else if (val < 1.75f) code = 3;
    else if (val < 2.5f) code = 4;
    else if (val < 3.5f) code = 5;
    else if (val < 5.0f) code = 6;
    else code = 7;
    return (uint8_t)((sign << 3) | code);
}

/* packed FP4 encode with the reference thresholds, scaled as the reference
 * fp4_quantize does (fp8_mps_native.py:210): f32 product, then encode. */
void orc_fp4_encode_ref(const float *src, size_t n, uint8_t *dst, float scale, int use_scale)
{
    for (size_t i = 0; i + 1 < n; i += 2) {
        float lo = use_scale ? src[i] * scale : src[i];
        float hi = use_scale ? src[i + 1] * scale : src[i + 1];
        dst[i / 2] = (uint8_t)(orc_refshader_fp4(lo) | (orc_refshader_fp4(hi) << 4));
    }
}

/* ------------------------------------------------------------------------ */
/* Exhaustive helper: encode every f32 bit pattern in [lo, hi) and write the
 * bytes (dst has hi-lo entries). Used by the 2^32 sweep tests. */
void orc_encode_range(uint64_t lo, uint64_t hi, int fmt, uint8_t *dst)
{
    for (uint64_t b = lo; b < hi; b++)
        dst[b - lo] = fmt ? orc_e5m2_from_f32_bits((uint32_t)b) : orc_e4m3_from_f32_bits((uint32_t)b);
}

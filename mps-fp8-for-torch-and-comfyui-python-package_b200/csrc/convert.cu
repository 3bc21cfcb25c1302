// FP8 / FP4 conversion kernels for B200 (sm_100a).
//
// All of these are HBM-bound byte streams. Design:
//  * Every thread moves one "unit" per step: the input bytes that produce
//    exactly 32 output bytes (decoders) or 16 output bytes (encoders). The
//    unit index is `thread + j * total_threads`, so each warp-wide load and
//    store covers one contiguous span (a full 1 KiB for 32-byte stores):
//    every DRAM sector is written whole by a single instruction.
//  * 256-bit global accesses (ld/st .v8.u32, new on sm_100) halve the number
//    of memory instructions against 16-byte vectors; four units per thread
//    per step keep four independent loads in flight.
//  * Grid-stride over at most (blocks per SM) x (SM count) CTAs.
//  * Encode (float -> fp8): PTX cvt.rn.satfinite.{e4m3,e5m2}x2.f32 converts
//    two elements per instruction; the only cases where that instruction and
//    CPU PyTorch disagree (magnitudes that round past the largest finite
//    value, inf, NaN) are found with one integer max per 16 elements and
//    patched on a rare slow path.
//  * Decode (fp8 -> float, fp4 -> float): a per-block table in shared memory
//    maps each code (or each packed fp4 byte) to its output bit pattern, with
//    the scale already applied. The table is replicated 32 times, one copy per
//    lane, so lane L always reads bank L: every lookup is a single
//    conflict-free shared-memory wavefront.
//
// Semantics (bit-exact with CPU PyTorch on x86, NaN payloads included):
//   e4m3fn encode: RNE; |x| rounding past 448, inf, NaN -> 0x7F | sign
//   e5m2 encode:   RNE; rounding past 57344, inf -> 0x7C | sign; NaN -> 0x7F | sign
//   decode to f32: exact; e4m3fn NaN -> sign|0x7FF00000; e5m2 NaN quieted
//   decode to bf16: exact; every NaN -> 0x7FC0
//   decode to f16: exact; NaN -> sign|0x7E00|payload>>13
// The reference kernels these replace: shaders/fp8_matmul.metal:105-142 and
// :240-248 (encode), :229-237 (decode), :251-261 (fp4 decode), :88-102 and
// :264-274 (fp4 encode).
#include "common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

namespace fp8b200 {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;  // units per thread per step

// ------------------------------------------------------------------ loads/stores
struct U8x32 { uint32_t w[8]; };

__device__ __forceinline__ U8x32 ld_u256(const void *p) {
  U8x32 v;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                 "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_u128(void *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

inline bool aligned32(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

// ------------------------------------------------------------------ element semantics
// fp8 code -> float32 bit pattern (CPU PyTorch semantics).
__device__ __forceinline__ uint32_t fp8_to_f32_bits(uint32_t c, int fmt) {
  const uint32_t s = (c & 0x80u) << 24, mag = c & 0x7Fu;
  if (fmt == FP8B200_E4M3) {
    if (mag == 0x7Fu) return s | 0x7FF00000u;
    const uint32_t ef = mag >> 3, mf = mag & 7u;
    if (ef == 0) return s | f2u(__uint2float_rn(mf) * 0x1p-9f);  // exact
    return s | ((ef + 120u) << 23) | (mf << 20);
  }
  const uint32_t ef = mag >> 2, mf = mag & 3u;
  if (ef == 31u) return mf ? (s | 0x7FC00000u | (mf << 21)) : (s | 0x7F800000u);
  if (ef == 0) return s | f2u(__uint2float_rn(mf) * 0x1p-16f);  // exact
  return s | ((ef + 112u) << 23) | (mf << 21);
}

__device__ __forceinline__ bool is_nan_bits(uint32_t b) { return (b & 0x7FFFFFFFu) > 0x7F800000u; }

// float32 bits -> output dtype bits (f32 unchanged; bf16/f16 round to nearest even).
__device__ __forceinline__ uint32_t f32_to_out_bits(uint32_t b, int odt) {
  if (odt == FP8B200_F32) return b;
  const bool nan = is_nan_bits(b);
  if (odt == FP8B200_BF16)
    return nan ? 0x7FC0u : (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(u2f(b)));
  if (nan) return ((b >> 16) & 0x8000u) | 0x7E00u | ((b & 0x7FFFFFu) >> 13);
  return (uint32_t)__half_as_ushort(__float2half_rn(u2f(b)));
}

// value bits (f32) x scale according to scale_mode, result as out-dtype bits.
__device__ __forceinline__ uint32_t apply_scale(uint32_t vb, int odt, float scale, int mode) {
  if (mode == FP8B200_SCALE_F32) {
    if (!is_nan_bits(vb)) vb = f2u(__fmul_rn(u2f(vb), scale));
    return f32_to_out_bits(vb, odt);
  }
  if (mode == FP8B200_SCALE_F16_REF) {
    // f16(value) * f16(scale) rounded to f16 (output dtype is f16 here)
    const uint32_t h = f32_to_out_bits(vb, FP8B200_F16);
    if (is_nan_bits(vb)) return h;
    const float s16 = __half2float(__float2half_rn(scale));
    const float v16 = __half2float(__ushort_as_half((unsigned short)h));
    return f32_to_out_bits(f2u(__fmul_rn(v16, s16)), FP8B200_F16);
  }
  return f32_to_out_bits(vb, odt);
}

__device__ __forceinline__ float load_scale(const float *scale, int mode) {
  return (mode != FP8B200_SCALE_NONE && scale != nullptr) ? __ldg(scale) : 1.0f;
}

__constant__ float kFp4Values[16] = {
    0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
    -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f,
};

// ------------------------------------------------------------------ decoders
// Bulk-copy pipeline. A CTA streams chunks of CIN input bytes that decode to
// exactly 16 KiB of output: one thread issues cp.async.bulk loads of the next
// chunks into a 3-stage shared-memory ring (mbarrier completion); all threads
// decode from shared memory through the table into a 3-stage output ring; one
// thread writes each finished output chunk back with a single
// cp.async.bulk store. HBM traffic is then only bulk transfers, no LSU global
// loads or stores, and the bytes in flight do not depend on registers.
//
// Tables (replicated per lane so lane L reads bank L, conflict-free):
//   fp8 -> any:     256 codes -> output bits (u32)            32 KiB
//   fp4 -> 16-bit:  256 bytes -> (lo, hi) output pair (u32)   32 KiB
//   fp4 -> f32:     16 nibbles -> output bits (u32)            2 KiB
// Each thread step reads G input bytes and writes 8 or 16 contiguous output
// bytes at thread-contiguous offsets (conflict-free shared stores).
constexpr int kDecThreads = 256;
constexpr int kStages = 3;
constexpr int kOutChunk = 16384;

enum DecKind { DEC_FP8_16 = 0, DEC_FP8_32 = 1, DEC_FP4_16 = 2, DEC_FP4_32 = 3 };

template <int KIND>
struct Dec {
  static constexpr int kOutPerIn = KIND == DEC_FP8_16 ? 2 : KIND == DEC_FP8_32 ? 4 : KIND == DEC_FP4_16 ? 4 : 8;
  static constexpr int kIn = kOutChunk / kOutPerIn;            // input bytes per chunk
  static constexpr int kG = KIND == DEC_FP4_32 ? 2 : 4;         // input bytes per thread step
  static constexpr int kSteps = kIn / kG / kDecThreads;
  static constexpr int kLutEntries = KIND == DEC_FP4_32 ? 16 : 256;
  static constexpr int kLutBytes = kLutEntries * 32 * 4;
  static constexpr int kSmem = kLutBytes + kStages * (kIn + kOutChunk) + 64;
};

// output bits for input code c (fp8 code, fp4 byte pair, or fp4 nibble)
template <int KIND>
__device__ __forceinline__ uint32_t dec_entry(uint32_t c, int fmt, int odt, float s, int mode) {
  if constexpr (KIND == DEC_FP8_16 || KIND == DEC_FP8_32) return apply_scale(fp8_to_f32_bits(c, fmt), odt, s, mode);
  else if constexpr (KIND == DEC_FP4_16)
    return apply_scale(f2u(kFp4Values[c & 15u]), odt, s, mode) | (apply_scale(f2u(kFp4Values[c >> 4]), odt, s, mode) << 16);
  else return apply_scale(f2u(kFp4Values[c & 15u]), odt, s, mode);
}

// decode one thread step: G input bytes -> 8 or 16 output bytes
template <int KIND>
__device__ __forceinline__ void dec_step(const uint8_t *in, uint8_t *out, int idx, const uint32_t *tab) {
#define T(c) tab[(uint32_t)(c) << 5]
  if constexpr (KIND == DEC_FP8_16) {
    const uint32_t x = reinterpret_cast<const uint32_t *>(in)[idx];
    reinterpret_cast<uint2 *>(out)[idx] =
        make_uint2(T(x & 255u) | (T((x >> 8) & 255u) << 16), T((x >> 16) & 255u) | (T(x >> 24) << 16));
  } else if constexpr (KIND == DEC_FP8_32 || KIND == DEC_FP4_16) {
    const uint32_t x = reinterpret_cast<const uint32_t *>(in)[idx];
    reinterpret_cast<uint4 *>(out)[idx] = make_uint4(T(x & 255u), T((x >> 8) & 255u), T((x >> 16) & 255u), T(x >> 24));
  } else {
    const uint32_t x = reinterpret_cast<const uint16_t *>(in)[idx];
    reinterpret_cast<uint4 *>(out)[idx] = make_uint4(T(x & 15u), T((x >> 4) & 15u), T((x >> 8) & 15u), T(x >> 12));
  }
#undef T
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Wait-loop bound for the bulk pipeline (the loads it waits for are plain
// global->shared copies, complete in microseconds).
constexpr long long kBulkSpinLimit = 1ll << 24;
__device__ int g_bulk_status;
// After a timed-out wait a CTA stops early, while bulk loads it issued for
// later chunks may still be landing in its shared memory: its thread 0 holds
// the CTA (and so its shared memory) for a bounded 200 us before it exits.
__device__ __forceinline__ void drain_loads() {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    __nanosleep(1000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < 200000ull);
}

// Programmatic dependent launch: the bulk converters let the next kernel in
// the stream launch as soon as every CTA of this one has started, and wait
// for the previous kernel's completion (and memory) only before their first
// global access, so launch and prologue overlap the previous kernel's tail.
// Both are no-ops for launches without the programmatic-serialization
// attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Bring `bytes` of global memory at `src` into L2 ahead of their bulk load. Issued before
// pdl_wait_prior by the bulk converters: a prefetch writes nothing, and L2 is where global
// memory is coherent, so a line it fetches before the previous kernel's writes land is
// updated by those writes, and the bulk loads after the wait read current data. It takes
// the DRAM latency of a launch's first chunks off the time after the wait (~1.4 us of a
// ~16 us 4096^2 decode).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

template <int KIND>
__global__ void __launch_bounds__(kDecThreads)
decode_bulk_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t nbytes, int fmt, int odt,
                   const float *__restrict__ scale, int mode) {
  using C = Dec<KIND>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint32_t *lut = reinterpret_cast<uint32_t *>(smem_raw);
  uint8_t *in_ring = smem_raw + C::kLutBytes;
  uint8_t *out_ring = in_ring + kStages * C::kIn;
  uint64_t *bar = reinterpret_cast<uint64_t *>(out_ring + kStages * kOutChunk);
  const int64_t nch = nbytes / C::kIn;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar + i)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_prefetch_l2(src + c * C::kIn, C::kIn);
    }
  }
  pdl_launch_dependents();
  pdl_wait_prior();  // nothing in global memory is read or written before this (the L2 prefetch above excepted)
  const float s = load_scale(scale, mode);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_load(smem_addr(in_ring + i * C::kIn), src + c * C::kIn, C::kIn, smem_addr(bar + i));
    }
  }
  {  // table: distinct entries once, then one copy per lane
    __shared__ uint32_t distinct[C::kLutEntries];
    for (int c = threadIdx.x; c < C::kLutEntries; c += kDecThreads) distinct[c] = dec_entry<KIND>(c, fmt, odt, s, mode);
    __syncthreads();
    for (int i = threadIdx.x; i < C::kLutEntries * 32; i += kDecThreads) lut[i] = distinct[i >> 5];
    __syncthreads();
  }
  const uint32_t *tab = lut + (threadIdx.x & 31u);

  bool failed = false;
  for (int64_t i = 0;; i++) {
    const int64_t c = blockIdx.x + i * gridDim.x;
    if (c >= nch) break;
    const int st = (int)(i % kStages);
    const uint32_t ph = (uint32_t)((i / kStages) & 1);
    int timed_out = 0;
    for (long long n = 0; !mbar_try(smem_addr(bar + st), ph);)
      if (++n > kBulkSpinLimit) { timed_out = 1; break; }
    if (__syncthreads_or(timed_out)) {  // block-uniform exit; the host sees the status word
      if (threadIdx.x == 0) atomicExch(&g_bulk_status, 1);
      failed = true;
      break;
    }
    // the store issued kStages chunks ago must have finished reading out[st]
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kStages - 1) : "memory");
    __syncthreads();
    const uint8_t *in = in_ring + st * C::kIn;
    uint8_t *out = out_ring + st * kOutChunk;
#pragma unroll
    for (int j = 0; j < C::kSteps; j++) dec_step<KIND>(in, out, threadIdx.x + j * kDecThreads, tab);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy smem accesses before the bulk copies
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + c * kOutChunk),
                   "r"(smem_addr(out)), "r"(kOutChunk)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      const int64_t c2 = blockIdx.x + (i + kStages) * gridDim.x;
      if (c2 < nch) bulk_load(smem_addr(in_ring + st * C::kIn), src + c2 * C::kIn, C::kIn, smem_addr(bar + st));
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (failed && threadIdx.x == 0) drain_loads();  // loads issued before the timeout may still be landing

  // ragged tail (fewer than kIn input bytes), element-wise through the table
  if (blockIdx.x == gridDim.x - 1) {
    for (int64_t b = nch * C::kIn + threadIdx.x; b < nbytes; b += kDecThreads) {
      const uint32_t code = src[b];
      if constexpr (KIND == DEC_FP8_16) reinterpret_cast<uint16_t *>(dst)[b] = (uint16_t)tab[code << 5];
      else if constexpr (KIND == DEC_FP8_32 || KIND == DEC_FP4_16) reinterpret_cast<uint32_t *>(dst)[b] = tab[code << 5];
      else reinterpret_cast<uint2 *>(dst)[b] = make_uint2(tab[(code & 15u) << 5], tab[(code >> 4) << 5]);
    }
  }
}

// Unaligned buffers: one input byte per thread, same semantics, no table.
__global__ void __launch_bounds__(kThreads)
decode_scalar_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t nbytes, int fp4, int fmt,
                     int odt, const float *__restrict__ scale, int mode) {
  const float s = load_scale(scale, mode);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nbytes; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t b = src[i];
    if (!fp4) {
      const uint32_t r = apply_scale(fp8_to_f32_bits(b, fmt), odt, s, mode);
      if (odt == FP8B200_F32) reinterpret_cast<uint32_t *>(dst)[i] = r;
      else reinterpret_cast<uint16_t *>(dst)[i] = (uint16_t)r;
    } else {
      const uint32_t lo = apply_scale(f2u(kFp4Values[b & 15u]), odt, s, mode);
      const uint32_t hi = apply_scale(f2u(kFp4Values[b >> 4]), odt, s, mode);
      if (odt == FP8B200_F32) {
        reinterpret_cast<uint32_t *>(dst)[2 * i] = lo;
        reinterpret_cast<uint32_t *>(dst)[2 * i + 1] = hi;
      } else {
        reinterpret_cast<uint16_t *>(dst)[2 * i] = (uint16_t)lo;
        reinterpret_cast<uint16_t *>(dst)[2 * i + 1] = (uint16_t)hi;
      }
    }
  }
}

// ------------------------------------------------------------------ encode
// Widen one source element to float (exact); `sign` receives the source sign
// bit (kept separately because NaN sign is not preserved by every widening).
template <int SRC>
__device__ __forceinline__ float widen(uint32_t raw, uint32_t &sign) {
  if constexpr (SRC == FP8B200_F32) { sign = raw & 0x80000000u; return u2f(raw); }
  else if constexpr (SRC == FP8B200_BF16) { sign = (raw & 0x8000u) << 16; return u2f(raw << 16); }
  else { sign = (raw & 0x8000u) << 16; return __half2float(__ushort_as_half((unsigned short)raw)); }
}

// x86 multiply NaN rule (what CPU torch's `x * scale` yields): a NaN operand x
// is kept (sign included); a NaN created from non-NaN operands is negative.
__device__ __forceinline__ float mul_scale(float x, uint32_t &sign, float s) {
  const float r = __fmul_rn(x, s);
  if (is_nan_bits(f2u(r)) && !is_nan_bits(f2u(x)))
    sign = is_nan_bits(f2u(s)) ? (f2u(s) & 0x80000000u) : 0x80000000u;
  else if (!is_nan_bits(f2u(r)))
    sign = f2u(r) & 0x80000000u;
  return r;
}

template <int FMT>
__device__ __forceinline__ uint32_t cvt_pair(float lo, float hi) {
  uint16_t r;  // PTX puts the first source operand in the upper byte
  if constexpr (FMT == FP8B200_E4M3)
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// magnitude bits above which cvt.satfinite differs from CPU torch
template <int FMT> constexpr uint32_t special_threshold() {
  return FMT == FP8B200_E4M3 ? 0x43E80000u /* 464 */ : 0x476FFFFFu /* just below 61440 */;
}

template <int FMT>
__device__ __forceinline__ uint32_t special_code(uint32_t absb, uint32_t sign) {
  const uint32_t s = sign >> 24;
  if constexpr (FMT == FP8B200_E4M3) return s | 0x7Fu;
  else return s | (absb > 0x7F800000u ? 0x7Fu : 0x7Cu);
}

template <int SRC, int FMT>
__device__ __forceinline__ uint32_t encode_one(uint32_t raw, bool scaled, float s) {
  uint32_t sign;
  float x = widen<SRC>(raw, sign);
  if (scaled) x = mul_scale(x, sign, s);
  const uint32_t absb = f2u(x) & 0x7FFFFFFFu;
  if (absb > special_threshold<FMT>()) return special_code<FMT>(absb, sign);
  return cvt_pair<FMT>(x, 0.0f) & 0xFFu;
}

template <int SRC>
__device__ __forceinline__ uint32_t load_raw(const void *src, int64_t i) {
  if constexpr (SRC == FP8B200_F32) return reinterpret_cast<const uint32_t *>(src)[i];
  else return reinterpret_cast<const uint16_t *>(src)[i];
}

// One unit = 16 elements (64 or 32 input bytes) -> 16 output bytes.
template <int SRC>
struct EncIn { U8x32 a[SRC == FP8B200_F32 ? 2 : 1]; };

template <int SRC>
__device__ __forceinline__ EncIn<SRC> load_enc(const uint8_t *in) {
  EncIn<SRC> e;
  e.a[0] = ld_u256(in);
  if constexpr (SRC == FP8B200_F32) e.a[1] = ld_u256(in + 32);
  return e;
}

template <int SRC, int FMT>
__device__ __forceinline__ void encode_unit(const EncIn<SRC> &e, uint8_t *out, bool scaled, float s) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  uint32_t raw[16];
  if constexpr (EB == 4) {
#pragma unroll
    for (int j = 0; j < 8; j++) { raw[j] = e.a[0].w[j]; raw[8 + j] = e.a[1].w[j]; }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++) { raw[2 * j] = e.a[0].w[j] & 0xFFFFu; raw[2 * j + 1] = e.a[0].w[j] >> 16; }
  }
  float x[16];
  uint32_t amax = 0;
#pragma unroll
  for (int i = 0; i < 16; i++) {
    uint32_t sg;
    x[i] = widen<SRC>(raw[i], sg);
    if (scaled) x[i] = __fmul_rn(x[i], s);
    amax = max(amax, f2u(x[i]) & 0x7FFFFFFFu);
  }
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; q++)
    o[q] = cvt_pair<FMT>(x[4 * q], x[4 * q + 1]) | (cvt_pair<FMT>(x[4 * q + 2], x[4 * q + 3]) << 16);
  if (amax > special_threshold<FMT>()) {  // rare: overflow, inf or NaN present
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const uint32_t c = encode_one<SRC, FMT>(raw[i], scaled, s);
      o[i >> 2] = (o[i >> 2] & ~(0xFFu << (8 * (i & 3)))) | (c << (8 * (i & 3)));
    }
  }
  st_u128(out, o[0], o[1], o[2], o[3]);
}

// Packed two-lane f32 arithmetic (sm_100 f32x2: one instruction for two
// IEEE round-to-nearest operations, bit-identical to two scalar ones).
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(unsigned long long v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long mul_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float ex2_approx_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max |x| bits (as f32 bit patterns) over one 16-value unit
template <int SRC>
__device__ __forceinline__ uint32_t unit_absmax(const EncIn<SRC> &e) {
  uint32_t m = 0, sg;
#pragma unroll
  for (int h = 0; h < (SRC == FP8B200_F32 ? 2 : 1); h++) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if constexpr (SRC == FP8B200_F32) m = max(m, e.a[h].w[j] & 0x7FFFFFFFu);
      else {
        m = max(m, f2u(widen<SRC>(e.a[h].w[j] & 0xFFFFu, sg)) & 0x7FFFFFFFu);
        m = max(m, f2u(widen<SRC>(e.a[h].w[j] >> 16, sg)) & 0x7FFFFFFFu);
      }
    }
  }
  return m;
}

// Per-row scale from the row's amax bits t: scale = fmax / amax (1 when amax
// is 0 or NaN), computed in double and rounded to float; inv = 1 / scale.
// Returns whether amax and the scale are finite (encode_unit_finite applies).
__device__ __forceinline__ int row_scale_of(uint32_t t, float fmax, float &scale, float *inv) {
  const double a = (double)u2f(t);
  const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
  scale = (float)sd;
  *inv = (float)(1.0 / sd);
  return t < 0x7F800000u && __float_as_uint(scale) < 0x7F800000u;
}

// encode_unit for rows whose amax and scale are finite: |x * s| <= fmax (1 +
// 2^-23) for every element, so no element needs the fix-up and the products
// run as f32x2 pairs (the same IEEE roundings as one multiply each).
template <int SRC, int FMT>
__device__ __forceinline__ void encode_unit_finite(const EncIn<SRC> &e, uint8_t *out, float s) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  float x[16];
  const unsigned long long ss = f2pack(s, s);
#pragma unroll
  for (int j = 0; j < 8; j++) {
    uint32_t sg;
    float lo, hi;
    if constexpr (EB == 4) { lo = u2f(e.a[j >> 2].w[2 * (j & 3)]); hi = u2f(e.a[j >> 2].w[2 * (j & 3) + 1]); }
    else { lo = widen<SRC>(e.a[0].w[j] & 0xFFFFu, sg); hi = widen<SRC>(e.a[0].w[j] >> 16, sg); }
    f2unpack(mul_f32x2(f2pack(lo, hi), ss), x[2 * j], x[2 * j + 1]);
  }
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; q++)
    o[q] = cvt_pair<FMT>(x[4 * q], x[4 * q + 1]) | (cvt_pair<FMT>(x[4 * q + 2], x[4 * q + 3]) << 16);
  st_u128(out, o[0], o[1], o[2], o[3]);
}

// vec: source 32-byte and destination 16-byte aligned; otherwise every
// element goes through the scalar loop (still on the GPU).
template <int SRC, int FMT>
__global__ void __launch_bounds__(kThreads)
encode_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t n, int64_t nunits,
              const float *__restrict__ scale) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  const bool scaled = scale != nullptr;
  const float s = scaled ? __ldg(scale) : 1.0f;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int U = SRC == FP8B200_F32 ? 2 : kUnroll;  // 32 or 64 KiB of loads in flight per CTA step
  for (; u + (U - 1) * nthreads < nunits; u += U * nthreads) {
    EncIn<SRC> in[U];
#pragma unroll
    for (int j = 0; j < U; j++) in[j] = load_enc<SRC>(src + (u + j * nthreads) * 16 * EB);
#pragma unroll
    for (int j = 0; j < U; j++) encode_unit<SRC, FMT>(in[j], dst + (u + j * nthreads) * 16, scaled, s);
  }
  for (; u < nunits; u += nthreads) encode_unit<SRC, FMT>(load_enc<SRC>(src + u * 16 * EB), dst + u * 16, scaled, s);
  for (int64_t i = nunits * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += nthreads)
    dst[i] = (uint8_t)encode_one<SRC, FMT>(load_raw<SRC>(src, i), scaled, s);
}

// Bulk-copy pipeline for the encoders (same ring structure as the decoders):
// chunks of 4096 elements (16 KiB of f32 or 8 KiB of 16-bit input) encode to
// 4 KiB of fp8; each thread step converts 4 elements with one shared load.
constexpr int kEncElems = 4096;

template <int SRC>
struct Enc {
  static constexpr int kEB = SRC == FP8B200_F32 ? 4 : 2;
  static constexpr int kIn = kEncElems * kEB;
  static constexpr int kOut = kEncElems;
  static constexpr int kSteps = kEncElems / 4 / kDecThreads;
  static constexpr int kSmem = kStages * (kIn + kOut) + 64;
};

template <int SRC, int FMT>
__device__ __forceinline__ uint32_t encode4(const uint8_t *in, int idx, bool scaled, float s) {
  uint32_t raw[4];
  if constexpr (SRC == FP8B200_F32) {
    const uint4 v = reinterpret_cast<const uint4 *>(in)[idx];
    raw[0] = v.x; raw[1] = v.y; raw[2] = v.z; raw[3] = v.w;
  } else {
    const uint2 v = reinterpret_cast<const uint2 *>(in)[idx];
    raw[0] = v.x & 0xFFFFu; raw[1] = v.x >> 16; raw[2] = v.y & 0xFFFFu; raw[3] = v.y >> 16;
  }
  float x[4];
  uint32_t amax = 0, sg;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    x[i] = widen<SRC>(raw[i], sg);
    if (scaled) x[i] = __fmul_rn(x[i], s);
    amax = max(amax, f2u(x[i]) & 0x7FFFFFFFu);
  }
  uint32_t o = cvt_pair<FMT>(x[0], x[1]) | (cvt_pair<FMT>(x[2], x[3]) << 16);
  if (amax > special_threshold<FMT>()) {  // rare: overflow, inf or NaN present
    o = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) o |= encode_one<SRC, FMT>(raw[i], scaled, s) << (8 * i);
  }
  return o;
}

// Scale of a per-tensor quantisation from the amax bits left by amax_kernel:
// fmax / amax in double rounded to float (1 if amax is 0 or NaN); block 0
// also publishes {scale, 1/scale} to scale_out.
__device__ __forceinline__ float scale_from_amax(const uint32_t *amax_bits, float fmax, float *scale_out) {
  const double a = (double)u2f(__ldg(amax_bits));
  const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    scale_out[0] = (float)sd;
    scale_out[1] = (float)(1.0 / sd);
  }
  return (float)sd;
}

// scale: multiply by *scale; or amax_bits: the scale of a per-tensor
// quantisation (scale_from_amax); neither: plain encode.
template <int SRC, int FMT>
__global__ void __launch_bounds__(kDecThreads)
encode_bulk_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t n,
                   const float *__restrict__ scale, const uint32_t *__restrict__ amax_bits, float fmax,
                   float *__restrict__ scale_out) {
  using C = Enc<SRC>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint8_t *in_ring = smem_raw;
  uint8_t *out_ring = in_ring + kStages * C::kIn;
  uint64_t *bar = reinterpret_cast<uint64_t *>(out_ring + kStages * C::kOut);
  const int64_t nch = n / kEncElems;
  // A per-tensor quantisation reads its input twice (amax pass, then this
  // encode). Walking the chunks last-to-first here starts on the part the
  // amax pass read most recently, which is still in L2; `at` maps the
  // walk position to the chunk (a bijection of [0, nch)).
  const bool rev = amax_bits != nullptr;
  auto at = [&](int64_t c) { return rev ? nch - 1 - c : c; };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar + i)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_prefetch_l2(src + at(c) * C::kIn, C::kIn);
    }
  }
  pdl_launch_dependents();
  pdl_wait_prior();  // nothing in global memory is read or written before this (the L2 prefetch above excepted)
  const bool scaled = scale != nullptr || amax_bits != nullptr;
  const float s = amax_bits ? scale_from_amax(amax_bits, fmax, scale_out) : scale ? __ldg(scale) : 1.0f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_load(smem_addr(in_ring + i * C::kIn), src + at(c) * C::kIn, C::kIn, smem_addr(bar + i));
    }
  }
  __syncthreads();
  bool failed = false;
  for (int64_t i = 0;; i++) {
    const int64_t c = blockIdx.x + i * gridDim.x;
    if (c >= nch) break;
    const int st = (int)(i % kStages);
    const uint32_t ph = (uint32_t)((i / kStages) & 1);
    int timed_out = 0;
    for (long long k = 0; !mbar_try(smem_addr(bar + st), ph);)
      if (++k > kBulkSpinLimit) { timed_out = 1; break; }
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) atomicExch(&g_bulk_status, 1);
      failed = true;
      break;
    }
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kStages - 1) : "memory");
    __syncthreads();
    const uint8_t *in = in_ring + st * C::kIn;
    uint32_t *out = reinterpret_cast<uint32_t *>(out_ring + st * C::kOut);
#pragma unroll
    for (int j = 0; j < C::kSteps; j++) {
      const int idx = threadIdx.x + j * kDecThreads;
      out[idx] = encode4<SRC, FMT>(in, idx, scaled, s);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + at(c) * C::kOut),
                   "r"(smem_addr(out)), "r"(C::kOut)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      const int64_t c2 = blockIdx.x + (i + kStages) * gridDim.x;
      if (c2 < nch) bulk_load(smem_addr(in_ring + st * C::kIn), src + at(c2) * C::kIn, C::kIn, smem_addr(bar + st));
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (failed && threadIdx.x == 0) drain_loads();  // loads issued before the timeout may still be landing
  if (blockIdx.x == gridDim.x - 1)
    for (int64_t e = nch * kEncElems + threadIdx.x; e < n; e += kDecThreads)
      dst[e] = (uint8_t)encode_one<SRC, FMT>(load_raw<SRC>(src, e), scaled, s);
}

// ------------------------------------------------------------------ fp4 encode
// The reference's nearest-of-8 threshold encoder (shaders/fp8_matmul.metal:
// 88-102): not round-to-nearest-even at ties (0.25 -> 0.5, 1.25 -> 1.5), NaN
// -> +6, -0.0 -> +0. Element 2i goes to the low nibble (:271-273).
// The threshold chain v < 0.25 -> 0, < 0.75 -> 1, < 1.25 -> 2, < 1.75 -> 3,
// < 2.5 -> 4, < 3.5 -> 5, < 5 -> 6, else 7 (sign bit from v < 0, so NaN and
// -0 give positive codes) on the float's bits: the e2m1 values from 1.0 up
// (1, 1.5, 2, 3, 4, 6) are the floats with one mantissa bit, so adding half
// of their spacing (float bit 21) and truncating rounds |v| half up, and
// (bits >> 22) - 252 numbers them 2..7 (8.0 and above, inf and NaN clamp to
// 7); the two compares supply codes 1 ([0.25, 0.75)) and 2 ([0.75, 1)).
// Equal to the chain for all 2^32 float bit patterns (checked exhaustively).
__device__ __forceinline__ uint32_t fp4_code(float v) {
  const uint32_t sign = (v < 0.0f) ? 8u : 0u;
  const uint32_t m = __float_as_uint(v) & 0x7FFFFFFFu;
  const int low = (int)(m >= 0x3E800000u) + (int)(m >= 0x3F400000u);
  const int c = min(max((int)((m + 0x00200000u) >> 22) - 252, low), 7);
  return sign | (uint32_t)c;
}

// Packed byte (lo in the low nibble) from cvt.rn.satfinite.e2m1x2. Over all
// 2^32 float inputs it differs from fp4_code only at +-0.25, +-1.25, +-2.5,
// +-5 (round-to-nearest-even takes the lower neighbour at these ties; the
// reference thresholds take the upper) and at -0 (sign kept; the reference
// gives +0); NaN and inf already agree. Callers add +0.0 first (-0 becomes
// +0, every other value is unchanged) and repair the ties: a tie is a
// rounding boundary, so the code of the next float up in magnitude (bits + 1)
// differs from it, and at a tie that code is the reference's. Where the two
// conversions differ the value is either such a tie or one ulp below a tie
// that rounds up; only the former has its low 21 bits clear, so those
// nibbles take the next-up code (fp4_fix_ties). Checked against the
// thresholds on the device for all 2^32 inputs.
__device__ __forceinline__ uint32_t fp4x2_cvt(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float fp4_next_up(float x) { return __uint_as_float(__float_as_uint(x) + 1u); }

// o, up: packed codes of x[0..N) and of their next-up floats; returns o with
// the nibbles of exact ties (low 21 bits clear, finite) taken from up.
template <int N>
__device__ __forceinline__ uint32_t fp4_fix_ties(uint32_t o, uint32_t up, const float (&x)[N]) {
  uint32_t m = 0;
#pragma unroll
  for (int e = 0; e < N; e++) {
    const uint32_t b = __float_as_uint(x[e]);
    if ((b & 0x1FFFFFu) == 0u && (b & 0x7F800000u) != 0x7F800000u) m |= 0xFu << (4 * e);
  }
  return (o & ~m) | (up & m);
}

template <int SRC>
__device__ __forceinline__ float load_elem(const void *src, int64_t i) {
  uint32_t sg;
  return widen<SRC>(load_raw<SRC>(src, i), sg);
}

// One unit = 32 elements -> 16 packed bytes; vec units need a 32-byte
// aligned source and a 16-byte aligned destination.
template <int SRC>
__global__ void __launch_bounds__(kThreads)
fp4_encode_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t npairs, int64_t nunits,
                  const float *__restrict__ scale) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  const bool scaled = scale != nullptr;
  const float s = scaled ? __ldg(scale) : 1.0f;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < nunits; u += nthreads) {
    const uint8_t *in = src + u * 32 * EB;
    uint32_t o[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int h = 0; h < EB; h++) {  // 32-byte chunks: 8 (f32) or 16 (16-bit) elements each
      const U8x32 a = ld_u256(in + 32 * h);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        uint32_t sg;
        if constexpr (EB == 4) {
          float x = widen<SRC>(a.w[j], sg);
          if (scaled) x = __fmul_rn(x, s);
          const int e = 8 * h + j;
          o[e >> 3] |= fp4_code(x) << (4 * (e & 7));
        } else {
          float x0 = widen<SRC>(a.w[j] & 0xFFFFu, sg), x1 = widen<SRC>(a.w[j] >> 16, sg);
          if (scaled) { x0 = __fmul_rn(x0, s); x1 = __fmul_rn(x1, s); }
          const int e = 16 * h + 2 * j;
          o[e >> 3] |= (fp4_code(x0) | (fp4_code(x1) << 4)) << (4 * (e & 7));
        }
      }
    }
    st_u128(dst + u * 16, o[0], o[1], o[2], o[3]);
  }
  for (int64_t p = nunits * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < npairs; p += nthreads) {
    float lo = load_elem<SRC>(src, 2 * p), hi = load_elem<SRC>(src, 2 * p + 1);
    if (scaled) { lo = __fmul_rn(lo, s); hi = __fmul_rn(hi, s); }
    dst[p] = (uint8_t)(fp4_code(lo) | (fp4_code(hi) << 4));
  }
}

// FP4 encode in the bulk-copy pipeline of the fp8 encoders: chunks of
// kEncElems elements (16 or 8 KiB of input) encode to kEncElems / 2 packed
// bytes; each thread step reads 16 bytes of shared memory (4 f32 or 8 16-bit
// values) and writes their 2 or 4 packed bytes. Scale options as for
// encode_bulk_kernel.
template <int SRC>
struct Fp4Enc {
  static constexpr int kEB = SRC == FP8B200_F32 ? 4 : 2;
  static constexpr int kPer = 16 / kEB;  // elements per thread step
  static constexpr int kIn = kEncElems * kEB;
  static constexpr int kOut = kEncElems / 2;
  static constexpr int kSteps = kEncElems / kPer / kDecThreads;
  static constexpr int kSmem = kStages * (kIn + kOut) + 64;
};

template <int SRC>
__global__ void __launch_bounds__(kDecThreads)
fp4_encode_bulk_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t n,
                       const float *__restrict__ scale, const uint32_t *__restrict__ amax_bits, float fmax,
                       float *__restrict__ scale_out) {
  using C = Fp4Enc<SRC>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint8_t *in_ring = smem_raw;
  uint8_t *out_ring = in_ring + kStages * C::kIn;
  uint64_t *bar = reinterpret_cast<uint64_t *>(out_ring + kStages * C::kOut);
  const int64_t nch = n / kEncElems;
  // A per-tensor quantisation reads its input twice (amax pass, then this
  // encode). Walking the chunks last-to-first here starts on the part the
  // amax pass read most recently, which is still in L2; `at` maps the
  // walk position to the chunk (a bijection of [0, nch)).
  const bool rev = amax_bits != nullptr;
  auto at = [&](int64_t c) { return rev ? nch - 1 - c : c; };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar + i)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_prefetch_l2(src + at(c) * C::kIn, C::kIn);
    }
  }
  pdl_launch_dependents();
  pdl_wait_prior();  // nothing in global memory is read or written before this (the L2 prefetch above excepted)
  const bool scaled = scale != nullptr || amax_bits != nullptr;
  const float s = amax_bits ? scale_from_amax(amax_bits, fmax, scale_out) : scale ? __ldg(scale) : 1.0f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      const int64_t c = blockIdx.x + (int64_t)i * gridDim.x;
      if (c < nch) bulk_load(smem_addr(in_ring + i * C::kIn), src + at(c) * C::kIn, C::kIn, smem_addr(bar + i));
    }
  }
  __syncthreads();
  bool failed = false;
  for (int64_t i = 0;; i++) {
    const int64_t c = blockIdx.x + i * gridDim.x;
    if (c >= nch) break;
    const int st = (int)(i % kStages);
    const uint32_t ph = (uint32_t)((i / kStages) & 1);
    int timed_out = 0;
    for (long long k = 0; !mbar_try(smem_addr(bar + st), ph);)
      if (++k > kBulkSpinLimit) { timed_out = 1; break; }
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) atomicExch(&g_bulk_status, 1);
      failed = true;
      break;
    }
    if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kStages - 1) : "memory");
    __syncthreads();
    const uint4 *in = reinterpret_cast<const uint4 *>(in_ring + st * C::kIn);
    uint8_t *out = out_ring + st * C::kOut;
    const unsigned long long ss = f2pack(s, s);
#pragma unroll
    for (int j = 0; j < C::kSteps; j++) {
      const int idx = threadIdx.x + j * kDecThreads;
      const uint4 v = in[idx];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      constexpr int NX = C::kPer;  // 4 (f32) or 8 (16-bit) values
      float x[NX];
      uint32_t sg;
#pragma unroll
      for (int q = 0; q < NX / 2; q++) {
        float a, b;
        if constexpr (SRC == FP8B200_F32) { a = u2f(w[2 * q]); b = u2f(w[2 * q + 1]); }
        else { a = widen<SRC>(w[q] & 0xFFFFu, sg); b = widen<SRC>(w[q] >> 16, sg); }
        unsigned long long ab = f2pack(a, b);
        if (scaled) ab = mul_f32x2(ab, ss);
        f2unpack(add_f32x2(ab, 0ull), a, b);  // + 0.0: -0 -> +0
        x[2 * q] = a;
        x[2 * q + 1] = b;
      }
      uint32_t o = 0, up = 0;
#pragma unroll
      for (int q = 0; q < NX / 2; q++) {
        o |= fp4x2_cvt(x[2 * q], x[2 * q + 1]) << (8 * q);
        up |= fp4x2_cvt(fp4_next_up(x[2 * q]), fp4_next_up(x[2 * q + 1])) << (8 * q);
      }
      if (o != up) o = fp4_fix_ties<NX>(o, up, x);  // a value at or one ulp below a rounding boundary
      if constexpr (SRC == FP8B200_F32) reinterpret_cast<uint16_t *>(out)[idx] = (uint16_t)o;
      else reinterpret_cast<uint32_t *>(out)[idx] = o;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + at(c) * C::kOut),
                   "r"(smem_addr(out)), "r"(C::kOut)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      const int64_t c2 = blockIdx.x + (i + kStages) * gridDim.x;
      if (c2 < nch) bulk_load(smem_addr(in_ring + st * C::kIn), src + at(c2) * C::kIn, C::kIn, smem_addr(bar + st));
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (failed && threadIdx.x == 0) drain_loads();  // loads issued before the timeout may still be landing
  if (blockIdx.x == gridDim.x - 1)
    for (int64_t p = nch * (kEncElems / 2) + threadIdx.x; p < n / 2; p += kDecThreads) {
      float lo = load_elem<SRC>(src, 2 * p), hi = load_elem<SRC>(src, 2 * p + 1);
      if (scaled) { lo = __fmul_rn(lo, s); hi = __fmul_rn(hi, s); }
      dst[p] = (uint8_t)(fp4_code(lo) | (fp4_code(hi) << 4));
    }
}

// ------------------------------------------------------------------ amax / quantize
// max |x| as float bits (NaN sorts above inf, so a NaN anywhere wins).
// nunits: 32-byte chunks read vectorised (0 for an unaligned source); the
// remaining elements go through the scalar loop.
template <int SRC>
__global__ void __launch_bounds__(kThreads)
amax_kernel(const uint8_t *__restrict__ src, int64_t n, int64_t nunits, uint32_t *__restrict__ amax_out) {
  pdl_launch_dependents();
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  constexpr int PER = 32 / EB;
  uint32_t m = 0, sg;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  auto fold = [&](const U8x32 &a) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
      if constexpr (EB == 4) m = max(m, f2u(widen<SRC>(a.w[j], sg)) & 0x7FFFFFFFu);
      else {
        m = max(m, f2u(widen<SRC>(a.w[j] & 0xFFFFu, sg)) & 0x7FFFFFFFu);
        m = max(m, f2u(widen<SRC>(a.w[j] >> 16, sg)) & 0x7FFFFFFFu);
      }
    }
  };
  // four 32-byte loads in flight per thread, the last round predicated (a
  // unit past the end reads as zeros, which leave the max unchanged), so no
  // thread ends on a chain of one-load rounds
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < nunits; u += 4 * nthreads) {
    U8x32 a[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int64_t v = u + k * nthreads;
      if (v < nunits) a[k] = ld_u256(src + v * 32);
      else a[k] = U8x32{};
    }
#pragma unroll
    for (int k = 0; k < 4; k++) fold(a[k]);
  }
  for (int64_t i = nunits * PER + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += nthreads)
    m = max(m, f2u(load_elem<SRC>(src, i)) & 0x7FFFFFFFu);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t r = threadIdx.x < blockDim.x / 32 ? warp_max[threadIdx.x] : 0u;
    r = __reduce_max_sync(0xFFFFFFFFu, r);
    // the input was final before clear_amax_kernel started; amax_out is
    // cleared by that kernel, so wait for it before the first global write
    pdl_wait_prior();
    if (threadIdx.x == 0 && r) atomicMax(amax_out, r);
  }
}

// Clears the amax word of a per-tensor quantisation. Launched without the
// programmatic attribute, so it starts after all earlier work in the stream
// (the input is final from then on); the amax reduction after it is a
// programmatic dependent launch that streams the input meanwhile and waits
// for this kernel only before its atomicMax.
__global__ void clear_amax_kernel(uint32_t *__restrict__ amax_out) {
  pdl_launch_dependents();
  if (threadIdx.x == 0) *amax_out = 0u;
}

// scale = fmax/amax (1 if amax is 0 or NaN), computed in double as the
// reference does on the host (fp8_mps_native.py:107-108, :119).
__global__ void quant_scale_kernel(const uint32_t *__restrict__ amax_bits, float fmax, float *__restrict__ scale_out) {
  const double a = (double)u2f(*amax_bits);
  const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
  scale_out[0] = (float)sd;
  scale_out[1] = (float)(1.0 / sd);
}

// ------------------------------------------------------------------ per-row quantize
// One CTA per row (grid-stride over rows): pass 1 reduces max|x| over the
// row, pass 2 re-reads the row (from L2: a row is at most a few tens of KiB)
// and encodes x * scale_r with scale_r = fmax / amax_r computed in double,
// exactly the reference's per-tensor quantize (fp8_mps_native.py:101-120)
// applied to each row; inv_scale[r] = 1 / scale_r. Rows whose amax is 0 or
// NaN use scale 1.
constexpr int kRowThreads = 256;

template <int SRC, int FMT>
__global__ void __launch_bounds__(kRowThreads)
quantize_rows_kernel(const uint8_t *__restrict__ src, int64_t ld_src, uint8_t *__restrict__ dst, int64_t ld_dst,
                     int64_t rows, int64_t cols, int vec, float fmax, float *__restrict__ inv_scale) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  __shared__ uint32_t warp_max[kRowThreads / 32];
  __shared__ float row_scale;
  const int64_t nchunks = vec ? cols / 16 : 0;  // 16-element chunks read 32 bytes at a time
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint8_t *rs = src + r * ld_src * EB;
    uint8_t *rd = dst + r * ld_dst;
    uint32_t m = 0, sg;
    for (int64_t c = threadIdx.x; c < nchunks; c += kRowThreads) {
#pragma unroll
      for (int h = 0; h < EB / 2; h++) {
        const U8x32 a = ld_u256(rs + c * 16 * EB + 32 * h);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          if constexpr (EB == 4) m = max(m, f2u(widen<SRC>(a.w[j], sg)) & 0x7FFFFFFFu);
          else {
            m = max(m, f2u(widen<SRC>(a.w[j] & 0xFFFFu, sg)) & 0x7FFFFFFFu);
            m = max(m, f2u(widen<SRC>(a.w[j] >> 16, sg)) & 0x7FFFFFFFu);
          }
        }
      }
    }
    for (int64_t i = nchunks * 16 + threadIdx.x; i < cols; i += kRowThreads)
      m = max(m, f2u(load_elem<SRC>(rs, i)) & 0x7FFFFFFFu);
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = 0;
      for (int w = 0; w < kRowThreads / 32; w++) t = max(t, warp_max[w]);
      const double a = (double)u2f(t);
      const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
      row_scale = (float)sd;
      inv_scale[r] = (float)(1.0 / sd);
    }
    __syncthreads();
    const float s = row_scale;
    for (int64_t c = threadIdx.x; c < nchunks; c += kRowThreads)
      encode_unit<SRC, FMT>(load_enc<SRC>(rs + c * 16 * EB), rd + c * 16, true, s);
    for (int64_t i = nchunks * 16 + threadIdx.x; i < cols; i += kRowThreads)
      rd[i] = (uint8_t)encode_one<SRC, FMT>(load_raw<SRC>(rs, i), true, s);
    __syncthreads();  // warp_max / row_scale are reused by the next row
  }
}

// Register-resident variant for rows of at most KV * 256 * 16 elements whose
// rows start 32-byte aligned (source) and 16-byte aligned (destination):
// each thread loads its KV 16-element units once, keeps them in registers
// through the amax reduction and encodes from registers, so every row is
// read from HBM exactly once. Same results as quantize_rows_kernel.
template <int SRC, int FMT, int KV>
__global__ void __launch_bounds__(kRowThreads)
quantize_rows_reg_kernel(const uint8_t *__restrict__ src, int64_t ld_src, uint8_t *__restrict__ dst, int64_t ld_dst,
                         int64_t rows, int64_t cols, float fmax, float *__restrict__ inv_scale) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  __shared__ uint32_t warp_max[kRowThreads / 32];
  __shared__ float row_scale;
  __shared__ int row_finite;
  const int nunits = (int)(cols / 16);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint8_t *rs = src + r * ld_src * EB;
    uint8_t *rd = dst + r * ld_dst;
    EncIn<SRC> in[KV];
#pragma unroll
    for (int k = 0; k < KV; k++) {
      const int u = threadIdx.x + k * kRowThreads;
      if (u < nunits) in[k] = load_enc<SRC>(rs + (int64_t)u * 16 * EB);
    }
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < KV; k++)
      if (threadIdx.x + k * kRowThreads < nunits) m = max(m, unit_absmax<SRC>(in[k]));
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = 0;
      for (int w = 0; w < kRowThreads / 32; w++) t = max(t, warp_max[w]);
      float sc;
      row_finite = row_scale_of(t, fmax, sc, inv_scale + r);
      row_scale = sc;
    }
    __syncthreads();
    const float s = row_scale;
    const bool finite = row_finite;
#pragma unroll
    for (int k = 0; k < KV; k++) {
      const int u = threadIdx.x + k * kRowThreads;
      if (u < nunits) {
        if (finite) encode_unit_finite<SRC, FMT>(in[k], rd + (int64_t)u * 16, s);
        else encode_unit<SRC, FMT>(in[k], rd + (int64_t)u * 16, true, s);
      }
    }
    __syncthreads();  // warp_max / row_scale are reused by the next row
  }
}

// Rows of at most 32 x KW units (16 values each; 4096 bf16 values at KW = 8)
// are quantised one row per warp: the whole row sits in the warp's
// registers, its amax is one warp reduction and no block barrier separates
// the load, reduce and encode steps, so the SM's other warps keep their rows'
// loads in flight meanwhile. Same results as quantize_rows_kernel.
template <int SRC, int FMT, int KW>
__global__ void __launch_bounds__(kRowThreads)
quantize_rows_warp_kernel(const uint8_t *__restrict__ src, int64_t ld_src, uint8_t *__restrict__ dst, int64_t ld_dst,
                          int64_t rows, int64_t cols, float fmax, float *__restrict__ inv_scale) {
  constexpr int EB = SRC == FP8B200_F32 ? 4 : 2;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (kRowThreads / 32);
  const int nunits = (int)(cols / 16);
  for (int64_t r = (int64_t)blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const uint8_t *rs = src + r * ld_src * EB;
    uint8_t *rd = dst + r * ld_dst;
    EncIn<SRC> in[KW];
#pragma unroll
    for (int k = 0; k < KW; k++) {
      const int u = lane + 32 * k;
      if (u < nunits) in[k] = load_enc<SRC>(rs + (int64_t)u * 16 * EB);
    }
    uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < KW; k++)
      if (lane + 32 * k < nunits) m = max(m, unit_absmax<SRC>(in[k]));
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    float s = 0.0f;
    int finite = 0;
    if (lane == 0) finite = row_scale_of(m, fmax, s, inv_scale + r);
    s = __shfl_sync(0xFFFFFFFFu, s, 0);
    finite = __shfl_sync(0xFFFFFFFFu, finite, 0);
#pragma unroll
    for (int k = 0; k < KW; k++) {
      const int u = lane + 32 * k;
      if (u < nunits) {
        if (finite) encode_unit_finite<SRC, FMT>(in[k], rd + (int64_t)u * 16, s);
        else encode_unit<SRC, FMT>(in[k], rd + (int64_t)u * 16, true, s);
      }
    }
  }
}

// ------------------------------------------------------------------ fused SiLU-gate quantize
// For a row [g | u] of 2F bf16 values (the output of a fused gate/up
// projection), y = bf16(bf16(silu(g)) * u) exactly as PyTorch's bf16 ops
// compute F.silu(g) * u (silu in float: x / (1 + exp(-x)), rounded; product
// in float, rounded), then y is quantised per row like quantize_rows_kernel.
// One CTA per row; y is kept in shared memory between the two passes, so the
// row is read from HBM once and the bf16 activation is never written.
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// bf16(silu(x)) for PyTorch's float formula x / (1 + expf(-x)) (expf, IEEE
// division). Fast path: __expf and __fdividef, whose float result is within a
// few tens of ulp of the formula for |x| <= 16; the rounding to bf16 agrees
// whenever the fast value is more than 64 ulp from a bf16 rounding midpoint
// (low 16 bits 0x8000). Otherwise, and for |x| > 16 or non-finite x, the
// formula itself is evaluated. The inputs are bf16, so the agreement is checked
// exhaustively (all 65536 gate values) against PyTorch on the device.
__device__ __forceinline__ float silu_bf16(float x) {
  if (fabsf(x) <= 16.0f) {
    const float s = __fdividef(x, 1.0f + __expf(-x));
    const int d = (int)(__float_as_uint(s) & 0xFFFFu) - 0x8000;
    if (d > 64 || d < -64) return bf16_round(s);
  }
  return bf16_round(x / (1.0f + expf(-x)));
}

__device__ __forceinline__ uint32_t silu_mul_bf16(uint32_t g, uint32_t u) {
  const float gf = u2f(g << 16), uf = u2f(u << 16);
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(silu_bf16(gf) * uf));
}

// Two bf16(silu(g)) * u products from packed bf16x2 words g and u. The fast
// silu value x * 1/(1 + 2^(-x log2 e)) comes from the hardware ex2 and rcp
// approximations (on |x| <= 16 neither sees a subnormal, so their
// flush-to-zero forms are exact-range safe) with paired f32x2 arithmetic; as
// in silu_bf16, the formula itself is evaluated whenever a value of the pair is
// within 64 ulp of a bf16 rounding midpoint (low 16 bits 0x7FC0..0x8040), or
// |x| > 16, or x is not finite. The product of two bf16 values is exact in
// float, so one bf16x2 multiply (round to nearest even, no contraction) equals
// PyTorch's float product rounded to bf16.
__device__ __forceinline__ uint32_t silu_mul_bf16x2(uint32_t g, uint32_t u) {
  const float x0 = u2f(g << 16), x1 = u2f(g & 0xFFFF0000u);
  const unsigned long long xx = f2pack(x0, x1);
  float t0, t1, d0, d1, s0, s1;
  f2unpack(mul_f32x2(xx, f2pack(-1.4426950408889634f, -1.4426950408889634f)), t0, t1);
  f2unpack(add_f32x2(f2pack(ex2_approx_ftz(t0), ex2_approx_ftz(t1)), f2pack(1.0f, 1.0f)), d0, d1);
  f2unpack(mul_f32x2(xx, f2pack(rcp_approx_ftz(d0), rcp_approx_ftz(d1))), s0, s1);
  const bool near0 = ((__float_as_uint(s0) - 0x7FC0u) & 0xFFFFu) <= 128u;
  const bool near1 = ((__float_as_uint(s1) - 0x7FC0u) & 0xFFFFu) <= 128u;
  if (!(fabsf(x0) <= 16.0f) || !(fabsf(x1) <= 16.0f) || near0 || near1) {  // rare
    s0 = x0 / (1.0f + expf(-x0));
    s1 = x1 / (1.0f + expf(-x1));
  }
  const __nv_bfloat162 s2 = __floats2bfloat162_rn(s0, s1);
  uint32_t y;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(y) : "r"(*reinterpret_cast<const uint32_t *>(&s2)), "r"(u));
  return y;
}

// Running max of |y| over bf16x2 words, NaN-propagating: for non-NaN values
// the result equals an integer max of the magnitude bits; any NaN makes the
// lane NaN (the row's scale then takes its NaN branch either way).
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t m, uint32_t y) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(y & 0x7FFF7FFFu));
  return r;
}

// Eight bf16 values (one 16-byte vector) -> eight fp8 codes of value * s,
// with the same results as encode_one (cvt pairs; per-element fix-up only
// when an overflow, inf or NaN is present).
template <int FMT>
__device__ __forceinline__ uint2 encode8_bf16(uint4 v, float s) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float x[8];
  uint32_t amax = 0;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    x[2 * q] = __fmul_rn(u2f(w[q] << 16), s);
    x[2 * q + 1] = __fmul_rn(u2f(w[q] & 0xFFFF0000u), s);
    amax = max(amax, max(f2u(x[2 * q]) & 0x7FFFFFFFu, f2u(x[2 * q + 1]) & 0x7FFFFFFFu));
  }
  uint32_t o[2];
#pragma unroll
  for (int h = 0; h < 2; h++)
    o[h] = cvt_pair<FMT>(x[4 * h], x[4 * h + 1]) | (cvt_pair<FMT>(x[4 * h + 2], x[4 * h + 3]) << 16);
  if (amax > special_threshold<FMT>()) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t c = encode_one<FP8B200_BF16, FMT>((w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu, true, s);
      o[i >> 2] = (o[i >> 2] & ~(0xFFu << (8 * (i & 3)))) | (c << (8 * (i & 3)));
    }
  }
  return make_uint2(o[0], o[1]);
}

// encode8_bf16 for a row whose amax and scale are finite: then every
// |value * s| <= fmax (1 + 2^-23), below the first value that rounds past the
// largest finite code, so the cvt pairs alone give CPU PyTorch's codes.
template <int FMT>
__device__ __forceinline__ uint2 encode8_bf16_finite(uint4 v, float s) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const unsigned long long ss = f2pack(s, s);
  float x[8];
#pragma unroll
  for (int q = 0; q < 4; q++) f2unpack(mul_f32x2(f2pack(u2f(w[q] << 16), u2f(w[q] & 0xFFFF0000u)), ss), x[2 * q], x[2 * q + 1]);
  return make_uint2(cvt_pair<FMT>(x[0], x[1]) | (cvt_pair<FMT>(x[2], x[3]) << 16),
                    cvt_pair<FMT>(x[4], x[5]) | (cvt_pair<FMT>(x[6], x[7]) << 16));
}

template <int FMT>
__global__ void __launch_bounds__(kRowThreads)
silu_mul_quantize_kernel(const uint16_t *__restrict__ gu, int64_t ld, uint8_t *__restrict__ dst, int64_t ld_dst,
                         int64_t rows, int64_t F, int vec, float fmax, float *__restrict__ inv_scale) {
  extern __shared__ __align__(16) uint16_t ybuf[];  // F bf16 values of the current row
  __shared__ uint32_t warp_max[kRowThreads / 32];
  __shared__ float row_scale;
  __shared__ int row_finite;  // amax and scale finite: the cvt pairs need no fix-up
  const int64_t nvec = vec ? F / 8 : 0;  // 8 bf16 per 16-byte vector
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t *g = gu + r * ld, *u = g + F;
    const uint4 *g4 = reinterpret_cast<const uint4 *>(g), *u4 = reinterpret_cast<const uint4 *>(u);
    uint32_t m2 = 0;  // |y| max of the low and high bf16 lanes
    int64_t v = threadIdx.x;
    for (; v + kRowThreads < nvec; v += 2 * kRowThreads) {  // two vectors of g and u in flight
      const uint4 ga = g4[v], ua = u4[v], gb = g4[v + kRowThreads], ub = u4[v + kRowThreads];
      const uint4 ya = make_uint4(silu_mul_bf16x2(ga.x, ua.x), silu_mul_bf16x2(ga.y, ua.y),
                                  silu_mul_bf16x2(ga.z, ua.z), silu_mul_bf16x2(ga.w, ua.w));
      const uint4 yb = make_uint4(silu_mul_bf16x2(gb.x, ub.x), silu_mul_bf16x2(gb.y, ub.y),
                                  silu_mul_bf16x2(gb.z, ub.z), silu_mul_bf16x2(gb.w, ub.w));
      const uint32_t ys[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
#pragma unroll
      for (int q = 0; q < 8; q++) m2 = absmax_bf16x2(m2, ys[q]);
      reinterpret_cast<uint4 *>(ybuf)[v] = ya;
      reinterpret_cast<uint4 *>(ybuf)[v + kRowThreads] = yb;
    }
    for (; v < nvec; v += kRowThreads) {
      const uint4 ga = g4[v], ua = u4[v];
      const uint4 ya = make_uint4(silu_mul_bf16x2(ga.x, ua.x), silu_mul_bf16x2(ga.y, ua.y),
                                  silu_mul_bf16x2(ga.z, ua.z), silu_mul_bf16x2(ga.w, ua.w));
      const uint32_t ys[4] = {ya.x, ya.y, ya.z, ya.w};
#pragma unroll
      for (int q = 0; q < 4; q++) m2 = absmax_bf16x2(m2, ys[q]);
      reinterpret_cast<uint4 *>(ybuf)[v] = ya;
    }
    for (int64_t i = nvec * 8 + threadIdx.x; i < F; i += kRowThreads) {
      const uint32_t y = silu_mul_bf16(g[i], u[i]);
      m2 = absmax_bf16x2(m2, y & 0xFFFFu);
      ybuf[i] = (uint16_t)y;
    }
    uint32_t m = max(m2 << 16, m2 & 0xFFFF0000u);
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t t = 0;
      for (int w = 0; w < kRowThreads / 32; w++) t = max(t, warp_max[w]);
      const double a = (double)u2f(t);
      const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
      row_scale = (float)sd;
      row_finite = t < 0x7F800000u && __float_as_uint((float)sd) < 0x7F800000u;
      inv_scale[r] = (float)(1.0 / sd);
    }
    __syncthreads();
    const float s = row_scale;
    uint8_t *rd = dst + r * ld_dst;
    if (row_finite)
      for (int64_t w = threadIdx.x; w < nvec; w += kRowThreads)  // 8 elements -> 8 bytes
        reinterpret_cast<uint2 *>(rd)[w] = encode8_bf16_finite<FMT>(reinterpret_cast<const uint4 *>(ybuf)[w], s);
    else
      for (int64_t w = threadIdx.x; w < nvec; w += kRowThreads)
        reinterpret_cast<uint2 *>(rd)[w] = encode8_bf16<FMT>(reinterpret_cast<const uint4 *>(ybuf)[w], s);
    for (int64_t i = nvec * 8 + threadIdx.x; i < F; i += kRowThreads)
      rd[i] = (uint8_t)encode_one<FP8B200_BF16, FMT>(ybuf[i], true, s);
    __syncthreads();  // ybuf / warp_max / row_scale are reused by the next row
  }
}

// ------------------------------------------------------------------ launch helpers
// Resident CTAs per SM for `kernel` (queried once per kernel and device),
// after raising its dynamic shared-memory limit when it needs more than 48 KiB.
// The cache is keyed by the kernel's address (many kernels share one type) and
// the dynamic shared memory, which the fused row kernels size per call.
int resident_per_sm(const void *kernel, int smem_bytes, int threads = kThreads) {
  struct Entry { const void *k; int dev; int smem; int n; };
  static Entry cache[128];
  static int used = 0;
  struct Limit { const void *k; int dev; int smem; };  // dynamic shared memory limit set so far
  static Limit limits[64];
  static int nlimits = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (smem_bytes > 48 * 1024) {  // the limit only ever rises, so every size seen before still launches
    int i = 0;
    while (i < nlimits && !(limits[i].k == kernel && limits[i].dev == dev)) i++;
    if (i == nlimits || limits[i].smem < smem_bytes) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      if (i == nlimits && nlimits < 64) limits[nlimits++] = Limit{kernel, dev, smem_bytes};
      else if (i < nlimits) limits[i].smem = smem_bytes;
    }
  }
  for (int i = 0; i < used; i++)
    if (cache[i].k == kernel && cache[i].dev == dev && cache[i].smem == smem_bytes) return cache[i].n;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem_bytes) != cudaSuccess || n < 1) n = 1;
  if (used < 128) cache[used++] = Entry{kernel, dev, smem_bytes, n};
  return n;
}

// Launch with programmatic stream serialization (see pdl_wait_prior).
template <typename... Params, typename... Args>
void launch_pdl(void (*kernel)(Params...), int grid, int threads, int smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int KIND>
void launch_decode(const void *src, void *dst, int64_t nbytes, int fmt, int odt, const float *scale, int mode,
                   cudaStream_t st) {
  constexpr int smem = Dec<KIND>::kSmem;
  const int per_sm = resident_per_sm((const void *)decode_bulk_kernel<KIND>, smem, kDecThreads);
  const int64_t nch = nbytes / Dec<KIND>::kIn;
  const int g = (int)std::max<int64_t>(1, std::min<int64_t>(nch, (int64_t)current_sm_count() * per_sm));
  launch_pdl(decode_bulk_kernel<KIND>, g, kDecThreads, smem, st, (const uint8_t *)src, (uint8_t *)dst, nbytes, fmt,
             odt, scale, mode);
}

// amax_bits (per-tensor quantisation): the kernel derives the scale from the
// amax and publishes it to scale_out; the bulk path only (callers check
// alignment first).
template <int SRC, int FMT>
void launch_encode(const void *src, void *dst, int64_t n, const float *scale, cudaStream_t st,
                   const uint32_t *amax_bits = nullptr, float fmax = 0.0f, float *scale_out = nullptr) {
  if (aligned16(src) && aligned16(dst)) {
    constexpr int smem = Enc<SRC>::kSmem;
    const int per_sm = resident_per_sm((const void *)encode_bulk_kernel<SRC, FMT>, smem, kDecThreads);
    const int64_t nch = n / kEncElems;
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>(nch, (int64_t)current_sm_count() * per_sm));
    launch_pdl(encode_bulk_kernel<SRC, FMT>, g, kDecThreads, smem, st, (const uint8_t *)src, (uint8_t *)dst, n, scale,
               amax_bits, fmax, scale_out);
  } else {  // unaligned: element-wise (the kernel's scalar loop)
    const int g = grid_for(std::max<int64_t>(n, 1), kThreads, resident_per_sm((const void *)encode_kernel<SRC, FMT>, 0));
    encode_kernel<SRC, FMT><<<g, kThreads, 0, st>>>((const uint8_t *)src, (uint8_t *)dst, n, 0, scale);
  }
}

void launch_encode_any(int sdt, int fmt, const void *src, void *dst, int64_t n, const float *scale, cudaStream_t st,
                       const uint32_t *amax_bits = nullptr, float fmax = 0.0f, float *scale_out = nullptr) {
  if (fmt == FP8B200_E4M3) {
    if (sdt == FP8B200_F32) launch_encode<FP8B200_F32, FP8B200_E4M3>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
    else if (sdt == FP8B200_BF16) launch_encode<FP8B200_BF16, FP8B200_E4M3>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
    else launch_encode<FP8B200_F16, FP8B200_E4M3>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
  } else {
    if (sdt == FP8B200_F32) launch_encode<FP8B200_F32, FP8B200_E5M2>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
    else if (sdt == FP8B200_BF16) launch_encode<FP8B200_BF16, FP8B200_E5M2>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
    else launch_encode<FP8B200_F16, FP8B200_E5M2>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
  }
}

template <int SRC>
void launch_fp4_encode(const void *src, void *dst, int64_t n, const float *scale, cudaStream_t st,
                       const uint32_t *amax_bits = nullptr, float fmax = 0.0f, float *scale_out = nullptr) {
  if (aligned16(src) && aligned16(dst)) {
    constexpr int smem = Fp4Enc<SRC>::kSmem;
    const int per_sm = resident_per_sm((const void *)fp4_encode_bulk_kernel<SRC>, smem, kDecThreads);
    const int64_t nch = n / kEncElems;
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>(nch, (int64_t)current_sm_count() * per_sm));
    launch_pdl(fp4_encode_bulk_kernel<SRC>, g, kDecThreads, smem, st, (const uint8_t *)src, (uint8_t *)dst, n, scale,
               amax_bits, fmax, scale_out);
    return;
  }
  const int64_t npairs = n / 2;
  const int64_t nunits = (aligned32(src) && aligned16(dst)) ? n / 32 : 0;
  const int g = grid_for(std::max<int64_t>(nunits ? nunits : npairs, 1), kThreads,
                         resident_per_sm((const void *)fp4_encode_kernel<SRC>, 0));
  fp4_encode_kernel<SRC><<<g, kThreads, 0, st>>>((const uint8_t *)src, (uint8_t *)dst, npairs, nunits, scale);
}

void launch_fp4_encode_any(int sdt, const void *src, void *dst, int64_t n, const float *scale, cudaStream_t st,
                           const uint32_t *amax_bits = nullptr, float fmax = 0.0f, float *scale_out = nullptr) {
  if (sdt == FP8B200_F32) launch_fp4_encode<FP8B200_F32>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
  else if (sdt == FP8B200_BF16) launch_fp4_encode<FP8B200_BF16>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
  else launch_fp4_encode<FP8B200_F16>(src, dst, n, scale, st, amax_bits, fmax, scale_out);
}

bool is_float_dtype(int dt) { return dt == FP8B200_F32 || dt == FP8B200_BF16 || dt == FP8B200_F16; }
bool is_fp8_dtype(int dt) { return dt == FP8B200_E4M3 || dt == FP8B200_E5M2; }

int check_scale_mode(int mode, const float *scale, int odt) {
  if (mode < FP8B200_SCALE_NONE || mode > FP8B200_SCALE_F16_REF)
    return set_error(FP8B200_EINVAL, "unknown scale_mode %d", mode);
  if (mode != FP8B200_SCALE_NONE && scale == nullptr)
    return set_error(FP8B200_EINVAL, "scale_mode %d needs a scale pointer", mode);
  if (mode == FP8B200_SCALE_F16_REF && odt != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "the f16 reference scale semantics produce float16 output only");
  return FP8B200_OK;
}

// Per-tensor quantisation, first half: clear the scratch and reduce max|x|
// into it; with `with_scale` also run the one-thread scale kernel (for the
// element-wise encoders; the bulk encoders derive the scale themselves).
int launch_amax_and_scale(const void *src, int src_dtype, int64_t n, float fmax, float *scale_out,
                          uint32_t *amax_scratch, cudaStream_t st, bool with_scale = true) {
  clear_amax_kernel<<<1, 32, 0, st>>>(amax_scratch);
  count_launch();
  if (int rc = check_launch("quantize amax clear")) return rc;
  if (n > 0) {
    const int eb = src_dtype == FP8B200_F32 ? 4 : 2;
    const int64_t nunits = aligned32(src) ? (n * eb) / 32 : 0;
    // one wave: as many CTAs as fit on the SMs at once (the f32 variant holds
    // twice the registers of the 16-bit ones, so fewer CTAs fit)
    const void *k = src_dtype == FP8B200_F32    ? (const void *)amax_kernel<FP8B200_F32>
                    : src_dtype == FP8B200_BF16 ? (const void *)amax_kernel<FP8B200_BF16>
                                                : (const void *)amax_kernel<FP8B200_F16>;
    const int g = grid_for(std::max<int64_t>(nunits ? nunits : n, 1), kThreads, resident_per_sm(k, 0));
    const uint8_t *s = (const uint8_t *)src;
    if (src_dtype == FP8B200_F32) launch_pdl(amax_kernel<FP8B200_F32>, g, kThreads, 0, st, s, n, nunits, amax_scratch);
    else if (src_dtype == FP8B200_BF16) launch_pdl(amax_kernel<FP8B200_BF16>, g, kThreads, 0, st, s, n, nunits, amax_scratch);
    else launch_pdl(amax_kernel<FP8B200_F16>, g, kThreads, 0, st, s, n, nunits, amax_scratch);
    count_launch();
    if (int rc = check_launch("quantize amax")) return rc;
  }
  if (!with_scale) return FP8B200_OK;
  quant_scale_kernel<<<1, 1, 0, st>>>(amax_scratch, fmax, scale_out);
  count_launch();
  return check_launch("quantize scale");
}

}  // namespace
}  // namespace fp8b200

using namespace fp8b200;

extern "C" int fp8b200_encode_fp8(const void *src, int src_dtype, void *dst, int fp8_dtype, int64_t n,
                                  const float *scale, void *stream) {
  if (n < 0) return set_error(FP8B200_EINVAL, "negative element count");
  if (!is_float_dtype(src_dtype)) return set_error(FP8B200_EINVAL, "encode: source dtype %d is not f32/bf16/f16", src_dtype);
  if (!is_fp8_dtype(fp8_dtype)) return set_error(FP8B200_EINVAL, "encode: target dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (n == 0) return FP8B200_OK;
  if (!src || !dst) return set_error(FP8B200_EINVAL, "encode: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  launch_encode_any(src_dtype, fp8_dtype, src, dst, n, scale, (cudaStream_t)stream);
  count_launch();
  return check_launch("fp8 encode");
}

extern "C" int fp8b200_decode_fp8(const void *src, int fp8_dtype, void *dst, int out_dtype, int64_t n,
                                  const float *scale, int scale_mode, void *stream) {
  if (n < 0) return set_error(FP8B200_EINVAL, "negative element count");
  if (!is_fp8_dtype(fp8_dtype)) return set_error(FP8B200_EINVAL, "decode: source dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (!is_float_dtype(out_dtype)) return set_error(FP8B200_EINVAL, "decode: output dtype %d is not f32/bf16/f16", out_dtype);
  if (int rc = check_scale_mode(scale_mode, scale, out_dtype)) return rc;
  if (n == 0) return FP8B200_OK;
  if (!src || !dst) return set_error(FP8B200_EINVAL, "decode: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (aligned16(src) && aligned16(dst)) {
    if (out_dtype == FP8B200_F32) launch_decode<DEC_FP8_32>(src, dst, n, fp8_dtype, out_dtype, scale, scale_mode, st);
    else launch_decode<DEC_FP8_16>(src, dst, n, fp8_dtype, out_dtype, scale, scale_mode, st);
  } else {
    const int g = grid_for(n, kThreads, 4);
    decode_scalar_kernel<<<g, kThreads, 0, st>>>((const uint8_t *)src, (uint8_t *)dst, n, 0, fp8_dtype, out_dtype,
                                                 scale, scale_mode);
  }
  count_launch();
  return check_launch("fp8 decode");
}

extern "C" int fp8b200_decode_fp4(const void *src, int64_t nbytes, void *dst, int out_dtype, const float *scale,
                                  int scale_mode, void *stream) {
  if (nbytes < 0) return set_error(FP8B200_EINVAL, "negative byte count");
  if (!is_float_dtype(out_dtype)) return set_error(FP8B200_EINVAL, "fp4 decode: output dtype %d is not f32/bf16/f16", out_dtype);
  if (int rc = check_scale_mode(scale_mode, scale, out_dtype)) return rc;
  if (nbytes == 0) return FP8B200_OK;
  if (!src || !dst) return set_error(FP8B200_EINVAL, "fp4 decode: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (aligned16(src) && aligned16(dst)) {
    if (out_dtype == FP8B200_F32) launch_decode<DEC_FP4_32>(src, dst, nbytes, 0, out_dtype, scale, scale_mode, st);
    else launch_decode<DEC_FP4_16>(src, dst, nbytes, 0, out_dtype, scale, scale_mode, st);
  } else {
    const int g = grid_for(nbytes, kThreads, 4);
    decode_scalar_kernel<<<g, kThreads, 0, st>>>((const uint8_t *)src, (uint8_t *)dst, nbytes, 1, 0, out_dtype,
                                                 scale, scale_mode);
  }
  count_launch();
  return check_launch("fp4 decode");
}

extern "C" int fp8b200_quantize_fp8(const void *src, int src_dtype, void *dst, int fp8_dtype, int64_t n,
                                    float *scale_out, uint32_t *amax_scratch, void *stream) {
  if (n < 0) return set_error(FP8B200_EINVAL, "negative element count");
  if (!is_float_dtype(src_dtype)) return set_error(FP8B200_EINVAL, "quantize: source dtype %d is not f32/bf16/f16", src_dtype);
  if (!is_fp8_dtype(fp8_dtype)) return set_error(FP8B200_EINVAL, "quantize: target dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (!scale_out || !amax_scratch) return set_error(FP8B200_EINVAL, "quantize: null scale/scratch pointer");
  if (n > 0 && (!src || !dst)) return set_error(FP8B200_EINVAL, "quantize: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const float fmax = fp8_dtype == FP8B200_E4M3 ? 448.0f : 57344.0f;
  const bool bulk = n > 0 && aligned16(src) && aligned16(dst);  // the encoder derives the scale from the amax
  if (int rc = launch_amax_and_scale(src, src_dtype, n, fmax, scale_out, amax_scratch, st, !bulk)) return rc;
  if (n > 0) {
    if (bulk) launch_encode_any(src_dtype, fp8_dtype, src, dst, n, nullptr, st, amax_scratch, fmax, scale_out);
    else launch_encode_any(src_dtype, fp8_dtype, src, dst, n, scale_out, st);
    count_launch();
    return check_launch("quantize encode");
  }
  return FP8B200_OK;
}

extern "C" int fp8b200_encode_fp4(const void *src, int src_dtype, void *dst, int64_t n, const float *scale,
                                  void *stream) {
  if (n < 0 || (n & 1)) return set_error(FP8B200_EINVAL, "fp4 encode: element count must be even and non-negative");
  if (!is_float_dtype(src_dtype)) return set_error(FP8B200_EINVAL, "fp4 encode: source dtype %d is not f32/bf16/f16", src_dtype);
  if (n == 0) return FP8B200_OK;
  if (!src || !dst) return set_error(FP8B200_EINVAL, "fp4 encode: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  launch_fp4_encode_any(src_dtype, src, dst, n, scale, (cudaStream_t)stream);
  count_launch();
  return check_launch("fp4 encode");
}

extern "C" int fp8b200_quantize_fp4(const void *src, int src_dtype, void *dst, int64_t n, float *scale_out,
                                    uint32_t *amax_scratch, void *stream) {
  if (n < 0 || (n & 1)) return set_error(FP8B200_EINVAL, "fp4 quantize: element count must be even and non-negative");
  if (!is_float_dtype(src_dtype)) return set_error(FP8B200_EINVAL, "fp4 quantize: source dtype %d is not f32/bf16/f16", src_dtype);
  if (!scale_out || !amax_scratch) return set_error(FP8B200_EINVAL, "fp4 quantize: null scale/scratch pointer");
  if (n > 0 && (!src || !dst)) return set_error(FP8B200_EINVAL, "fp4 quantize: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool bulk = n > 0 && aligned16(src) && aligned16(dst);  // the encoder derives the scale from the amax
  if (int rc = launch_amax_and_scale(src, src_dtype, n, 6.0f, scale_out, amax_scratch, st, !bulk)) return rc;
  if (n > 0) {
    if (bulk) launch_fp4_encode_any(src_dtype, src, dst, n, nullptr, st, amax_scratch, 6.0f, scale_out);
    else launch_fp4_encode_any(src_dtype, src, dst, n, scale_out, st);
    count_launch();
    return check_launch("fp4 quantize encode");
  }
  return FP8B200_OK;
}

template <int SRC, int FMT, int KV>
void launch_rows_reg_t(const uint8_t *s, int64_t ld_src, uint8_t *d, int64_t ld_dst, int64_t rows, int64_t cols,
                       float fmax, float *inv, cudaStream_t st) {
  const void *k = (const void *)quantize_rows_reg_kernel<SRC, FMT, KV>;
  const int g = (int)std::min<int64_t>(rows, (int64_t)current_sm_count() * resident_per_sm(k, 0, kRowThreads));
  quantize_rows_reg_kernel<SRC, FMT, KV><<<g, kRowThreads, 0, st>>>(s, ld_src, d, ld_dst, rows, cols, fmax, inv);
}

template <int SRC, int FMT>
void launch_rows_reg_kv(int kv, const uint8_t *s, int64_t ld_src, uint8_t *d, int64_t ld_dst, int64_t rows,
                        int64_t cols, float fmax, float *inv, cudaStream_t st) {
  if (kv == 1) launch_rows_reg_t<SRC, FMT, 1>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else if (kv == 2) launch_rows_reg_t<SRC, FMT, 2>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else if (kv == 4) launch_rows_reg_t<SRC, FMT, 4>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else launch_rows_reg_t<SRC, FMT, 8>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
}

template <int SRC, int FMT, int KW>
void launch_rows_warp_t(const uint8_t *s, int64_t ld_src, uint8_t *d, int64_t ld_dst, int64_t rows, int64_t cols,
                        float fmax, float *inv, cudaStream_t st) {
  const void *k = (const void *)quantize_rows_warp_kernel<SRC, FMT, KW>;
  const int64_t blocks = (rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
  const int g = (int)std::min<int64_t>(blocks, (int64_t)current_sm_count() * resident_per_sm(k, 0, kRowThreads));
  quantize_rows_warp_kernel<SRC, FMT, KW><<<g, kRowThreads, 0, st>>>(s, ld_src, d, ld_dst, rows, cols, fmax, inv);
}

template <int SRC, int FMT>
void launch_rows_warp_kw(int kw, const uint8_t *s, int64_t ld_src, uint8_t *d, int64_t ld_dst, int64_t rows,
                         int64_t cols, float fmax, float *inv, cudaStream_t st) {
  if (kw == 1) launch_rows_warp_t<SRC, FMT, 1>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else if (kw == 2) launch_rows_warp_t<SRC, FMT, 2>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else if (kw == 4) launch_rows_warp_t<SRC, FMT, 4>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  else if constexpr (SRC != FP8B200_F32) launch_rows_warp_t<SRC, FMT, 8>(s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
}

// One row per warp for rows of at most 32 x (8 units for 16-bit, 4 for f32).
void launch_rows_warp(int src_dtype, int fp8_dtype, int kw, const uint8_t *s, int64_t ld_src, uint8_t *d,
                      int64_t ld_dst, int64_t rows, int64_t cols, float fmax, float *inv, cudaStream_t st) {
  if (fp8_dtype == FP8B200_E4M3) {
    if (src_dtype == FP8B200_F32) launch_rows_warp_kw<FP8B200_F32, FP8B200_E4M3>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else if (src_dtype == FP8B200_BF16) launch_rows_warp_kw<FP8B200_BF16, FP8B200_E4M3>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else launch_rows_warp_kw<FP8B200_F16, FP8B200_E4M3>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  } else {
    if (src_dtype == FP8B200_F32) launch_rows_warp_kw<FP8B200_F32, FP8B200_E5M2>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else if (src_dtype == FP8B200_BF16) launch_rows_warp_kw<FP8B200_BF16, FP8B200_E5M2>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else launch_rows_warp_kw<FP8B200_F16, FP8B200_E5M2>(kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  }
}

void launch_rows_reg(int src_dtype, int fp8_dtype, int kv, const uint8_t *s, int64_t ld_src, uint8_t *d,
                     int64_t ld_dst, int64_t rows, int64_t cols, float fmax, float *inv, cudaStream_t st) {
  if (fp8_dtype == FP8B200_E4M3) {
    if (src_dtype == FP8B200_F32) launch_rows_reg_kv<FP8B200_F32, FP8B200_E4M3>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else if (src_dtype == FP8B200_BF16) launch_rows_reg_kv<FP8B200_BF16, FP8B200_E4M3>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else launch_rows_reg_kv<FP8B200_F16, FP8B200_E4M3>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  } else {
    if (src_dtype == FP8B200_F32) launch_rows_reg_kv<FP8B200_F32, FP8B200_E5M2>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else if (src_dtype == FP8B200_BF16) launch_rows_reg_kv<FP8B200_BF16, FP8B200_E5M2>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
    else launch_rows_reg_kv<FP8B200_F16, FP8B200_E5M2>(kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv, st);
  }
}

extern "C" int fp8b200_quantize_rows_fp8(const void *src, int src_dtype, int64_t rows, int64_t cols, int64_t ld_src,
                                         void *dst, int64_t ld_dst, int fp8_dtype, float *inv_scale, void *stream) {
  if (rows < 0 || cols < 0) return set_error(FP8B200_EINVAL, "quantize_rows: negative size");
  if (!is_float_dtype(src_dtype)) return set_error(FP8B200_EINVAL, "quantize_rows: source dtype %d is not f32/bf16/f16", src_dtype);
  if (!is_fp8_dtype(fp8_dtype)) return set_error(FP8B200_EINVAL, "quantize_rows: target dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (ld_src < cols || ld_dst < cols) return set_error(FP8B200_EINVAL, "quantize_rows: row stride smaller than the row");
  if (rows == 0) return FP8B200_OK;
  if (!src || !dst || !inv_scale) return set_error(FP8B200_EINVAL, "quantize_rows: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  const int eb = src_dtype == FP8B200_F32 ? 4 : 2;
  // 32-byte loads need every row start 32-byte aligned, 16-byte stores every output row 16-byte aligned
  const int vec = aligned32(src) && (ld_src * eb) % 32 == 0 && aligned16(dst) && ld_dst % 16 == 0;
  const float fmax = fp8_dtype == FP8B200_E4M3 ? 448.0f : 57344.0f;
  cudaStream_t st = (cudaStream_t)stream;
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  const int64_t nunits = cols / 16;
  if (vec && cols % 16 == 0 && nunits <= 32 * (eb == 4 ? 4 : 8)) {  // whole row in one warp's registers
    const int kw = nunits <= 32 ? 1 : nunits <= 64 ? 2 : nunits <= 128 ? 4 : 8;
    launch_rows_warp(src_dtype, fp8_dtype, kw, s, ld_src, d, ld_dst, rows, cols, fmax, inv_scale, st);
    count_launch();
    return check_launch("quantize_rows");
  }
  if (vec && cols % 16 == 0 && nunits <= 8 * kRowThreads) {  // whole row in the block's registers
    const int kv = nunits <= kRowThreads ? 1 : nunits <= 2 * kRowThreads ? 2 : nunits <= 4 * kRowThreads ? 4 : 8;
    launch_rows_reg(src_dtype, fp8_dtype, kv, s, ld_src, d, ld_dst, rows, cols, fmax, inv_scale, st);
    count_launch();
    return check_launch("quantize_rows");
  }
  const int g = (int)std::min<int64_t>(rows, (int64_t)current_sm_count() * 8);
#define QR(SRC, FMT) quantize_rows_kernel<SRC, FMT><<<g, kRowThreads, 0, st>>>(s, ld_src, d, ld_dst, rows, cols, vec, fmax, inv_scale)
  if (fp8_dtype == FP8B200_E4M3) {
    if (src_dtype == FP8B200_F32) QR(FP8B200_F32, FP8B200_E4M3);
    else if (src_dtype == FP8B200_BF16) QR(FP8B200_BF16, FP8B200_E4M3);
    else QR(FP8B200_F16, FP8B200_E4M3);
  } else {
    if (src_dtype == FP8B200_F32) QR(FP8B200_F32, FP8B200_E5M2);
    else if (src_dtype == FP8B200_BF16) QR(FP8B200_BF16, FP8B200_E5M2);
    else QR(FP8B200_F16, FP8B200_E5M2);
  }
#undef QR
  count_launch();
  return check_launch("quantize_rows");
}

extern "C" int fp8b200_silu_mul_quantize_rows_fp8(const void *gate_up, int64_t rows, int64_t f, int64_t ld,
                                                  void *dst, int64_t ld_dst, int fp8_dtype, float *inv_scale,
                                                  void *stream) {
  if (rows < 0 || f < 0) return set_error(FP8B200_EINVAL, "silu_mul_quantize: negative size");
  if (!is_fp8_dtype(fp8_dtype)) return set_error(FP8B200_EINVAL, "silu_mul_quantize: target dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (ld < 2 * f || ld_dst < f) return set_error(FP8B200_EINVAL, "silu_mul_quantize: row stride smaller than the row");
  const int64_t smem = f * 2;
  if (smem > 200 * 1024) return set_error(FP8B200_EINVAL, "silu_mul_quantize: F=%lld exceeds the 102400-element row limit", (long long)f);
  if (rows == 0) return FP8B200_OK;
  if (!gate_up || !dst || !inv_scale) return set_error(FP8B200_EINVAL, "silu_mul_quantize: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  // 16-byte vectors need every g and u row start 16-byte aligned (f and ld multiples of 8) and 8-byte output rows
  const int vec = aligned16(gate_up) && f % 8 == 0 && ld % 8 == 0 && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0 &&
                  ld_dst % 8 == 0;
  const float fmax = fp8_dtype == FP8B200_E4M3 ? 448.0f : 57344.0f;
  cudaStream_t st = (cudaStream_t)stream;
  const void *k = fp8_dtype == FP8B200_E4M3 ? (const void *)silu_mul_quantize_kernel<FP8B200_E4M3>
                                            : (const void *)silu_mul_quantize_kernel<FP8B200_E5M2>;
  const int per_sm = resident_per_sm(k, (int)smem, kRowThreads);
  const int g = (int)std::min<int64_t>(rows, (int64_t)current_sm_count() * per_sm);
  if (fp8_dtype == FP8B200_E4M3)
    silu_mul_quantize_kernel<FP8B200_E4M3><<<g, kRowThreads, smem, st>>>((const uint16_t *)gate_up, ld, (uint8_t *)dst,
                                                                        ld_dst, rows, f, vec, fmax, inv_scale);
  else
    silu_mul_quantize_kernel<FP8B200_E5M2><<<g, kRowThreads, smem, st>>>((const uint16_t *)gate_up, ld, (uint8_t *)dst,
                                                                        ld_dst, rows, f, vec, fmax, inv_scale);
  count_launch();
  return check_launch("silu_mul_quantize");
}

// ------------------------------------------------------------------ rotary embedding (bf16)
// Rotary position embedding of the q and k heads of a fused qkv projection,
// with the roundings of PyTorch's bf16 expression
//   cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)
// (each product of two bf16 values rounded to bf16, then the float difference
// / sum of those rounded to bf16). Both steps run as bf16x2 instructions
// (mul/sub/add .rn.bf16x2, rounding once from the exact result): a product of
// two bf16 values is exact in float, and for the sum and difference the float
// intermediate rounding is innocuous because float carries 24 >= 2 x 8 + 2
// significand bits, so one rounding from the exact value gives the same bf16
// as PyTorch's float operation followed by rounding. One thread produces 8
// outputs of each half of one head: 16-byte loads of x1, x2, cos and sin,
// 16-byte stores. Rows of qkv are tokens (position = token % seq); q heads come
// first, then k heads, head_dim contiguous elements each.
namespace fp8b200 {
namespace {

__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

template <typename I>  // index type: 32-bit when the work fits, else 64-bit
__global__ void __launch_bounds__(256)
rope_kernel(const uint16_t *__restrict__ qkv, int64_t ld, I tokens, I nq, I nk, I hd, I seq,
            const uint16_t *__restrict__ cosv, const uint16_t *__restrict__ sinv, uint16_t *__restrict__ oq,
            uint16_t *__restrict__ ok) {
  const I half = hd / 2, groups = half / 8, heads = nq + nk;
  const I total = tokens * heads * groups;
  for (I w = (I)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += (I)gridDim.x * blockDim.x) {
    const I th = w / groups, g = w - th * groups;
    const I t = th / heads, h = th - t * heads;
    const I pos = t % seq;
    const uint16_t *x = qkv + (int64_t)t * ld + (int64_t)h * hd + g * 8;
    const uint4 a = *reinterpret_cast<const uint4 *>(x);
    const uint4 b = *reinterpret_cast<const uint4 *>(x + half);
    const uint4 c = __ldg(reinterpret_cast<const uint4 *>(cosv + (int64_t)pos * half + g * 8));
    const uint4 s = __ldg(reinterpret_cast<const uint4 *>(sinv + (int64_t)pos * half + g * 8));
    const uint4 lo = make_uint4(bsub2(bmul2(a.x, c.x), bmul2(b.x, s.x)), bsub2(bmul2(a.y, c.y), bmul2(b.y, s.y)),
                                bsub2(bmul2(a.z, c.z), bmul2(b.z, s.z)), bsub2(bmul2(a.w, c.w), bmul2(b.w, s.w)));
    const uint4 hi = make_uint4(badd2(bmul2(b.x, c.x), bmul2(a.x, s.x)), badd2(bmul2(b.y, c.y), bmul2(a.y, s.y)),
                                badd2(bmul2(b.z, c.z), bmul2(a.z, s.z)), badd2(bmul2(b.w, c.w), bmul2(a.w, s.w)));
    uint16_t *o = h < nq ? oq + ((int64_t)t * nq + h) * hd : ok + ((int64_t)t * nk + (h - nq)) * hd;
    *reinterpret_cast<uint4 *>(o + g * 8) = lo;
    *reinterpret_cast<uint4 *>(o + half + g * 8) = hi;
  }
}

}  // namespace
}  // namespace fp8b200

extern "C" int fp8b200_rope_bf16(const void *qkv, int64_t tokens, int64_t ld, int n_q_heads, int n_k_heads,
                                 int head_dim, int seq, const void *cos_table, const void *sin_table, void *out_q,
                                 void *out_k, void *stream) {
  using namespace fp8b200;
  if (tokens < 0 || n_q_heads < 0 || n_k_heads < 0 || seq <= 0)
    return set_error(FP8B200_EINVAL, "rope: negative size or seq <= 0");
  if (head_dim <= 0 || head_dim % 16)
    return set_error(FP8B200_EINVAL, "rope: head_dim=%d must be a positive multiple of 16", head_dim);
  if (ld < (int64_t)(n_q_heads + n_k_heads) * head_dim || ld % 8)
    return set_error(FP8B200_EINVAL, "rope: row stride must cover the q and k heads and be a multiple of 8");
  if (tokens == 0 || n_q_heads + n_k_heads == 0) return FP8B200_OK;
  if (!qkv || !cos_table || !sin_table || (n_q_heads && !out_q) || (n_k_heads && !out_k))
    return set_error(FP8B200_EINVAL, "rope: null pointer");
  if (!aligned16(qkv) || !aligned16(cos_table) || !aligned16(sin_table) || (out_q && !aligned16(out_q)) ||
      (out_k && !aligned16(out_k)))
    return set_error(FP8B200_EINVAL, "rope: tensors must be 16-byte aligned");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  const int64_t work = tokens * (n_q_heads + n_k_heads) * (head_dim / 16);
  const int g = (int)std::min<int64_t>((work + 255) / 256, (int64_t)current_sm_count() * 8);
  const int64_t total = tokens * (n_q_heads + n_k_heads) * (head_dim / 16);
  if (total + (int64_t)g * 256 < ((int64_t)1 << 31) && tokens * (int64_t)(n_q_heads + n_k_heads) * head_dim < ((int64_t)1 << 31))
    rope_kernel<int><<<g, 256, 0, (cudaStream_t)stream>>>((const uint16_t *)qkv, ld, (int)tokens, n_q_heads, n_k_heads,
                                                          head_dim, seq, (const uint16_t *)cos_table,
                                                          (const uint16_t *)sin_table, (uint16_t *)out_q,
                                                          (uint16_t *)out_k);
  else
    rope_kernel<int64_t><<<g, 256, 0, (cudaStream_t)stream>>>((const uint16_t *)qkv, ld, tokens, n_q_heads,
                                                              n_k_heads, head_dim, seq, (const uint16_t *)cos_table,
                                                              (const uint16_t *)sin_table, (uint16_t *)out_q,
                                                              (uint16_t *)out_k);
  count_launch();
  return check_launch("rope");
}

// FP8 scaled GEMM for B200 on the 5th-generation tensor cores (tcgen05).
//
//   D[M,N] = (A[M,K] * sa) @ (B[N,K] * sb)^T  [+ bias[N]]  [* scale_result]
//
// A and B are float8 (e4m3fn or e5m2) codes with K contiguous ("K-major"), the
// layout torch._scaled_mm requires (self row-major, mat2 column-major). The
// accumulation is float32 in tensor memory (TMEM).
//
// Kernel structure (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: 128x128-byte A tiles and 256x128-byte B tiles,
//               128-byte swizzled, into a 4-stage shared-memory ring
//               (cp.async.bulk.tensor, no multicast; L2 gives the reuse).
//   warp 1      MMA issuer: one thread issues tcgen05.mma.kind::f8f6f4
//               (M=128, N=256, K=32) into one of two TMEM accumulators
//               (2 x 256 fp32 columns), commits to mbarriers.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp its own
//               32-lane quarter), scale, bias, convert, store to global. The
//               double-buffered accumulator lets the epilogue of tile i
//               overlap the MMAs of tile i+1.
// Every mbarrier wait is bounded (globaltimer): on timeout the kernel records
// a status word, stops issuing, releases TMEM and returns; the host reads the
// status with fp8b200_gemm_status().
//
// Replaces fp8_scaled_matmul_kernel / fp8_scaled_vecmat_kernel
// (shaders/fp8_matmul.metal:145-226) and the decode + fp16 matmul path
// (fp8_mps_native.py:129-159).
#include "common.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

namespace fp8b200 {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;           // bytes = fp8 elements per k-block (one 128B swizzle row)
constexpr int STAGES = 4;
constexpr int UMMA_K = 32;        // K per tcgen05.mma for 8-bit operands
constexpr int A_BYTES = BM * BK;  // 16 KiB
constexpr int B_BYTES = BN * BK;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;    // two 256-column fp32 accumulators
constexpr int GROUP_M = 16;       // tile raster: 16 M-tiles per group for L2 reuse
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 2 * BN * 4 /*column tables*/ + 256 /*barriers*/;

struct Params {
  int M, N, K, num_kb, tiles_m, tiles_n, num_tiles;
  const float *sa, *sb;
  int sa_rowwise, sb_rowwise;
  const void *bias;
  int bias_dtype;
  const float *scale_result;
  void *D;
  long long ldd;
  int out_dtype;
  int vec_store;
  uint32_t idesc;
  unsigned long long timeout_ns;
  uint32_t epoch;                             // launch number: scopes the status word to this launch
  uint32_t tx_bytes;                          // TMA bytes per stage credited to this CTA's full barrier
  int debug_skip_first_load;
  int sk_mt, sk_stages, sk_cs, sk_tmem_cols;  // small-M kernel: rows per tile, ring depth, split-K cluster, TMEM
  int tma_store;                              // epilogue stores through the output tensor map
  int w_fp8;                                  // fp8-weight linear: weight format (FP8B200_E4M3 / E5M2)
  int kb_elems;                               // elements per 128-byte k-block (128 fp8, 64 16-bit)
  int act_f16;                                // fp8-weight linear: activations f16 (1) or bf16 (0)
  int w_bn1;                                  // 256x512 kernel: width of the second 256-row MMA (256 or 224)
  uint32_t idesc1;                            // its instruction descriptor (N = w_bn1)
};

// Status word: 0 = ok, otherwise (launch epoch << 32) | (1 << 31) | site of
// the first wait that timed out in that launch. A launch gives up early only
// on a failure recorded under its own epoch, so a timed-out launch leaves
// every later launch unaffected; the word keeps the last failure until
// fp8b200_gemm_status() resets it.
__device__ unsigned long long g_status;

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// A role that gives up leaves its loop while copies and MMAs it or its CTA
// issued earlier may still be landing in the CTA's shared and tensor memory;
// the thread then holds the CTA (and so that memory) for a bounded 200 us
// before the caller goes on to the kernel's teardown.
__device__ __noinline__ void hold_after_failure() {
  const uint64_t t0 = globaltimer();
  while (globaltimer() - t0 < 200000ull) __nanosleep(1000);
}
// Bounded wait on phase `parity` of `bar`; false on timeout or if another
// role already recorded a failure. The first test is inlined at every call
// site: a wait whose phase has already completed (the common case in a
// pipeline that keeps up) costs one try_wait, not a function call; the
// timed loop is out of line.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, unsigned long long timeout_ns, uint32_t epoch,
                                            uint32_t site) {
  const uint64_t t0 = globaltimer();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 31u) == 0) {
      unsigned long long s = *reinterpret_cast<volatile unsigned long long *>(&g_status);
      if ((uint32_t)(s >> 32) == epoch) {  // another role of this launch gave up
        hold_after_failure();
        return false;
      }
      if (globaltimer() - t0 > timeout_ns) {
        // record the first failure of this launch, replacing an older launch's record
        const unsigned long long mine = ((unsigned long long)epoch << 32) | 0x80000000ull | site;
        while ((uint32_t)(s >> 32) != epoch) {
          const unsigned long long prev = atomicCAS(&g_status, s, mine);
          if (prev == s) break;
          s = prev;
        }
        hold_after_failure();
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned long long timeout_ns, uint32_t epoch,
                                          uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, timeout_ns, epoch, site);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void umma_f8f6f4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive fp32 columns: thread t receives lane t's 32 values.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Wait for the outstanding TMEM loads, with r as read-write operands so that
// no use of the loaded registers can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc_sw128_kmajor(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                    // descriptor version for sm_100
  d |= (uint64_t)2 << 61;                    // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tile_coords(const Params &p, int tile, int &tm, int &tn) {
  const int per_group = GROUP_M * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(p.tiles_m - first_m, GROUP_M);
  const int r = tile - group * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// ------------------------------------------------------------------ epilogue conversion
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}
// fp8 encode with CPU PyTorch semantics (as in convert.cu): cvt.satfinite
// plus the overflow / inf / NaN fix-up.
template <int FMT>
__device__ __forceinline__ uint32_t enc8(float x) {
  const uint32_t b = __float_as_uint(x), a = b & 0x7FFFFFFFu, s = (b >> 24) & 0x80u;
  uint16_t r;
  if constexpr (FMT == FP8B200_E4M3) {
    if (a > 0x43E80000u) return s | 0x7Fu;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  } else {
    if (a > 0x7F800000u) return s | 0x7Fu;
    if (a > 0x476FFFFFu) return s | 0x7Cu;
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  }
  return r & 0xFFu;
}

__device__ __forceinline__ float load_bias(const void *bias, int dt, int col) {
  if (dt == FP8B200_F32) return reinterpret_cast<const float *>(bias)[col];
  if (dt == FP8B200_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(bias)[col]);
  return __half2float(reinterpret_cast<const __half *>(bias)[col]);
}

// Scale, bias and store 32 consecutive columns of one output row. col_scale /
// col_bias point at this chunk's 32 entries of the tile's column tables in
// shared memory (every lane reads the same address: broadcast).
__device__ __forceinline__ void store_row_chunk(const Params &p, int row, int col0, const uint32_t (&acc)[32],
                                                float row_scale, const float *col_scale, const float *col_bias,
                                                float sr) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = (__uint_as_float(acc[j]) * (row_scale * col_scale[j]) + col_bias[j]) * sr;
  const bool full = p.vec_store && (col0 + 32 <= p.N);
  char *base = reinterpret_cast<char *>(p.D);
  switch (p.out_dtype) {
    case FP8B200_BF16:
    case FP8B200_F16: {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; j++)
        w[j] = p.out_dtype == FP8B200_BF16 ? pack_bf16(v[2 * j], v[2 * j + 1]) : pack_f16(v[2 * j], v[2 * j + 1]);
      uint16_t *rowp = reinterpret_cast<uint16_t *>(base) + (long long)row * p.ldd;
      if (full) {
        uint4 *dst = reinterpret_cast<uint4 *>(rowp + col0);
#pragma unroll
        for (int q = 0; q < 4; q++) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (col0 + j < p.N) rowp[col0 + j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
      }
      break;
    }
    case FP8B200_F32: {
      float *rowp = reinterpret_cast<float *>(base) + (long long)row * p.ldd;
      if (full) {
        float4 *dst = reinterpret_cast<float4 *>(rowp + col0);
#pragma unroll
        for (int q = 0; q < 8; q++) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (col0 + j < p.N) rowp[col0 + j] = v[j];
      }
      break;
    }
    default: {  // fp8 output
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        uint32_t c[4];
#pragma unroll
        for (int t = 0; t < 4; t++)
          c[t] = p.out_dtype == FP8B200_E4M3 ? enc8<FP8B200_E4M3>(v[4 * q + t]) : enc8<FP8B200_E5M2>(v[4 * q + t]);
        w[q] = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
      }
      uint8_t *rowp = reinterpret_cast<uint8_t *>(base) + (long long)row * p.ldd;
      if (full) {
        uint4 *dst = reinterpret_cast<uint4 *>(rowp + col0);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (col0 + j < p.N) rowp[col0 + j] = (uint8_t)(w[j >> 2] >> (8 * (j & 3)));
      }
      break;
    }
  }
}

// Named barrier among the four epilogue warps (128 threads).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Named barrier among the eight epilogue warps of the wide kernel (256 threads).
__device__ __forceinline__ void wide_epilogue_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The tile's per-column factors (tensorwise or rowwise scale_b; bias or 0),
// loaded once per tile by the 128 epilogue threads into shared memory.
__device__ __forceinline__ void stage_columns(const Params &p, int n0, float sb_t, float *s_scale, float *s_bias,
                                              int etid) {
  for (int j = etid; j < BN; j += 128) {
    const int col = n0 + j;
    const bool in = col < p.N;
    s_scale[j] = in ? (p.sb_rowwise ? __ldg(p.sb + col) : sb_t) : 0.0f;
    s_bias[j] = (in && p.bias != nullptr) ? load_bias(p.bias, p.bias_dtype, col) : 0.0f;
  }
}

// Drain one 128-row x 256-column accumulator: each epilogue warp reads its
// 32-lane quarter of TMEM (rows) in 32-column chunks.
__device__ __forceinline__ void drain_accumulator(const Params &p, uint32_t t_acc, int row0, int n0, int quarter,
                                                  int lane, float rs_t, const float *s_scale, const float *s_bias,
                                                  float sr, int cfirst = 0, int cstep = 1) {
  const int row = row0 + quarter * 32 + lane;
  const float rs = p.sa_rowwise ? ((row < p.M) ? __ldg(p.sa + row) : 0.0f) : rs_t;
  const uint32_t t_row = t_acc + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
  for (int c = cfirst; c < BN / 32; c += cstep) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + (uint32_t)(c * 32), r);
    tmem_ld_wait(r);
    const int col0 = n0 + c * 32;
    if (row < p.M && col0 < p.N) store_row_chunk(p, row, col0, r, rs, s_scale + c * 32, s_bias + c * 32, sr);
  }
}

// ---- epilogue through TMA stores
// Each epilogue warp converts a 32-row x 32-column chunk of its accumulator
// rows into a 2 KiB staging buffer in shared memory laid out as the TMA
// store's box (32 rows of 64 bytes: 32 bf16/f16 or 16 fp32 values; 32 rows of
// 32 bytes for fp8) with the tensor map's swizzle (the 16-byte unit u of row r
// sits at u ^ f(r)), so that the warp's 16-byte shared stores are
// conflict-free without dynamic register indexing; one lane then stores the
// box with cp.async.bulk.tensor (whole row segments, asynchronous, clipped at
// the tensor's edges). The buffer is rewritten only after the previous store
// from it has finished reading.
constexpr int W_STG_BYTES = 2048;  // per epilogue warp

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Convert one 32-column chunk (accumulator values r, row scale rs) and store
// it through this warp's staging buffer with TMA stores of box (col0, y0)
// (two 16-column boxes for fp32).
__device__ __forceinline__ void store_chunk_tma(const Params &p, const CUtensorMap *tmap_d, const uint32_t (&r)[32],
                                                float rs, const float *cs, const float *cb, float sr, int lane,
                                                int col0, int y0, int esz, uint32_t buf) {
  float v[32];
#pragma unroll
  for (int q = 0; q < 8; q++) {  // 16-byte broadcast reads of the column tables
    const float4 s4 = reinterpret_cast<const float4 *>(cs)[q];
    const float4 b4 = reinterpret_cast<const float4 *>(cb)[q];
    v[4 * q] = (__uint_as_float(r[4 * q]) * (rs * s4.x) + b4.x) * sr;
    v[4 * q + 1] = (__uint_as_float(r[4 * q + 1]) * (rs * s4.y) + b4.y) * sr;
    v[4 * q + 2] = (__uint_as_float(r[4 * q + 2]) * (rs * s4.z) + b4.z) * sr;
    v[4 * q + 3] = (__uint_as_float(r[4 * q + 3]) * (rs * s4.w) + b4.w) * sr;
  }
  const uint32_t row64 = buf + (uint32_t)lane * 64u;
  const uint32_t sw64 = (uint32_t)((lane >> 1) & 3);  // 64-byte swizzle of row `lane`
  if (esz == 4) {  // two boxes of 16 fp32 columns
#pragma unroll
    for (int h = 0; h < 2; h++) {
      if (lane == 0) bulk_wait_read_0();
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 4; u++)
        st_shared_v4(row64 + ((u ^ sw64) * 16u), __float_as_uint(v[16 * h + 4 * u]),
                     __float_as_uint(v[16 * h + 4 * u + 1]), __float_as_uint(v[16 * h + 4 * u + 2]),
                     __float_as_uint(v[16 * h + 4 * u + 3]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmap_d, buf, col0 + 16 * h, y0);
        bulk_commit();
      }
    }
    return;
  }
  if (lane == 0) bulk_wait_read_0();
  __syncwarp();
  if (esz == 2) {
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; j++)
      w[j] = p.out_dtype == FP8B200_BF16 ? pack_bf16(v[2 * j], v[2 * j + 1]) : pack_f16(v[2 * j], v[2 * j + 1]);
#pragma unroll
    for (int u = 0; u < 4; u++) st_shared_v4(row64 + ((u ^ sw64) * 16u), w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
  } else {  // fp8: 32-byte rows, 32-byte swizzle: unit u of row r at u ^ ((r >> 2) & 1)
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      uint32_t cc[4];
#pragma unroll
      for (int t = 0; t < 4; t++)
        cc[t] = p.out_dtype == FP8B200_E4M3 ? enc8<FP8B200_E4M3>(v[4 * q + t]) : enc8<FP8B200_E5M2>(v[4 * q + t]);
      w[q] = cc[0] | (cc[1] << 8) | (cc[2] << 16) | (cc[3] << 24);
    }
    const uint32_t rb = buf + (uint32_t)lane * 32u;
#pragma unroll
    for (int u = 0; u < 2; u++)
      st_shared_v4(rb + (uint32_t)((u ^ ((lane >> 2) & 1)) * 16), w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
  }
  fence_proxy_async_smem();  // make the generic-proxy writes visible to the bulk copy
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmap_d, buf, col0, y0);
    bulk_commit();
  }
}

// Drain chunks cfirst, cfirst + cstep, ... of 256 accumulator columns of this
// warp's 32 rows through TMA stores (buf: this warp's staging buffer). The
// TMEM loads run one chunk ahead of the conversion (two register sets), so
// their latency hides behind the previous chunk's arithmetic.
__device__ __forceinline__ void drain_accumulator_tma(const Params &p, const CUtensorMap *tmap_d, uint32_t t_acc,
                                                      int row0, int n0, int width, int quarter, int lane, float rs_t,
                                                      const float *col_scale, const float *col_bias, float sr,
                                                      uint32_t buf, int cfirst, int cstep) {
  const int row = row0 + quarter * 32 + lane;
  const float rs = p.sa_rowwise ? ((row < p.M) ? __ldg(p.sa + row) : 0.0f) : rs_t;
  const uint32_t t_row = t_acc + ((uint32_t)(quarter * 32) << 16);
  const int esz = p.out_dtype == FP8B200_F32 ? 4 : (p.out_dtype == FP8B200_BF16 || p.out_dtype == FP8B200_F16) ? 2 : 1;
  const int y0 = row0 + quarter * 32;
  const int nchunks = min(width / 32, (p.N - n0 + 31) / 32);  // chunks with at least one column in range
  if (cfirst >= nchunks) return;
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(t_row + (uint32_t)(cfirst * 32), ra);
  tmem_ld_wait(ra);
#pragma unroll 1
  for (int c = cfirst; c < nchunks; c += 2 * cstep) {
    const int c1 = c + cstep, c2 = c + 2 * cstep;
    if (c1 < nchunks) tmem_ld_32x32b_x32(t_row + (uint32_t)(c1 * 32), rb);
    store_chunk_tma(p, tmap_d, ra, rs, col_scale + c * 32, col_bias + c * 32, sr, lane, n0 + c * 32, y0, esz, buf);
    tmem_ld_wait(rb);
    if (c1 >= nchunks) break;
    if (c2 < nchunks) tmem_ld_32x32b_x32(t_row + (uint32_t)(c2 * 32), ra);
    store_chunk_tma(p, tmap_d, rb, rs, col_scale + c1 * 32, col_bias + c1 * 32, sr, lane, n0 + c1 * 32, y0, esz,
                    buf);
    tmem_ld_wait(ra);
  }
}

// ------------------------------------------------------------------ single-CTA kernel
__global__ void __launch_bounds__(THREADS, 1)
scaled_mm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled tiles
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  const uint32_t sA = base;                     // STAGES x 16 KiB
  const uint32_t sB = base + STAGES * A_BYTES;  // STAGES x 32 KiB
  float *s_scale = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES);
  float *s_bias = s_scale + BN;
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_bias + BN);
  // barriers: full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], then the TMEM address slot
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + 2 + b); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, p.epoch, 1)) { ok = false; break; }
          if (p.debug_skip_first_load) { ok = false; break; }  // test hook: never fill stage 0
          mbar_expect_tx(full_bar(stage), p.tx_bytes);
          tma_load_2d(sA + stage * A_BYTES, &tmap_a, full_bar(stage), kb * BK, tm * BM);
          tma_load_2d(sB + stage * B_BYTES, &tmap_b, full_bar(stage), kb * BK, tn * BN);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, p.epoch, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128_kmajor(sA + stage * A_BYTES);
          const uint64_t bdesc = sdesc_sw128_kmajor(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; k++) {
            // advance along K inside the 128-byte swizzled row: +32 bytes
            umma_f8f6f4(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4),
                        p.idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));  // frees the smem stage once these MMAs finish
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));  // accumulator ready for the epilogue
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5, TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    const int etid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    const float sa_t = p.sa_rowwise ? 0.0f : __ldg(p.sa);
    const float sb_t = p.sb_rowwise ? 0.0f : __ldg(p.sb);
    const float sr = p.scale_result ? __ldg(p.scale_result) : 1.0f;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      epilogue_sync();  // the previous tile's column tables are no longer read
      stage_columns(p, tn * BN, sb_t, s_scale, s_bias, etid);
      epilogue_sync();
      // warp-uniform bounded wait
      int ok = 0;
      if (lane == 0) ok = mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, p.epoch, 4) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      drain_accumulator(p, tmem_base + (uint32_t)(acc * BN), tm * BM, tn * BN, quarter, lane, sa_t, s_scale,
                        s_bias, sr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ CTA-pair kernel
// A cluster of two CTAs computes a 256x256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=32). Each CTA loads its own 128
// rows of A and its own 128-row half of B into its shared memory (same
// offsets in both CTAs); the MMA reads A rows and B halves from both. The
// loads of both CTAs complete on the leader's (rank 0) full barrier; the
// leader's single MMA thread commits to the empty and tmem_full barriers of
// both CTAs; each CTA's epilogue drains its own 128 accumulator rows and
// arrives on the leader's tmem_empty barrier.
constexpr int PAIR_BN = 256;              // output columns per pair tile
constexpr int HALF_B = PAIR_BN / 2;       // B rows loaded per CTA
constexpr int STAGES2_MAX = 7;
constexpr int A2_BYTES = BM * BK;         // 16 KiB
constexpr int B2_BYTES = HALF_B * BK;     // 16 KiB
constexpr int STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int SMEM2_TAIL = 2 * BN * 4 /*column tables*/ + 256 /*barriers*/;
// The per-CTA maximum: the ring takes as many 32 KiB stages as fit after the
// 1024-byte alignment of its base (7 when the dynamic shared memory starts at
// most 768 bytes before a 1024-byte boundary, else 6), then the tables.
constexpr int SMEM2_BYTES = 227 * 1024;
static_assert(6 * STAGE2_BYTES + 1023 + SMEM2_TAIL <= SMEM2_BYTES, "six stages always fit");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t leader_bar, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(map), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_f8f6f4_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at this shared offset in both CTAs of the pair when
// the issuing thread's MMAs complete
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
scaled_mm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  // ring depth: the same in both CTAs (same kernel, same dynamic shared-memory base)
  const int nst = min(STAGES2_MAX, (int)((raw_addr + SMEM2_BYTES - base - SMEM2_TAIL) / STAGE2_BYTES));
  const uint32_t sA = base;                   // nst x 16 KiB
  const uint32_t sB = base + nst * A2_BYTES;  // nst x 16 KiB
  float *s_scale = reinterpret_cast<float *>(smem + nst * STAGE2_BYTES);
  float *s_bias = s_scale + BN;
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_bias + BN);
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES2_MAX + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * STAGES2_MAX + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * STAGES2_MAX + 2 + b); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES2_MAX + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = (int)cluster_id_x();
  const int npairs = (int)num_clusters_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; s++) {
      mbar_init(full_bar(s), 1);   // used in the leader only
      mbar_init(empty_bar(s), 1);  // one multicast commit per use
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 8);  // four epilogue warps in each CTA (leader's barrier)
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {  // same warp in both CTAs, same destination offset
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        const int arow = tm * (2 * BM) + (int)rank * BM;
        const int brow = tn * PAIR_BN + (int)rank * HALF_B;
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, p.epoch, 1)) { ok = false; break; }
          if (p.debug_skip_first_load) { ok = false; break; }
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (rank == 0) mbar_expect_tx(full_bar(stage), p.tx_bytes);
          tma_load_2d_pair(sA + stage * A2_BYTES, &tmap_a, leader_full, kb * BK, arow);
          tma_load_2d_pair(sB + stage * B2_BYTES, &tmap_b, leader_full, kb * BK, brow);
          if (++stage == nst) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only)
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, p.epoch, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * PAIR_BN);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128_kmajor(sA + stage * A2_BYTES);
          const uint64_t bdesc = sdesc_sw128_kmajor(sB + stage * B2_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; k++)
            umma_f8f6f4_pair(d_tmem, adesc + (uint64_t)((k * UMMA_K) >> 4), bdesc + (uint64_t)((k * UMMA_K) >> 4),
                             p.idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair(empty_bar(stage));
          if (++stage == nst) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc));
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of the pair tile
    const int quarter = warp & 3;
    const int etid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    const float sa_t = p.sa_rowwise ? 0.0f : __ldg(p.sa);
    const float sb_t = p.sb_rowwise ? 0.0f : __ldg(p.sb);
    const float sr = p.scale_result ? __ldg(p.scale_result) : 1.0f;
    for (int tile = pair; tile < p.num_tiles; tile += npairs) {
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      epilogue_sync();
      stage_columns(p, tn * PAIR_BN, sb_t, s_scale, s_bias, etid);
      epilogue_sync();
      int ok = 0;
      if (lane == 0) ok = mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, p.epoch, 4) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      drain_accumulator(p, tmem_base + (uint32_t)(acc * PAIR_BN), tm * (2 * BM) + (int)rank * BM, tn * PAIR_BN,
                        quarter, lane, sa_t, s_scale, s_bias, sr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(acc), 0));
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still touch its shared memory
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Packed FP4 x FP4 with every block scale 1.0: kind::mxf4 multiplies two e2m1
// values per operand byte, K = 64 per instruction, at twice the f8f6f4 rate;
// its block32 scale factors (UE8M0) are read from tensor memory at sf (all
// 0x7F = 2^0 here), so the product equals the unscaled one.
__device__ __forceinline__ void umma_mxf4_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate, uint32_t sf) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%5], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sf)
      : "memory");
}

// KIND 0: kind::f8f6f4 (8-bit codes, or e2m1 padded to a byte, K = 32 per MMA);
// KIND 1: kind::f16 (16-bit operands, K = 16); KIND 2: kind::mxf4 (packed
// e2m1, K = 64, unit block scales at sf). Each steps through the 128-byte
// swizzled rows 32 bytes per MMA.
template <int KIND>
__device__ __forceinline__ void umma_pair(uint32_t sf, uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  if constexpr (KIND == 0) umma_f8f6f4_pair(tmem_d, adesc, bdesc, idesc, accumulate);
  else if constexpr (KIND == 1) umma_f16_pair(tmem_d, adesc, bdesc, idesc, accumulate);
  else umma_mxf4_pair(tmem_d, adesc, bdesc, idesc, accumulate, sf);
}

// ------------------------------------------------------------------ CTA-pair wide kernel
// 256 x 512 output tile per pair. Each K step issues two
// tcgen05.mma.cta_group::2 (M=256, N=256) that share the A tile, so a k-block
// moves 48 KiB per CTA (its 128 rows of A plus a 128-row half of each of the
// two B blocks) for twice the MMA work of the 256 x 256 kernel: a quarter
// fewer bytes from L2 per flop, which is what bounds the 256 x 256 kernel on
// large shapes. The two 256-column accumulators fill TMEM, so the accumulator
// is single-buffered: the MMA thread waits for the epilogue to drain it while
// the producer keeps prefetching the next tile's k-blocks into the 4-stage ring.
constexpr int WIDE_BN = 512;
constexpr int W_STAGES = 4;
constexpr int W_STAGE_BYTES = A2_BYTES + 2 * B2_BYTES;  // 48 KiB
constexpr int W_EPI_WARPS = 8;                       // two per TMEM lane quarter, splitting the columns
constexpr int W_THREADS = 64 + 32 * W_EPI_WARPS;     // producer warp, MMA warp, epilogue warps
constexpr int W_SMEM_BYTES = W_STAGES * W_STAGE_BYTES + W_EPI_WARPS * W_STG_BYTES /*epilogue staging*/ +
                             1024 /*align*/ + 2 * WIDE_BN * 4 /*column tables*/ + 256;

// TMEM columns of the unit block scales for kind::mxf4 (the 256 x 480 tile's
// accumulators use columns 0-479)
constexpr int W_SF_COL = 480;

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// KIND 0: kind::f8f6f4 (fp8 codes or byte-padded e2m1, K = 32 per MMA); 1: kind::f16 (16-bit
// operands, K = 16); 2: kind::mxf4 (packed e2m1, K = 64, unit block scales; 256 x 480 tiles)
template <int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W_THREADS, 1)
scaled_mm_wide_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_b1, const __grid_constant__ CUtensorMap tmap_d,
                      const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  // stage s: [A 16 KiB | B half of block 0, 16 KiB | B half of block 1, 16 KiB]
  auto stage_a = [&](int s) { return base + (uint32_t)(s * W_STAGE_BYTES); };
  const uint32_t stg_base = base + (uint32_t)(W_STAGES * W_STAGE_BYTES);  // W_EPI_WARPS x 2 KiB epilogue staging
  float *s_scale = reinterpret_cast<float *>(smem + W_STAGES * W_STAGE_BYTES + W_EPI_WARPS * W_STG_BYTES);
  float *s_bias = s_scale + WIDE_BN;
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_bias + WIDE_BN);
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (W_STAGES + s); };
  auto tfull_bar = [&](int h) { return bar_base + 8u * (2 * W_STAGES + h); };       // accumulator half h complete
  auto tempty_bar = [&](int h) { return bar_base + 8u * (2 * W_STAGES + 2 + h); };  // accumulator half h drained
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * W_STAGES + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = (int)cluster_id_x();
  const int npairs = (int)num_clusters_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < W_STAGES; s++) {
      mbar_init(full_bar(s), 1);   // used in the leader only
      mbar_init(empty_bar(s), 1);  // one multicast commit per use
    }
    mbar_init(tfull_bar(0), 1);
    mbar_init(tfull_bar(1), 1);
    mbar_init(tempty_bar(0), 2 * W_EPI_WARPS);  // every epilogue warp of both CTAs (leader's barriers)
    mbar_init(tempty_bar(1), 2 * W_EPI_WARPS);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_b1);
    if (p.tma_store) tma_prefetch_desc(&tmap_d);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
  const uint32_t sf_tmem = tmem_base + (uint32_t)W_SF_COL;
  if constexpr (KIND == 2) {
    // unit block scales: 0x7F (2^0 in UE8M0) in columns W_SF_COL.. of every lane of both
    // CTAs' tensor memory, written by four warps, one per 32-lane quarter (warp % 4)
    if (warp >= 2 && warp < 6) {
      uint32_t ones[32];
#pragma unroll
      for (int j = 0; j < 32; j++) ones[j] = 0x7F7F7F7Fu;
      tmem_st_32x32b_x32(sf_tmem + ((uint32_t)((warp & 3) * 32) << 16), ones);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
  }

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        const int arow = tm * (2 * BM) + (int)rank * BM;
        const int tw = PAIR_BN + p.w_bn1;  // tile width: 512, or 480 (second MMA N = 224)
        const int brow0 = tn * tw + (int)rank * HALF_B;
        // second block: each CTA holds w_bn1 / 2 rows of it (tmap_b1's box height)
        const int brow1 = tn * tw + PAIR_BN + (int)rank * (p.w_bn1 / 2);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, p.epoch, 1)) { ok = false; break; }
          if (p.debug_skip_first_load) { ok = false; break; }
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (rank == 0) mbar_expect_tx(full_bar(stage), p.tx_bytes);
          const uint32_t st = stage_a(stage);
          const int kx = kb * p.kb_elems;  // tensor-map coordinate of the k-block
          tma_load_2d_pair(st, &tmap_a, leader_full, kx, arow);
          tma_load_2d_pair(st + A2_BYTES, &tmap_b, leader_full, kx, brow0);
          tma_load_2d_pair(st + A2_BYTES + B2_BYTES, &tmap_b1, leader_full, kx, brow1);
          if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only)
    // From the second tile on, the first W_STAGES k-blocks are issued in two
    // passes: the half-0 MMAs as soon as the epilogue has drained accumulator
    // half 0, then (stages still resident, their empty barriers not yet
    // committed) the half-1 MMAs once half 1 is drained, so the tensor core
    // works through most of the previous tile's epilogue.
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        const int head = min(W_STAGES, p.num_kb);  // k-blocks issued in two passes
        if (!mbar_wait(tempty_bar(0), acc_phase ^ 1u, p.timeout_ns, p.epoch, 2)) break;
        tc_fence_after();
        {
          int st = stage;
          uint32_t ph = phase;
          for (int kb = 0; kb < head; kb++) {
            if (!mbar_wait(full_bar(st), ph, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = stage_a(st);
            const uint64_t adesc = sdesc_sw128_kmajor(sa);
            const uint64_t b0desc = sdesc_sw128_kmajor(sa + A2_BYTES);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; k++) {
              const uint64_t koff = (uint64_t)((k * UMMA_K) >> 4);
              umma_pair<KIND>(sf_tmem, tmem_base, adesc + koff, b0desc + koff, p.idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
            if (++st == W_STAGES) { st = 0; ph ^= 1u; }
          }
        }
        if (!ok) break;
        if (!mbar_wait(tempty_bar(1), acc_phase ^ 1u, p.timeout_ns, p.epoch, 2)) break;
        tc_fence_after();
        for (int kb = 0; kb < head; kb++) {  // same stages, already full
          const uint32_t sa = stage_a(stage);
          const uint64_t adesc = sdesc_sw128_kmajor(sa);
          const uint64_t b1desc = sdesc_sw128_kmajor(sa + A2_BYTES + B2_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; k++) {
            const uint64_t koff = (uint64_t)((k * UMMA_K) >> 4);
            umma_pair<KIND>(sf_tmem, tmem_base + (uint32_t)PAIR_BN, adesc + koff, b1desc + koff, p.idesc1,
                             (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(stage));
          if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
        }
        // the last `tail` k-blocks run in two passes as well: all their half-0
        // MMAs, then half 0 is reported complete (its drain starts), then their
        // half-1 MMAs (stages still resident), then half 1 is complete
        const int tail = min(W_STAGES, p.num_kb - head);
        for (int kb = head; kb < p.num_kb - tail; kb++) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = stage_a(stage);
          const uint64_t adesc = sdesc_sw128_kmajor(sa);
          const uint64_t b0desc = sdesc_sw128_kmajor(sa + A2_BYTES);
          const uint64_t b1desc = sdesc_sw128_kmajor(sa + A2_BYTES + B2_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; k++) {
            const uint64_t koff = (uint64_t)((k * UMMA_K) >> 4);
            umma_pair<KIND>(sf_tmem, tmem_base, adesc + koff, b0desc + koff, p.idesc, 1u);
            umma_pair<KIND>(sf_tmem, tmem_base + (uint32_t)PAIR_BN, adesc + koff, b1desc + koff, p.idesc1, 1u);
          }
          umma_commit_pair(empty_bar(stage));
          if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        {
          int st = stage;
          uint32_t ph = phase;
          for (int t = 0; t < tail; t++) {
            if (!mbar_wait(full_bar(st), ph, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = stage_a(st);
            const uint64_t adesc = sdesc_sw128_kmajor(sa);
            const uint64_t b0desc = sdesc_sw128_kmajor(sa + A2_BYTES);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; k++) {
              const uint64_t koff = (uint64_t)((k * UMMA_K) >> 4);
              umma_pair<KIND>(sf_tmem, tmem_base, adesc + koff, b0desc + koff, p.idesc, 1u);
            }
            if (++st == W_STAGES) { st = 0; ph ^= 1u; }
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(0));
        for (int t = 0; t < tail; t++) {  // same stages, already full
          const uint32_t sa = stage_a(stage);
          const uint64_t adesc = sdesc_sw128_kmajor(sa);
          const uint64_t b1desc = sdesc_sw128_kmajor(sa + A2_BYTES + B2_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; k++) {
            const uint64_t koff = (uint64_t)((k * UMMA_K) >> 4);
            umma_pair<KIND>(sf_tmem, tmem_base + (uint32_t)PAIR_BN, adesc + koff, b1desc + koff, p.idesc1, 1u);
          }
          umma_commit_pair(empty_bar(stage));
          if (++stage == W_STAGES) { stage = 0; phase ^= 1u; }
        }
        umma_commit_pair(tfull_bar(1));
        acc_phase ^= 1u;
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows x 512 columns;
    // warps w and w + 4 share TMEM lane quarter w % 4 and take alternate
    // 32-column chunks
    const int quarter = warp & 3;
    const int e = warp - 2;
    const int sub = e >> 2;
    const int etid = threadIdx.x - 64;
    const uint32_t buf = stg_base + (uint32_t)(e * W_STG_BYTES);
    uint32_t acc_phase = 0;
    const float sa_t = p.sa_rowwise ? 0.0f : (p.sa != nullptr ? __ldg(p.sa) : 1.0f);
    const float sb_t = p.sb_rowwise ? 0.0f : __ldg(p.sb);
    const float sr = p.scale_result ? __ldg(p.scale_result) : 1.0f;
    for (int tile = pair; tile < p.num_tiles; tile += npairs) {
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      wide_epilogue_sync();  // the previous tile's column tables are no longer read
      const int tw = PAIR_BN + p.w_bn1;
      for (int j = etid; j < tw; j += 32 * W_EPI_WARPS) {
        const int col = tn * tw + j;
        const bool in = col < p.N;
        s_scale[j] = in ? (p.sb_rowwise ? __ldg(p.sb + col) : sb_t) : 0.0f;
        s_bias[j] = (in && p.bias != nullptr) ? load_bias(p.bias, p.bias_dtype, col) : 0.0f;
      }
      wide_epilogue_sync();
      const int row0 = tm * (2 * BM) + (int)rank * BM;
      int ok = 1;
#pragma unroll 1
      for (int h = 0; h < 2 && ok; h++) {  // drain each half once it is complete; release it once read
        if (lane == 0) ok = mbar_wait(tfull_bar(h), acc_phase, p.timeout_ns, p.epoch, 4) ? 1 : 0;
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) break;
        tc_fence_after();
        drain_accumulator_tma(p, &tmap_d, tmem_base + (uint32_t)(h * PAIR_BN), row0, tn * tw + h * PAIR_BN,
                              h ? p.w_bn1 : PAIR_BN, quarter, lane, sa_t, s_scale + h * PAIR_BN, s_bias + h * PAIR_BN,
                              sr, buf, sub, 2);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(h), 0));
      }
      if (!ok) break;
      acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait_all();  // this warp's stores are done before its staging memory goes away
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still touch its shared memory
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ small-M kernel
// For few rows of A (decode-time activations, M <= 256) the tiles above leave
// most SMs idle: an M x N output has only ceil(N/256) column tiles. This
// kernel swaps the operands so that the weights fill the MMA's 128 rows:
// TMEM holds D^T for 128 output columns (lanes) x MT rows of A (fp32
// columns, MT = M rounded up to 16, at most 256), computed by
// tcgen05.mma.kind::f8f6f4 with M=128, N=MT, K=32. To fill the GPU when there
// are few column tiles, the K range of each tile is split over a cluster of
// `cs` CTAs (cs in 1, 2, 4, 8); after its MMAs every non-leader CTA writes
// its fp32 partial tile into its own (now idle) shared-memory ring and the
// leader adds the partials through distributed shared memory
// (ld.shared::cluster) before the epilogue. No global scratch, no atomics.
// Roles as in the other kernels: warp 0 TMA producer, warp 1 MMA issuer,
// warps 2-5 epilogue; one tile per cluster.
constexpr int SK_BN = 128;                 // output columns per tile (the MMA's M)
constexpr int SK_B_BYTES = SK_BN * BK;     // 16 KiB of weights per stage
constexpr int SK_MAX_MT = 256;
constexpr int SK_MAX_STAGES = 8;
constexpr int SK_RING_LIMIT = 192 * 1024;  // shared memory for the stage ring
constexpr int SK_SMEM_MAX = SK_RING_LIMIT + 1024 /*align*/ + SK_MAX_MT * 4 /*row scales*/ + 256 /*barriers*/;

constexpr int SK_MAX_CS = 8;               // largest split-K cluster

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// Store four consecutive columns col0..col0+3 of one output row. `full`: all
// four are in range and the row is 16-byte aligned (one vector store).
__device__ __forceinline__ void store_quad(const Params &p, long long row, int col0, const float (&v)[4], bool full) {
  char *base = reinterpret_cast<char *>(p.D);
  const long long off = row * p.ldd + col0;
  switch (p.out_dtype) {
    case FP8B200_BF16:
    case FP8B200_F16: {
      const bool bf = p.out_dtype == FP8B200_BF16;
      const uint32_t w0 = bf ? pack_bf16(v[0], v[1]) : pack_f16(v[0], v[1]);
      const uint32_t w1 = bf ? pack_bf16(v[2], v[3]) : pack_f16(v[2], v[3]);
      uint16_t *d = reinterpret_cast<uint16_t *>(base) + off;
      if (full) {
        *reinterpret_cast<uint2 *>(d) = make_uint2(w0, w1);
      } else {
        const uint32_t w[2] = {w0, w1};
#pragma unroll
        for (int j = 0; j < 4; j++)
          if (col0 + j < p.N) d[j] = (uint16_t)(w[j >> 1] >> (16 * (j & 1)));
      }
      break;
    }
    case FP8B200_F32: {
      float *d = reinterpret_cast<float *>(base) + off;
      if (full) {
        *reinterpret_cast<float4 *>(d) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++)
          if (col0 + j < p.N) d[j] = v[j];
      }
      break;
    }
    default: {
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 4; j++)
        w |= (p.out_dtype == FP8B200_E4M3 ? enc8<FP8B200_E4M3>(v[j]) : enc8<FP8B200_E5M2>(v[j])) << (8 * j);
      uint8_t *d = reinterpret_cast<uint8_t *>(base) + off;
      if (full) {
        *reinterpret_cast<uint32_t *>(d) = w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++)
          if (col0 + j < p.N) d[j] = (uint8_t)(w >> (8 * j));
      }
      break;
    }
  }
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int WF, bool TO_F16>
__device__ __forceinline__ void convert_weight_row(uint32_t raw, uint32_t dst, int r);

// W8 = false: fp8 x fp8 (kind::f8f6f4). W8 = true: float8 weights dequantised
// on load against 16-bit activations (kind::f16): each stage also holds the
// raw 128 x 64-byte weight tile (64-byte swizzle), and the epilogue warps,
// idle until the accumulator is ready, convert it into the MMA's A tile in
// two groups taking alternate k-blocks (CTA-local barriers only).
template <bool W8>
__global__ void __launch_bounds__(THREADS, 1)
scaled_mm_skinny_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  const int MT = p.sk_mt, S = p.sk_stages, CS = p.sk_cs;
  const uint32_t a_bytes = (uint32_t)MT * BK;
  // stage: [weights as the MMA's A (16 KiB) | rows of x (MT x 128 bytes) | W8: raw weights (8 KiB)]
  const uint32_t stage_bytes = SK_B_BYTES + a_bytes + (W8 ? SK_B_BYTES / 2 : 0u);
  float *s_rs = reinterpret_cast<float *>(smem + S * stage_bytes);  // row scales of this tile's MT rows
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_rs + SK_MAX_MT);
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (S + s); };
  const uint32_t tfull = bar_base + 8u * (2 * S);
  auto conv_bar = [&](int s) { return bar_base + 8u * (2 * S + 1 + s); };  // W8: A tile converted
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * S + 1);
  float *part = reinterpret_cast<float *>(smem);  // partial tile [MT][128] fp32, over the drained ring

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = CS > 1 ? cluster_rank() : 0u;
  const int tile = CS > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int tn = tile % p.tiles_n, tm = tile / p.tiles_n;
  const int kb0 = (int)((long long)rank * p.num_kb / CS), kb1 = (int)((long long)(rank + 1) * p.num_kb / CS);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull, 1);
    if (W8)
      for (int s = 0; s < S; s++) mbar_init(conv_bar(s), 2);  // the two warps of one converter group
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.sk_tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);
  // programmatic dependent launch: the next kernel may launch once every CTA
  // is here; this kernel touches global memory only after the previous one
  // has completed (both no-ops without the launch attribute)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  int ok = 1;
  if (warp == 0) {
    // ---------------- TMA producer: this CTA's K range of the tile
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; kb++) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, p.epoch, 1)) break;
        if (p.debug_skip_first_load) break;  // test hook: never fill stage 0
        const uint32_t st = base + (uint32_t)stage * stage_bytes;
        const int kx = kb * p.kb_elems;  // tensor-map coordinate of the k-block
        if (W8) {
          mbar_expect_tx(full_bar(stage), a_bytes + SK_B_BYTES / 2);
          tma_load_2d(st + SK_B_BYTES + a_bytes, &tmap_b, full_bar(stage), kx, tn * SK_BN);  // raw weights
        } else {
          mbar_expect_tx(full_bar(stage), p.tx_bytes);
          tma_load_2d(st, &tmap_b, full_bar(stage), kx, tn * SK_BN);
        }
        tma_load_2d(st + SK_B_BYTES, &tmap_a, full_bar(stage), kx, tm * MT);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: D^T[128 x MT] += B_tile . A_tile^T
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool fine = true;
      for (int kb = kb0; kb < kb1; kb++) {
        // W8: the converters saw the stage land before converting it
        if (!mbar_wait(W8 ? conv_bar(stage) : full_bar(stage), phase, p.timeout_ns, p.epoch, 3)) { fine = false; break; }
        tc_fence_after();
        const uint32_t st = base + (uint32_t)stage * stage_bytes;
        const uint64_t wdesc = sdesc_sw128_kmajor(st);
        const uint64_t xdesc = sdesc_sw128_kmajor(st + SK_B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; k++) {  // 4 MMAs of 32 bytes of K (fp8: K=32, 16-bit: K=16)
          if (W8)
            umma_f16(tmem_base, wdesc + (uint64_t)((k * UMMA_K) >> 4), xdesc + (uint64_t)((k * UMMA_K) >> 4), p.idesc,
                     (kb > kb0 || k > 0) ? 1u : 0u);
          else
            umma_f8f6f4(tmem_base, wdesc + (uint64_t)((k * UMMA_K) >> 4), xdesc + (uint64_t)((k * UMMA_K) >> 4),
                        p.idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(empty_bar(stage));
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      if (fine) umma_commit(tfull);
    }
  } else {
    // ---------------- epilogue, part 1: row scales; wait for the accumulator;
    // every CTA copies its fp32 tile (a partial sum when cs > 1) from TMEM
    // into its drained shared-memory ring as part[row][128 columns]
    const int etid = threadIdx.x - 64;
    if (W8) {
      // ---------------- weight converters during the mainloop: two groups of
      // two warps take alternate k-blocks; each thread converts rows gt, gt + 64
      const int group = (warp - 2) >> 1;
      const int gt = etid - group * 64;
      bool cok = true;
      for (int kb = kb0 + group; kb < kb1 && cok; kb += 2) {
        const int i = kb - kb0;
        const int stage = i % S;
        const uint32_t phase = (uint32_t)(i / S) & 1u;
        int got = 0;
        if (lane == 0) got = mbar_wait(full_bar(stage), phase, p.timeout_ns, p.epoch, 5) ? 1 : 0;
        got = __shfl_sync(0xFFFFFFFFu, got, 0);
        if (!got) { cok = false; break; }
        const uint32_t st = base + (uint32_t)stage * stage_bytes;
        const uint32_t raw = st + SK_B_BYTES + a_bytes;
#pragma unroll
        for (int r = gt; r < SK_BN; r += 64) {
          if (p.act_f16) {
            if (p.w_fp8 == FP8B200_E4M3) convert_weight_row<FP8B200_E4M3, true>(raw, st, r);
            else convert_weight_row<FP8B200_E5M2, true>(raw, st, r);
          } else {
            if (p.w_fp8 == FP8B200_E4M3) convert_weight_row<FP8B200_E4M3, false>(raw, st, r);
            else convert_weight_row<FP8B200_E5M2, false>(raw, st, r);
          }
        }
        fence_proxy_async_smem();  // the tensor core reads these writes through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(conv_bar(stage));
      }
    }
    const float sa_t = p.sa_rowwise ? 0.0f : (p.sa != nullptr ? __ldg(p.sa) : 1.0f);
    for (int t = etid; t < MT; t += 128) {
      const long long row = (long long)tm * MT + t;
      s_rs[t] = p.sa_rowwise ? (row < p.M ? __ldg(p.sa + row) : 0.0f) : sa_t;
    }
    if (lane == 0) ok = mbar_wait(tfull, 0, p.timeout_ns, p.epoch, 4) ? 1 : 0;
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    tc_fence_after();
    if (ok) {
      const int quarter = warp & 3, nl = quarter * 32 + lane;
      const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < MT; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + (uint32_t)c, r);
        tmem_ld_wait(r);
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (c + j < MT) part[(c + j) * SK_BN + nl] = __uint_as_float(r[j]);
      }
    }
  }
  __syncwarp();
  if (CS > 1) cluster_sync();  // every partial tile written; every CTA of the cluster is running
  else __syncthreads();

  if (warp >= 2) {
    // ---------------- epilogue, part 2: CTA `rank` owns rows [r0, r1) of the
    // tile; it sums the cs partial tiles (its own and its peers', through
    // distributed shared memory, 16 bytes per lane), scales, adds the bias
    // and stores. A warp handles one output row at a time: lane l covers
    // columns 4l..4l+3, so a row segment is written with contiguous stores.
    int okw = ok;
    okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
    const int rows_valid = min(MT, p.M - tm * MT);
    const int per = (rows_valid + CS - 1) / CS;
    const int r0 = (int)rank * per, r1 = min(rows_valid, r0 + per);
    const int ew = warp - 2;
    const int c0 = tn * SK_BN + 4 * lane;  // first of this lane's four columns
    float cs4[4], b4[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int col = c0 + j;
      const bool in = col < p.N;
      cs4[j] = in ? (p.sb_rowwise ? __ldg(p.sb + col) : __ldg(p.sb)) : 0.0f;
      b4[j] = (in && p.bias != nullptr) ? load_bias(p.bias, p.bias_dtype, col) : 0.0f;
    }
    const float sr = p.scale_result ? __ldg(p.scale_result) : 1.0f;
    const uint32_t part_addr = smem_u32(part);
    const bool full = p.vec_store && c0 + 4 <= p.N;
#pragma unroll 1
    for (int t = r0 + ew; okw && t < r1; t += 4) {
      const uint32_t off = (uint32_t)((t * SK_BN + 4 * lane) * 4);
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (CS == 1) {
        const float4 a = *reinterpret_cast<const float4 *>(reinterpret_cast<const uint8_t *>(part) + off);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      } else {
        float4 a[SK_MAX_CS];
#pragma unroll
        for (int q = 0; q < SK_MAX_CS; q++)
          if (q < CS) a[q] = ld_cluster_v4(map_to_rank(part_addr + off, (uint32_t)q));
#pragma unroll
        for (int q = 0; q < SK_MAX_CS; q++)
          if (q < CS) { v[0] += a[q].x; v[1] += a[q].y; v[2] += a[q].z; v[3] += a[q].w; }
      }
      const float rs = s_rs[t];
#pragma unroll
      for (int j = 0; j < 4; j++) v[j] = (v[j] * (rs * cs4[j]) + b4[j]) * sr;
      store_quad(p, (long long)tm * MT + t, c0, v, full);
    }
  }

  tc_fence_before();
  __syncwarp();
  if (CS > 1) cluster_sync();  // no CTA leaves while a peer may still read its shared memory
  else __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.sk_tmem_cols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ fp8-weight linear (dequant on load)
// D[M,N] = x[M,K] @ (w[N,K] * w_scale)^T [+ bias] for bf16 or f16 activations x
// and float8 weights w that are never materialised in a wider type in HBM.
// A cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2.kind::f16 (M=256, N=256, K=16): each CTA holds its
// 128 rows of x and converts its 128 of the tile's 256 weight rows, so every
// SM reads only half of the B operand from shared memory (16-bit operands at
// the single-CTA shape would need more shared-memory bandwidth than the SM
// has once the converted tile is also written there). Per CTA, a 6-slot ring
// holds each k-block's x tile (128 rows x 64 values, 128-byte swizzle; TMA,
// completing on the leader's barrier) and raw weight half tile (128 rows x 64
// bytes, 64-byte swizzle; TMA, completing on this CTA's barrier); four groups
// of two converter warps (two weight rows per thread, k-blocks in turn)
// convert the raw rows to the
// activation type (exact, fp8x4_fast), write the 128-byte-swizzled K-major
// half tile into a 4-slot ring, fence it to the async proxy and arrive on the
// leader's `converted` barrier. (The weights come in through TMA, not loads
// into registers: the release of that arrival would otherwise wait for every
// load the thread still has in flight.) The
// leader's MMA thread commits each slot back to both CTAs. The weight scale
// (per tensor or per output channel) and the bias are applied to the fp32
// accumulator in the epilogue, so the weight values enter the products
// exactly. Warps: 0 TMA producer, 1 MMA issuer (leader), 2-5 epilogue,
// 6-13 converters.
constexpr int LW_BK = 64;                          // elements per k-block (128 bytes of 16-bit x)
constexpr int LW_LOADS = 6;                        // x + raw weight ring
constexpr int LW_CONVS = 4;                        // converted-weight ring
constexpr int LW_A_BYTES = BM * LW_BK * 2;         // 16 KiB of x (128 rows)
constexpr int LW_RAW_BYTES = HALF_B * LW_BK;       // 8 KiB of fp8 weights (128 rows)
constexpr int LW_LOAD_BYTES = LW_A_BYTES + LW_RAW_BYTES;
constexpr int LW_W_BYTES = HALF_B * LW_BK * 2;     // 16 KiB of converted weights (128 rows)
constexpr int LW_CONV_WARPS = 8;                   // converter warps
constexpr int LW_GROUPS = 4;                       // converter groups taking k-blocks in turn
constexpr int LW_GROUP_THREADS = 32 * LW_CONV_WARPS / LW_GROUPS;
constexpr int LW_THREADS = 192 + 32 * LW_CONV_WARPS;
constexpr int LW_SMEM_BYTES = LW_LOADS * LW_LOAD_BYTES + LW_CONVS * LW_W_BYTES + 1024 /*align*/ +
                              2 * PAIR_BN * 4 /*column tables*/ + 256;

// Two fp8 codes (low byte = first element) -> two f16 values (low half first).
template <int WF>
__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint32_t two) {
  uint32_t h;
  const uint16_t in = (uint16_t)two;
  if constexpr (WF == FP8B200_E4M3) asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(in));
  else asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h) : "h"(in));
  return h;
}
// f16x2 -> bf16x2 for values with at most 3 significant mantissa bits (exact).
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(__half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu))),
                                                 __half2float(__ushort_as_half((uint16_t)(h >> 16))));
  return *reinterpret_cast<const uint32_t *>(&b);
}

// Fast exact fp8 -> 16-bit conversion of four codes (bytes of w) into the
// pairs (code 0, code 1), (code 2, code 3), without conversion instructions:
// each code's exponent and mantissa bits are placed where the target
// format's sit, its sign at bit 15, and each pair is scaled by a power of two
// (the difference of the exponent biases: e4m3 -> bf16 2^120, e4m3 -> f16
// 2^8, e5m2 -> bf16 2^112) with one packed multiply, which is exact for
// normal and subnormal codes alike. The placement takes one sign-replicating
// byte permute per pair (low byte of each half: the code; high byte: copies
// of its sign bit), one shift (the sign copies land on the sign bit) and one
// mask. Codes with an all-ones exponent (NaN for e4m3; inf / NaN for e5m2
// into bf16) must not come here (see fp8_unit_special); e5m2 -> f16 is a
// byte placement.
template <int WF, bool TO_F16>
__device__ __forceinline__ void fp8x4_fast(uint32_t w, uint32_t &o01, uint32_t &o23) {
  if constexpr (WF == FP8B200_E5M2 && TO_F16) {  // e5m2 is the high byte of an f16
    asm("prmt.b32 %0, %1, 0, 0x1404;" : "=r"(o01) : "r"(w));
    asm("prmt.b32 %0, %1, 0, 0x3424;" : "=r"(o23) : "r"(w));
  } else {
    uint32_t r01, r23;
    asm("prmt.b32 %0, %1, 0, 0x9180;" : "=r"(r01) : "r"(w));  // halves {sign x8, code 0}, {sign x8, code 1}
    asm("prmt.b32 %0, %1, 0, 0xB3A2;" : "=r"(r23) : "r"(w));  // codes 2, 3
    constexpr int SH = WF == FP8B200_E4M3 ? (TO_F16 ? 7 : 4) : 5;
    constexpr uint32_t MASK = WF == FP8B200_E4M3 ? (TO_F16 ? 0xBF80BF80u : 0x87F087F0u) : 0x8FE08FE0u;
    constexpr uint32_t SCALE = WF == FP8B200_E4M3 ? (TO_F16 ? 0x5C005C00u : 0x7B807B80u) : 0x77807780u;
    const uint32_t b01 = (r01 << SH) & MASK, b23 = (r23 << SH) & MASK;
    if constexpr (TO_F16) {
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o01) : "r"(b01), "r"(SCALE));
      asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o23) : "r"(b23), "r"(SCALE));
    } else {
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o01) : "r"(b01), "r"(SCALE));
      asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(o23) : "r"(b23), "r"(SCALE));
    }
  }
}

// Nonzero if any of the 16 codes in q needs the exact path.
template <int WF, bool TO_F16>
__device__ __forceinline__ uint32_t fp8_unit_special(const uint32_t (&q)[4]) {
  if constexpr (WF == FP8B200_E5M2 && TO_F16) return 0u;
  uint32_t any = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    if constexpr (WF == FP8B200_E4M3) any |= ((q[i] & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;  // 0x7F / 0xFF
    else any |= ((q[i] & 0x7C7C7C7Cu) + 0x04040404u) & 0x80808080u;                              // exponent 31
  }
  return any;
}

// Convert row r of a raw weight half tile (64 bytes, 64-byte swizzle: unit c
// at c ^ ((r >> 1) & 3)) into row r of the MMA half tile (64 16-bit values =
// 128 bytes, 128-byte swizzle: unit j at j ^ (r & 7)). Both swizzles put the
// 8 rows a quarter-warp touches in distinct 16-byte bank groups.
template <int WF, bool TO_F16>
__device__ __forceinline__ void convert_weight_row(uint32_t raw, uint32_t dst, int r) {
  uint32_t q[4][4];
#pragma unroll
  for (int c = 0; c < 4; c++)  // all four 16-byte units of the row in flight at once
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(q[c][0]), "=r"(q[c][1]), "=r"(q[c][2]), "=r"(q[c][3])
                 : "r"(raw + (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) * 16))));
  uint32_t o[4][8];
  const bool special = (fp8_unit_special<WF, TO_F16>(q[0]) | fp8_unit_special<WF, TO_F16>(q[1]) |
                        fp8_unit_special<WF, TO_F16>(q[2]) | fp8_unit_special<WF, TO_F16>(q[3])) != 0u;
  if (!special) {
#pragma unroll
    for (int c = 0; c < 4; c++)
#pragma unroll
      for (int i = 0; i < 4; i++) fp8x4_fast<WF, TO_F16>(q[c][i], o[c][2 * i], o[c][2 * i + 1]);
  } else {  // NaN / inf present: conversion instructions
#pragma unroll
    for (int c = 0; c < 4; c++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t lo = fp8x2_to_f16x2<WF>(q[c][i] & 0xFFFFu), hi = fp8x2_to_f16x2<WF>(q[c][i] >> 16);
        o[c][2 * i] = TO_F16 ? lo : f16x2_to_bf16x2(lo);
        o[c][2 * i + 1] = TO_F16 ? hi : f16x2_to_bf16x2(hi);
      }
  }
#pragma unroll
  for (int j = 0; j < 8; j++)  // output unit j = codes 8j .. 8j+7
    st_shared_v4(dst + (uint32_t)(r * 128 + ((j ^ (r & 7)) * 16)), o[j >> 1][4 * (j & 1)],
                 o[j >> 1][4 * (j & 1) + 1], o[j >> 1][4 * (j & 1) + 2], o[j >> 1][4 * (j & 1) + 3]);
}


__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(LW_THREADS, 1)
linear_fp8w_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t *smem = smem_raw + (base - raw_addr);
  // load slot s: [x 16 KiB | raw weights 8 KiB]; then the converted-weight slots (16 KiB); same offsets in both CTAs
  auto sx = [&](int s) { return base + (uint32_t)(s * LW_LOAD_BYTES); };
  auto sraw = [&](int s) { return sx(s) + (uint32_t)LW_A_BYTES; };
  auto sw = [&](int c) { return base + (uint32_t)(LW_LOADS * LW_LOAD_BYTES + c * LW_W_BYTES); };
  float *s_scale = reinterpret_cast<float *>(smem + LW_LOADS * LW_LOAD_BYTES + LW_CONVS * LW_W_BYTES);
  float *s_bias = s_scale + PAIR_BN;
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_bias + PAIR_BN);
  const uint32_t bar_base = smem_u32(bars);
  auto full_bar = [&](int s) { return bar_base + 8u * s; };                                // x of both CTAs (leader)
  auto empty_bar = [&](int s) { return bar_base + 8u * (LW_LOADS + s); };                  // x slot read
  auto conv_bar = [&](int c) { return bar_base + 8u * (2 * LW_LOADS + c); };  // both halves converted (leader)
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * LW_LOADS + LW_CONVS + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * LW_LOADS + LW_CONVS + 2 + b); };
  auto rfull_bar = [&](int s) { return bar_base + 8u * (2 * LW_LOADS + LW_CONVS + 4 + s); };  // raw weights (own)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * LW_LOADS + LW_CONVS + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = (int)cluster_id_x();
  const int npairs = (int)num_clusters_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < LW_LOADS; s++) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(rfull_bar(s), 1);
    }
    for (int c = 0; c < LW_CONVS; c++) mbar_init(conv_bar(c), 2 * LW_CONV_WARPS / LW_GROUPS);  // a group's warps, both CTAs
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 8);  // four epilogue warps in each CTA
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs): this CTA's 128 rows of x
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        const int xrow = tm * (2 * BM) + (int)rank * BM;
        const int wrow = tn * PAIR_BN + (int)rank * HALF_B;
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, p.epoch, 1)) { ok = false; break; }
          if (p.debug_skip_first_load) { ok = false; break; }
          const uint32_t leader_full = map_to_rank(full_bar(stage), 0);
          if (rank == 0) mbar_expect_tx(full_bar(stage), 2 * LW_A_BYTES);
          tma_load_2d_pair(sx(stage), &tmap_x, leader_full, kb * LW_BK, xrow);
          mbar_expect_tx(rfull_bar(stage), LW_RAW_BYTES);
          tma_load_2d(sraw(stage), &tmap_w, rfull_bar(stage), kb * LW_BK, wrow);
          if (++stage == LW_LOADS) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only)
    if (rank == 0 && lane == 0) {
      int stage = 0, cs = 0;
      uint32_t phase = 0, cphase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, p.epoch, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * PAIR_BN);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, p.epoch, 3)) { ok = false; break; }
          if (!mbar_wait(conv_bar(cs), cphase, p.timeout_ns, p.epoch, 7)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sdesc_sw128_kmajor(sx(stage));
          const uint64_t bdesc = sdesc_sw128_kmajor(sw(cs));
#pragma unroll
          for (int k = 0; k < LW_BK / 16; k++)  // K = 16 per MMA: +32 bytes along the swizzled row
            umma_f16_pair(d_tmem, adesc + (uint64_t)((k * 32) >> 4), bdesc + (uint64_t)((k * 32) >> 4), p.idesc,
                          (kb > 0 || k > 0) ? 1u : 0u);
          // x slot free in both CTAs; the converters also take this commit as "converted slot cs free"
          umma_commit_pair(empty_bar(stage));
          if (++stage == LW_LOADS) { stage = 0; phase ^= 1u; }
          if (++cs == LW_CONVS) { cs = 0; cphase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(tfull_bar(acc));
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else if (warp >= 6) {
    // ---------------- weight converters (both CTAs): LW_GROUPS groups take
    // k-blocks in turn, so that several k-blocks' conversions and their
    // fence + arrival latencies overlap; within a group each thread converts
    // rows ctid, ctid + LW_GROUP_THREADS, ... Slots and phases follow a running
    // k-block counter.
    const int group = (threadIdx.x - 192) / LW_GROUP_THREADS;
    const int ctid = threadIdx.x - 192 - group * LW_GROUP_THREADS;
    const uint32_t leader_conv0 = map_to_rank(conv_bar(0), 0);
    uint32_t it = 0;  // k-blocks seen so far (both groups count all of them)
    bool ok = true;
    for (int tile = pair; tile < p.num_tiles && ok; tile += npairs) {
      for (int kb = 0; kb < p.num_kb; kb++, it++) {
        if ((int)(it % LW_GROUPS) != group) continue;
        const int stage = (int)(it % LW_LOADS), cs = (int)(it % LW_CONVS);
        const uint32_t phase = (it / LW_LOADS) & 1u;
        int got = 0;
        if (lane == 0) {
          got = mbar_wait(rfull_bar(stage), phase, p.timeout_ns, p.epoch, 5) ? 1 : 0;
          // converted slot cs was last read by the MMAs of k-block it - LW_CONVS, whose commit completes phase
          // (it - LW_CONVS) / LW_LOADS of x slot (it - LW_CONVS) % LW_LOADS (this group's previous k-block
          // waited for a later commit, so the phase before that one has completed: no early parity match)
          if (got && it >= (uint32_t)LW_CONVS) {
            const uint32_t prev = it - (uint32_t)LW_CONVS;
            got = mbar_wait(empty_bar((int)(prev % LW_LOADS)), (prev / LW_LOADS) & 1u, p.timeout_ns, p.epoch, 6) ? 1 : 0;
          }
        }
        got = __shfl_sync(0xFFFFFFFFu, got, 0);
        if (!got) { ok = false; break; }
#pragma unroll
        for (int r = ctid; r < HALF_B; r += LW_GROUP_THREADS) {
          if (p.act_f16) {
            if (p.w_fp8 == FP8B200_E4M3) convert_weight_row<FP8B200_E4M3, true>(sraw(stage), sw(cs), r);
            else convert_weight_row<FP8B200_E5M2, true>(sraw(stage), sw(cs), r);
          } else {
            if (p.w_fp8 == FP8B200_E4M3) convert_weight_row<FP8B200_E4M3, false>(sraw(stage), sw(cs), r);
            else convert_weight_row<FP8B200_E5M2, false>(sraw(stage), sw(cs), r);
          }
        }
        fence_proxy_async_smem();  // the tensor core reads these writes through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(leader_conv0 + 8u * (uint32_t)cs);
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of the pair tile
    const int quarter = warp & 3;
    const int etid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    const float sb_t = p.sb_rowwise ? 0.0f : __ldg(p.sb);
    const float sr = p.scale_result ? __ldg(p.scale_result) : 1.0f;
    for (int tile = pair; tile < p.num_tiles; tile += npairs) {
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      epilogue_sync();
      stage_columns(p, tn * PAIR_BN, sb_t, s_scale, s_bias, etid);
      epilogue_sync();
      int ok = 0;
      if (lane == 0) ok = mbar_wait(tfull_bar(acc), acc_phase, p.timeout_ns, p.epoch, 4) ? 1 : 0;
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      drain_accumulator(p, tmem_base + (uint32_t)(acc * PAIR_BN), tm * (2 * BM) + (int)rank * BM, tn * PAIR_BN,
                        quarter, lane, 1.0f, s_scale, s_bias, sr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(acc), 0));
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still touch its shared memory
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int encode_kmajor_map(CUtensorMap *m, const void *ptr, int64_t rows, int64_t k, int64_t ld, int box_rows, int fp4);

// Tensor maps describe only an address, extents, a stride and a box, so an
// encoded map stays valid for any later call with the same five values. A
// small per-thread cache skips the driver's encode on repeated calls (the
// decode-time case: the same weights and activation buffers every step).
int make_kmajor_map(CUtensorMap *m, const void *ptr, int64_t rows, int64_t k, int64_t ld, int box_rows,
                    int fp4 = 0) {
  struct Entry { const void *ptr; int64_t rows, k, ld; int box; int dev; int fp4; CUtensorMap map; };
  constexpr int kEntries = 32;
  thread_local Entry cache[kEntries];
  thread_local int used = 0, next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < used; i++) {
    const Entry &e = cache[i];
    if (e.ptr == ptr && e.rows == rows && e.k == k && e.ld == ld && e.box == box_rows && e.dev == dev &&
        e.fp4 == fp4) {
      *m = e.map;
      return FP8B200_OK;
    }
  }
  if (int rc = encode_kmajor_map(m, ptr, rows, k, ld, box_rows, fp4)) return rc;
  int slot;
  if (used < kEntries) {
    slot = used++;
  } else {  // round-robin replacement
    slot = next;
    next = (next + 1) % kEntries;
  }
  cache[slot] = Entry{ptr, rows, k, ld, box_rows, dev, fp4, *m};
  return FP8B200_OK;
}

// K-major operand map: boxes of one 128-byte swizzled row x box_rows rows.
// fp4 = 0: fp8 codes, 128 values per box row, landing as they are.
// fp4 = 1: packed FP4 (e2m1, two values per byte, k-value 2i in the low
// nibble) read as 16U4_ALIGN16B: every 8 bytes (16 values) of a row land in a
// 16-byte unit of shared memory followed by 8 bytes of padding, the layout
// tcgen05.mma kind::f8f6f4 reads 4-bit operands in; 128 values per box row
// again, so the kernels' stage layout and descriptors are the fp8 ones. The
// TMA transaction counts the 64 bytes of packed data per box row, not the
// padding. Requirements (checked by the caller): k a multiple of 128, ld a
// multiple of 32 bytes, a 32-byte aligned base.
// fp4 = 2: packed FP4 kept packed (16U4_ALIGN8B), 256 values per 128-byte box
// row: the operand layout of kind::mxf4.
int encode_kmajor_map(CUtensorMap *m, const void *ptr, int64_t rows, int64_t k, int64_t ld, int box_rows, int fp4) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(FP8B200_ELAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)(fp4 == 2 ? 2 * BK : BK), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = fp4 == 2 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN8B
                                 : fp4 == 1 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUresult r = enc(m, dt, 2,
                   const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FP8B200_EINVAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FP8B200_OK;
}

// Output tensor map for the TMA-store epilogue: rows x cols of esz-byte
// elements, row stride ldd elements, boxes of 32 rows x 64 bytes (32 bytes
// for fp8), swizzle matching the staging layout.
int make_out_map(CUtensorMap *m, void *D, int64_t rows, int64_t cols, int64_t ldd, int esz) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(FP8B200_ELAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ldd * esz)};
  cuuint32_t box[2] = {esz == 4 ? 16u : 32u, 32u};  // 64-byte box rows (32 bytes for fp8)
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : esz == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = esz == 1 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(m, dt, 2, D, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FP8B200_EINVAL, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return FP8B200_OK;
}

// ------------------------------------------------------------------ few-row float8-weight linear
// For M <= 64 activation rows the float8-weight linear is bound by the
// weight bytes and their conversion: every weight is used by at most 64
// rows, so the tcgen05 path's shared-memory hand-off of converted weights
// costs more than the math. This kernel converts weights in registers and
// feeds them straight to the warp-level tensor-core instruction
// mma.sync.m16n8k16 computing D^T = W x^T: 16 weight rows as the A operand,
// 8 x rows as B (NT = 1, 2, 4 or 8 tiles, zero rows past M), float32 accumulators.
//   CTA: 16 NRG output channels (NRG = 4, or 7 where 64-channel CTAs would
//   fill the SMs unevenly: 14336 channels are 224 CTAs of 64, two on 76 of
//   the 148 SMs, or 128 CTAs of 112, one per SM; see gv_plan); a producer
//   warp whose lane 0 streams, per 128-value
//   k-block, the 16 NRG x 128-byte weight tile and the block's x tile
//   (8 NT rows x 128 values, two 128-byte-wide boxes; rows past M are the
//   TMA's zero fill) into a GV_STAGES-deep ring (128-byte swizzle, full /
//   empty mbarriers, bounded waits); 2 NRG consumer warps, two per 16-row
//   group of channels, taking alternate k-blocks, so one warp's conversion
//   and MMAs overlap its partner's shared-memory loads; nothing in the
//   k-loop reads global memory;
//   cluster: ks CTAs splitting K, partial sums reduced through distributed
//   shared memory (each CTA reduces and stores 16 NRG / ks columns), so no
//   global scratch and a fixed summation order; launched with programmatic
//   stream serialization (launch and prologue overlap the previous kernel).
//   k-loop: lane (g, t) reads 32 weight bytes of rows g and 8 + g of its
//   group and 32 x values of x row g (and g + 8). Within a block the lane's
//   32 physical k positions 32t .. 32t+31 are the logical positions {2t,
//   2t+1, 2t+8, 2t+9} of eight consecutive m16n8k16 steps (four positions
//   per step), the same permutation for A and B, which leaves the sum
//   unchanged, and makes both operands' register pairs come straight from
//   the conversions and the 16-byte loads.
constexpr int GV_BK = 128;
// k-blocks in flight per CTA (TMA ring): fewer for 32 or 64 rows of x, whose larger x tiles would
// otherwise keep two 64-channel CTAs off one SM (a deeper ring for the 112-channel CTAs, one per SM,
// measured no faster: those shapes are bound by the conversion, the MMAs and the x reads)
__host__ __device__ constexpr int gv_stages(int nt, int) { return nt <= 2 ? 8 : nt == 4 ? 6 : 4; }
__host__ __device__ constexpr int gv_bn(int nrg) { return 16 * nrg; }          // output channels per CTA
__host__ __device__ constexpr int gv_threads(int nrg) { return 32 * (2 * nrg + 1); }  // consumers + producer
__host__ __device__ constexpr int gv_tile(int nrg) { return gv_bn(nrg) * GV_BK; }  // weight rows x 128 codes
// x tile of a k-block: two 128-byte-wide boxes (values 0-63, 64-127) of 8 NT rows
__host__ __device__ constexpr int gv_x_half(int nt) { return 8 * nt * 128; }
__host__ __device__ constexpr int gv_stage(int nt, int nrg) { return gv_tile(nrg) + 2 * gv_x_half(nt); }
// Partial sums [2 k-block parities][rows][channels]: beside the ring for NT <= 2 (16 rows), inside the
// drained ring for NT > 2 (8 NT rows)
__host__ __device__ constexpr int gv_part_rows(int nt) { return nt <= 2 ? 16 : 8 * nt; }
__host__ __device__ constexpr int gv_smem(int nt, int nrg) {
  return 1024 + gv_stages(nt, nrg) * gv_stage(nt, nrg) + (nt <= 2 ? 2 * 16 * gv_bn(nrg) * 4 : 0) /*partials*/ +
         2 * gv_stages(nt, nrg) * 8 /*barriers*/;
}
static_assert(2 * gv_part_rows(8) * gv_bn(7) * 4 <= gv_stages(8, 7) * gv_stage(8, 7) &&
                  2 * gv_part_rows(4) * gv_bn(7) * 4 <= gv_stages(4, 7) * gv_stage(4, 7) &&
                  2 * gv_part_rows(8) * gv_bn(4) * 4 <= gv_stages(8, 4) * gv_stage(8, 4) &&
                  2 * gv_part_rows(4) * gv_bn(4) * 4 <= gv_stages(4, 4) * gv_stage(4, 4),
              "partial sums fit the drained ring");
static_assert(gv_smem(8, 7) <= 232448 && gv_smem(4, 7) <= 232448 && 2 * (gv_smem(8, 4) + 1024) <= 233472 &&
                  2 * (gv_smem(4, 4) + 1024) <= 233472 && 2 * (gv_smem(2, 4) + 1024) <= 233472,
              "one 112-channel or two 64-channel CTAs per SM");
static_assert(gv_stage(1, 7) % 1024 == 0 && gv_stage(2, 4) % 1024 == 0, "ring stages stay 1 KiB aligned");
struct GvPlan {
  int nrg, ks;  // 16-row groups of channels per CTA, CTAs splitting K
};

template <int WF, bool F16>
__device__ __forceinline__ void gv_convert32(const uint4 (&raw)[2], uint32_t (&o)[16]) {
  const uint32_t q[2][4] = {{raw[0].x, raw[0].y, raw[0].z, raw[0].w}, {raw[1].x, raw[1].y, raw[1].z, raw[1].w}};
  if ((fp8_unit_special<WF, F16>(q[0]) | fp8_unit_special<WF, F16>(q[1])) == 0u) {
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int i = 0; i < 4; i++) fp8x4_fast<WF, F16>(q[h][i], o[8 * h + 2 * i], o[8 * h + 2 * i + 1]);
  } else {  // NaN / inf codes: conversion instructions
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t lo = fp8x2_to_f16x2<WF>(q[h][i] & 0xFFFFu), hi = fp8x2_to_f16x2<WF>(q[h][i] >> 16);
        o[8 * h + 2 * i] = F16 ? lo : f16x2_to_bf16x2(lo);
        o[8 * h + 2 * i + 1] = F16 ? hi : f16x2_to_bf16x2(hi);
      }
  }
}

// 16 codes (one 16-byte unit) -> 8 pairs; o[2i], o[2i+1] = codes 4i, 4i+1 and 4i+2, 4i+3.
template <int WF, bool F16>
__device__ __forceinline__ void gv_convert16(const uint4 &raw, uint32_t (&o)[8]) {
  const uint32_t q[4] = {raw.x, raw.y, raw.z, raw.w};
  if (fp8_unit_special<WF, F16>(q) == 0u) {
#pragma unroll
    for (int i = 0; i < 4; i++) fp8x4_fast<WF, F16>(q[i], o[2 * i], o[2 * i + 1]);
  } else {  // NaN / inf codes: conversion instructions
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t lo = fp8x2_to_f16x2<WF>(q[i] & 0xFFFFu), hi = fp8x2_to_f16x2<WF>(q[i] >> 16);
      o[2 * i] = F16 ? lo : f16x2_to_bf16x2(lo);
      o[2 * i + 1] = F16 ? hi : f16x2_to_bf16x2(hi);
    }
  }
}

template <bool F16>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if constexpr (F16)
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// NT: 8-row tiles of x (1, 2, 4 or 8 for M <= 8, 16, 32, 64); NRG: 16-row groups of channels per CTA
// (4: two CTAs fit on an SM, 7: one)
template <int WF, bool F16, int NT, int NRG>
__global__ void __launch_bounds__(gv_threads(NRG), NRG == 4 ? 2 : 1)
linear_fp8w_gemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                        int M, int N, int kslice, const Params p) {
  extern __shared__ uint8_t gv_raw[];
  constexpr int XH = gv_x_half(NT), ST = gv_stage(NT, NRG), GV_BN = gv_bn(NRG), GV_TILE = gv_tile(NRG);
  constexpr int GV_CONSUMERS = 2 * NRG, GV_STAGES = gv_stages(NT, NRG), PROWS = gv_part_rows(NT);
  const uint32_t raw_addr = smem_u32(gv_raw);
  const uint32_t ring = (raw_addr + 1023u) & ~1023u;  // GV_STAGES x [w tile | x half 0 | x half 1], 1 KiB aligned
  uint8_t *base = gv_raw + (ring - raw_addr);
  float *part = reinterpret_cast<float *>(NT <= 2 ? base + GV_STAGES * ST : base);  // [2][PROWS][GV_BN]
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + GV_STAGES * ST + (NT <= 2 ? 2 * 16 * GV_BN * 4 : 0));
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int st) { return bar0 + 8u * st; };
  auto empty_bar = [&](int st) { return bar0 + 8u * (GV_STAGES + st); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rank = cluster_rank(), ks = p.sk_cs;
  const int n0 = blockIdx.y * GV_BN;
  const int k0 = (int)rank * kslice;
  const int nblk = kslice / GV_BK;

  if (threadIdx.x == 0) {
    for (int st = 0; st < GV_STAGES; st++) {
      mbar_init(full_bar(st), 1);
      mbar_init(empty_bar(st), NRG);  // the warps (one per row group) that read the stage
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  __syncthreads();
  // programmatic dependent launch: the next kernel may launch now; nothing in
  // global memory is read or written before the previous kernel has completed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  float acc[NT][4] = {};
  const int rg = warp % NRG, par = warp / NRG;  // consumers: row group, k-block parity
  if (warp == GV_CONSUMERS) {
    // ---------------- producer: one lane streams the CTA's weight rows and the x rows, one k-block per stage
    if (lane == 0) {
      for (int kb = 0; kb < nblk; kb++) {
        const int st = kb % GV_STAGES;
        const uint32_t ph = (uint32_t)((kb / GV_STAGES) & 1);
        if (!mbar_wait(empty_bar(st), ph ^ 1u, p.timeout_ns, p.epoch, 20)) break;
        if (p.debug_skip_first_load) break;  // test hook: no tile ever lands, the consumers' waits run out
        const uint32_t sa = ring + (uint32_t)(st * ST);
        const int kx = k0 + kb * GV_BK;
        mbar_expect_tx(full_bar(st), (uint32_t)ST);
        tma_load_2d(sa, &tmap_w, full_bar(st), kx, n0);
        tma_load_2d(sa + GV_TILE, &tmap_x, full_bar(st), kx, 0);
        tma_load_2d(sa + GV_TILE + XH, &tmap_x, full_bar(st), kx + 64, 0);
      }
    }
  } else {
    // ---------------- consumers: D^T = W x^T; warp (rg, par) takes k-blocks par, par + 2, ... Its 16
    // weight rows (tile rows 16 rg + g, + 8) are the m16n8k16 A operand, x rows the 8-column B
    // operand (NT tiles: rows 0-7, 8-15). Lane (g, t) reads 16-byte units 2t, 2t + 1 of its two
    // weight rows (unit u of tile row r at u ^ (r & 7): conflict-free), and of x row 8u + g the
    // units 4 (t & 1) .. + 3 of box t >> 1 (same swizzle).
    const uint32_t row_off[2] = {(uint32_t)((16 * rg + g) * 128), (uint32_t)((16 * rg + 8 + g) * 128)};
    const uint32_t unit_off[2] = {(uint32_t)(((2 * t) ^ g) * 16), (uint32_t)(((2 * t + 1) ^ g) * 16)};
    const uint32_t x_off = (uint32_t)(GV_TILE + (t >> 1) * XH + g * 128);
#pragma unroll 1
    for (int kb = par; kb < nblk; kb += 2) {
      const int st = kb % GV_STAGES;
      const uint32_t ph = (uint32_t)((kb / GV_STAGES) & 1);
      const bool landed = mbar_wait(full_bar(st), ph, p.timeout_ns, p.epoch, 21);  // every lane waits (visibility)
      if (!__all_sync(0xFFFFFFFFu, landed)) break;                                // and the warp leaves as one
      const uint32_t tile = ring + (uint32_t)(st * ST);
      uint4 raw[2][2];
#pragma unroll
      for (int h = 0; h < 2; h++)
#pragma unroll
        for (int c = 0; c < 2; c++)
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(raw[h][c].x), "=r"(raw[h][c].y), "=r"(raw[h][c].z), "=r"(raw[h][c].w)
                       : "r"(tile + row_off[h] + unit_off[c]));
      if constexpr (NT <= 2) {
        uint32_t wv[2][16];  // weight rows g and g + 8 converted: the A operand pairs
        gv_convert32<WF, F16>(raw[0], wv[0]);
        gv_convert32<WF, F16>(raw[1], wv[1]);
        uint32_t xv[NT][16];  // x rows g (+ 8): 32 values each, the B operand pairs
#pragma unroll
        for (int u = 0; u < NT; u++)
#pragma unroll
          for (int v = 0; v < 4; v++)
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(xv[u][4 * v]), "=r"(xv[u][4 * v + 1]), "=r"(xv[u][4 * v + 2]), "=r"(xv[u][4 * v + 3])
                         : "r"(tile + x_off + (uint32_t)(u * 1024) + (uint32_t)(((4 * (t & 1) + v) ^ g) * 16)));
        // the stage's bytes are now in registers (the conversions consumed the weights, the MMAs below
        // read only registers): only then may the producer's next TMA overwrite it. The arrival's
        // release, which the producer acquires before it issues that TMA, orders these completed reads
        // before the write (a buffer that is only read needs no proxy fence before its release)
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(st));  // this warp is done with the stage
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
          for (int u = 0; u < NT; u++)
            mma_16816<F16>(acc[u], wv[0][2 * j], wv[1][2 * j], wv[0][2 * j + 1], wv[1][2 * j + 1], xv[u][2 * j],
                           xv[u][2 * j + 1]);
      } else {
        // 32 or 64 x rows: the weights converted 16 codes at a time (k-steps 4 hk .. 4 hk + 3), x read
        // one 16-byte unit per row tile at a time (k-steps 4 hk + 2 kp, + 1), so that the registers
        // hold one unit of every x tile instead of the whole block
#pragma unroll
        for (int hk = 0; hk < 2; hk++) {
          uint32_t wv[2][8];  // weight rows g and g + 8, codes 16 hk .. 16 hk + 15 of the lane
          gv_convert16<WF, F16>(raw[0][hk], wv[0]);
          gv_convert16<WF, F16>(raw[1][hk], wv[1]);
#pragma unroll
          for (int kp = 0; kp < 2; kp++) {
            uint32_t xq[NT][4];  // x rows 8u + g: values 16 (2 hk + kp) .. + 7 of the lane's 32
#pragma unroll
            for (int u = 0; u < NT; u++)
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(xq[u][0]), "=r"(xq[u][1]), "=r"(xq[u][2]), "=r"(xq[u][3])
                           : "r"(tile + x_off + (uint32_t)(u * 1024) +
                                 (uint32_t)(((4 * (t & 1) + 2 * hk + kp) ^ g) * 16)));
            if (hk == 1 && kp == 1) {
              // every read of the stage has returned its value (the conversion and these loads' values are
              // used below only from registers): count this warp out of the stage; the arrival's release
              // orders the reads before the producer's next TMA write into it
              __syncwarp();
              if (lane == 0) mbar_arrive(empty_bar(st));
            }
#pragma unroll
            for (int k2 = 0; k2 < 2; k2++)
#pragma unroll
              for (int u = 0; u < NT; u++) {
                const int i = 2 * kp + k2;
                mma_16816<F16>(acc[u], wv[0][2 * i], wv[1][2 * i], wv[0][2 * i + 1], wv[1][2 * i + 1],
                               xq[u][2 * k2], xq[u][2 * k2 + 1]);
              }
          }
        }
      }
    }
  }

  if constexpr (NT > 2) __syncthreads();  // the ring is drained: the partial sums reuse it
  if (warp < GV_CONSUMERS) {
    // partial sums part[par][x row][channel] (rows < 8 NT, all written): acc[u] = D^T rows
    // (channels) g / g + 8, columns (x rows) 8u + 2t (+1)
    float *pp = part + par * PROWS * GV_BN;
#pragma unroll
    for (int u = 0; u < NT; u++) {
      const int ch = 16 * rg + g, xrow = 8 * u + 2 * t;
      pp[xrow * GV_BN + ch] = acc[u][0];
      pp[(xrow + 1) * GV_BN + ch] = acc[u][1];
      pp[xrow * GV_BN + ch + 8] = acc[u][2];
      pp[(xrow + 1) * GV_BN + ch + 8] = acc[u][3];
    }
  }
  __syncthreads();
  // the two parities' sums, in a fixed order, into part[0]
  for (int i = threadIdx.x; i < 8 * NT * GV_BN; i += blockDim.x) part[i] += part[PROWS * GV_BN + i];
  __syncwarp();
  cluster_sync();  // every CTA's partial sums are complete
  // this CTA reduces and stores columns [rank * cw, (rank + 1) * cw) of the 64
  const int cw = GV_BN / (int)ks;
  const uint32_t part_addr = smem_u32(part);
  for (int i = threadIdx.x; i < M * cw; i += blockDim.x) {
    const int m = i / cw, col = (int)rank * cw + (i - m * cw);
    const int n = n0 + col;
    float v = 0.f;
    for (uint32_t q = 0; q < ks; q++) {
      float pv;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv)
                   : "r"(map_to_rank(part_addr + (uint32_t)((m * GV_BN + col) * 4), q)));
      v += pv;
    }
    if (n < N) {
      const float cs = p.sb_rowwise ? __ldg(p.sb + n) : __ldg(p.sb);
      const float bb = p.bias ? load_bias(p.bias, p.bias_dtype, n) : 0.0f;
      v = v * cs + bb;
      char *d = reinterpret_cast<char *>(p.D);
      const int64_t off = (int64_t)m * p.ldd + n;
      if (p.out_dtype == FP8B200_F32) reinterpret_cast<float *>(d)[off] = v;
      else if (p.out_dtype == FP8B200_BF16) reinterpret_cast<__nv_bfloat16 *>(d)[off] = __float2bfloat16_rn(v);
      else reinterpret_cast<__half *>(d)[off] = __float2half_rn(v);
    }
  }
  cluster_sync();  // no CTA leaves while a peer may still read its partial sums
}

// Test and tuning hooks, per host thread: a hook set by one thread (a test,
// a tuning sweep) never changes the launches of another thread (one thread
// per GPU is the supported threading model).
thread_local unsigned long long g_timeout_ns = 2000000000ull;  // 2 s per wait
thread_local int g_debug_skip_first_load = 0;
thread_local int g_path = 0;  // 0 = by shape, 1 = single-CTA, 2 = CTA-pair 256x256, 3 = small-M, 4 = CTA-pair 256x512

// Launch numbers for the status word (never 0, which means "no failure").
uint32_t next_epoch() {
  static std::atomic<uint32_t> counter{0};
  uint32_t e;
  do e = counter.fetch_add(1, std::memory_order_relaxed) + 1; while (e == 0);
  return e;
}

// Resident 2-CTA clusters of the pair kernel (wide = false) or the wide
// kernel (wide = true) on device `dev`.
int pair_clusters(int dev, bool wide) {
  static std::atomic<int> cached[2][64];  // 0 = not yet queried; concurrent first calls store the same value
  if (dev < 0 || dev >= 64) return 1;
  std::atomic<int> &c = cached[wide ? 1 : 0][dev];
  if (!c.load(std::memory_order_acquire)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(wide ? W_THREADS : THREADS, 1, 1);
    cfg.dynamicSmemBytes = wide ? W_SMEM_BYTES : SMEM2_BYTES;
    int n = 0;
    const cudaError_t e = wide ? cudaOccupancyMaxActiveClusters(&n, scaled_mm_wide_kernel<0>, &cfg)
                               : cudaOccupancyMaxActiveClusters(&n, scaled_mm_pair_kernel, &cfg);
    if (e != cudaSuccess || n < 1) n = current_sm_count() / 2;
    c.store(n, std::memory_order_release);
  }
  return c.load(std::memory_order_acquire);
}

// Tile width of the wide kernel: 512 columns, or 480 (second MMA N = 224)
// where that fills the resident CTA pairs in fewer column-waves: cost =
// waves x width, and 480 must win by 5 % (it moves 7 % more operand bytes
// per flop). 4096^3 and the 1024-8192-row shards of 8192^3: 2 x 480 against
// 2 x 512 (or 1 x 480 against 1 x 512).
int wide_width(int dev, int64_t M, int64_t N) {
  const int64_t slots = pair_clusters(dev, true);
  const int64_t tm = (M + 2 * BM - 1) / (2 * BM);
  auto cost = [&](int64_t w) { return (double)((tm * ((N + w - 1) / w) + slots - 1) / slots) * (double)w; };
  return (N > 480 && cost(480) <= 0.95 * cost(WIDE_BN)) ? 480 : WIDE_BN;
}

// The wide kernel does about twice the work per tile; prefer it unless its
// tile count fills the resident clusters in so few waves that the coarser
// granularity costs more than 10 % against 256 x 256 tiles.
bool prefer_wide(int dev, int64_t M, int64_t N) {
  if (N < WIDE_BN) return false;
  const int64_t slots = pair_clusters(dev, true);
  const int64_t tm = (M + 2 * BM - 1) / (2 * BM);
  const int64_t w = wide_width(dev, M, N);
  const int64_t waves_pair = (tm * ((N + PAIR_BN - 1) / PAIR_BN) + slots - 1) / slots;
  const int64_t waves_wide = (tm * ((N + w - 1) / w) + slots - 1) / slots;
  return (double)(waves_wide * w) <= 1.1 * (double)(waves_pair * PAIR_BN);
}

// Resident clusters of `cs` CTAs of the small-M kernel with `smem` bytes of
// dynamic shared memory on device `dev` (cs == 1: resident CTAs).
template <bool W8>
int skinny_resident(int dev, int cs, int smem) {
  struct Entry { int dev, cs, smem, n; };
  static Entry cache[64];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; i++)
    if (cache[i].dev == dev && cache[i].cs == cs && cache[i].smem == smem) return cache[i].n;
  int n = 0;
  if (cs == 1) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scaled_mm_skinny_kernel<W8>, THREADS, smem) != cudaSuccess)
      per_sm = 1;
    n = std::max(per_sm, 1) * current_sm_count();
  } else {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)cs, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, scaled_mm_skinny_kernel<W8>, &cfg) != cudaSuccess) n = 0;
    cudaGetLastError();  // an unsupported cluster size only disqualifies that size
  }
  if (used < 64) cache[used++] = Entry{dev, cs, smem, n};
  return n;
}

// Split-K cluster size for `tiles` output tiles of `num_kb` k-blocks: the
// size that keeps the most CTAs busy per wave; a larger cluster must gain at
// least 15 % over the best smaller one (the partial reduction is not free).
template <bool W8>
int skinny_cluster_size(int dev, long long tiles, int num_kb, int smem) {
  int best_cs = 1;
  double best = 0.0;
  for (int cs = 1; cs <= 8; cs *= 2) {
    if (cs > num_kb) break;
    const int n = skinny_resident<W8>(dev, cs, smem);
    if (n < 1) continue;
    const long long waves = (tiles + n - 1) / n;
    const double score = (double)(tiles * cs) / (double)waves;
    if (cs == 1 || score > best * 1.15) {
      if (score > best) { best = score; best_cs = cs; }
    }
  }
  return best_cs;
}

// CTA shape of the few-row kernel for an N x K weight matrix: 16 NRG channels
// per CTA and K split over a cluster of ks CTAs. 64-channel CTAs (NRG = 4, two
// fit on an SM) with the smallest split whose CTAs cover every SM once, except
// where those CTAs would fill the SMs unevenly without a split (more CTAs
// than SMs, fewer than two per SM: some SMs then hold two and set the time)
// and 112-channel CTAs (NRG = 7) fit one per SM: then every SM converts at
// most 7 row groups over K instead of 8 (14336 x 4096: 224 CTAs of 64 on 148
// SMs against 128 of 112; measured 20.9 -> 19.8 us at 16 rows). Two 64-channel
// CTAs per SM stream faster than one of either size, so other shapes keep them.
GvPlan gv_plan(int64_t N, int64_t K, int sms) {
  const int64_t nb4 = (N + gv_bn(4) - 1) / gv_bn(4), nb7 = (N + gv_bn(7) - 1) / gv_bn(7);
  int ks = 1;
  while (ks < 8 && K % (GV_BK * 2 * ks) == 0 && nb4 * ks < (int64_t)sms) ks *= 2;
  if (ks == 1 && nb4 > sms && nb4 < 2 * (int64_t)sms && nb7 <= sms) return GvPlan{7, 1};
  return GvPlan{4, ks};
}

}  // namespace gemm
}  // namespace fp8b200

using namespace fp8b200;
using namespace fp8b200::gemm;

extern "C" int fp8b200_scaled_mm(const void *A, int a_dtype, int64_t lda, const void *B, int b_dtype, int64_t ldb,
                                 int64_t M, int64_t N, int64_t K, const float *scale_a, int scale_a_layout,
                                 const float *scale_b, int scale_b_layout, const void *bias, int bias_dtype,
                                 const float *scale_result, void *D, int out_dtype, int64_t ldd, void *stream) {
  auto fp8 = [](int d) { return d == FP8B200_E4M3 || d == FP8B200_E5M2; };
  auto operand = [&](int d) { return fp8(d) || d == FP8B200_E2M1; };
  if (!operand(a_dtype) || !operand(b_dtype))
    return set_error(FP8B200_EINVAL, "scaled_mm: operands must be e4m3fn, e5m2 or e2m1 (packed float4)");
  const bool a4 = a_dtype == FP8B200_E2M1, b4 = b_dtype == FP8B200_E2M1;
  if (out_dtype != FP8B200_F32 && out_dtype != FP8B200_BF16 && out_dtype != FP8B200_F16 && !fp8(out_dtype))
    return set_error(FP8B200_EINVAL, "scaled_mm: unsupported output dtype %d", out_dtype);
  if (M < 0 || N < 0 || K < 0) return set_error(FP8B200_EINVAL, "scaled_mm: negative size");
  if (M == 0 || N == 0) return FP8B200_OK;
  if (K == 0) return set_error(FP8B200_EINVAL, "scaled_mm: K must be positive");
  if (K % 16) return set_error(FP8B200_EINVAL, "scaled_mm: K=%lld must be a multiple of 16", (long long)K);
  if (M > 0x7FFFFFFFLL || N > 0x7FFFFFFFLL || K > 0x7FFFFFFFLL)
    return set_error(FP8B200_EINVAL, "scaled_mm: dimension too large");
  if ((a4 || b4) && K % 128)
    return set_error(FP8B200_EINVAL, "scaled_mm: K=%lld must be a multiple of 128 with a float4 operand", (long long)K);
  // row strides in bytes: K codes per row for float8, K/2 packed bytes for float4
  const int64_t a_row = a4 ? K / 2 : K, b_row = b4 ? K / 2 : K;
  if (lda < a_row || ldb < b_row || (lda % (a4 ? 32 : 16)) || (ldb % (b4 ? 32 : 16)))
    return set_error(FP8B200_EINVAL,
                     "scaled_mm: row strides must cover a row and be multiples of 16 bytes (32 for float4)");
  if (ldd < N) return set_error(FP8B200_EINVAL, "scaled_mm: output row stride < N");
  if (!A || !B || !D || !scale_a || !scale_b) return set_error(FP8B200_EINVAL, "scaled_mm: null pointer");
  if (!aligned16(A) || !aligned16(B)) return set_error(FP8B200_EINVAL, "scaled_mm: operands must be 16-byte aligned");
  if ((a4 && (reinterpret_cast<uintptr_t>(A) & 31)) || (b4 && (reinterpret_cast<uintptr_t>(B) & 31)))
    return set_error(FP8B200_EINVAL, "scaled_mm: float4 operands must be 32-byte aligned");
  if ((scale_a_layout != FP8B200_SCALE_TENSOR && scale_a_layout != FP8B200_SCALE_ROWWISE) ||
      (scale_b_layout != FP8B200_SCALE_TENSOR && scale_b_layout != FP8B200_SCALE_ROWWISE))
    return set_error(FP8B200_EINVAL, "scaled_mm: unknown scale layout");
  if (bias && bias_dtype != FP8B200_F32 && bias_dtype != FP8B200_BF16 && bias_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "scaled_mm: bias must be f32/bf16/f16");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  static std::atomic<bool> attr_done[64];  // set-once flags; concurrent first calls both set the attribute
  if (dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(scaled_mm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(scaled_mm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(scaled_mm_skinny_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SK_SMEM_MAX);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(scaled_mm_wide_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, W_SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(scaled_mm_wide_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, W_SMEM_BYTES);
    if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "scaled_mm: smem attribute: %s", cudaGetErrorString(e));
    attr_done[dev].store(true, std::memory_order_release);
  }

  const bool skinny = g_path == 3 || (g_path == 0 && M <= SK_MAX_MT);
  const bool pair = !skinny && (g_path == 2 || g_path == 4 || (g_path == 0 && M >= 2 * BM && N >= PAIR_BN));
  // the 256x512 kernel stores through an output tensor map: 16-byte aligned output rows only
  const bool out_aligned = aligned16(D) && ((ldd * dtype_size(out_dtype)) % 16 == 0);
  const bool wide = pair && out_aligned && (g_path == 4 || (g_path == 0 && prefer_wide(dev, M, N)));
  // FP4 x FP4 on the CTA-pair 256-row tiles runs as kind::mxf4 (packed operands, K = 64 per
  // MMA at twice the f8f6f4 rate, unit block scales) on 256 x 480 tiles, which leave TMEM
  // columns for the scales; 256-value k-blocks, so K a multiple of 256
  const bool mx = a4 && b4 && wide && K % 256 == 0;
  // small-M kernel: MT rows of A per tile (M rounded up to 16, at most 256)
  const int mt = skinny ? (int)std::min<int64_t>(SK_MAX_MT, (M + 15) / 16 * 16) : 0;
  CUtensorMap ma, mb;
  const int a_box = skinny ? mt : BM, b_box = skinny ? SK_BN : (pair ? HALF_B : BN);
  const int a_mode = mx ? 2 : (a4 ? 1 : 0), b_mode = mx ? 2 : (b4 ? 1 : 0);
  if (int rc = make_kmajor_map(&ma, A, M, K, lda, a_box, a_mode)) return rc;
  if (int rc = make_kmajor_map(&mb, B, N, K, ldb, b_box, b_mode)) return rc;

  Params p;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  const int kb_elems = mx ? 2 * BK : BK;  // k-values per 128-byte smem row
  p.num_kb = (int)((K + kb_elems - 1) / kb_elems);
  if (skinny) {
    p.tiles_m = (int)((M + mt - 1) / mt);
    p.tiles_n = (int)((N + SK_BN - 1) / SK_BN);
  } else {
    p.tiles_m = (int)((M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
    const int tw = mx ? 480 : wide ? wide_width(dev, M, N) : BN;
    p.tiles_n = (int)((N + tw - 1) / tw);
  }
  p.w_bn1 = mx ? 480 - PAIR_BN : wide ? wide_width(dev, M, N) - PAIR_BN : 0;
  if ((long long)p.tiles_m * p.tiles_n > 0x7FFFFFFFLL / 8) return set_error(FP8B200_EINVAL, "scaled_mm: too many tiles");
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.sa = scale_a; p.sb = scale_b;
  p.sa_rowwise = scale_a_layout == FP8B200_SCALE_ROWWISE;
  p.sb_rowwise = scale_b_layout == FP8B200_SCALE_ROWWISE;
  p.bias = bias; p.bias_dtype = bias_dtype;
  p.scale_result = scale_result;
  p.D = D; p.ldd = ldd; p.out_dtype = out_dtype;
  const int esz = dtype_size(out_dtype);
  p.vec_store = out_aligned;
  // kind::f8f6f4 operand formats: 0 e4m3, 1 e5m2, 5 e2m1
  auto mma_fmt = [](int d) { return d == FP8B200_E5M2 ? 1u : d == FP8B200_E2M1 ? 5u : 0u; };
  const uint32_t afmt = mma_fmt(a_dtype), bfmt = mma_fmt(b_dtype);
  // TMA bytes per stage: a box row carries 128 bytes of float8 or 64 bytes of packed float4; the CTA
  // pairs credit both CTAs' loads to the leader's barrier
  const uint32_t a_rb = (a4 && !mx) ? 64u : 128u, b_rb = (b4 && !mx) ? 64u : 128u;
  p.tx_bytes = (uint32_t)a_box * a_rb + (uint32_t)b_box * b_rb + (wide ? (uint32_t)(p.w_bn1 / 2) * b_rb : 0u);
  if (pair) p.tx_bytes *= 2u;
  // instruction descriptor: f32 accumulate, A/B formats, both K-major, N>>3, M>>4
  const uint32_t mma_m = pair ? 2 * BM : BM;
  p.idesc = (1u << 4) | (afmt << 7) | (bfmt << 10) | ((uint32_t)(BN >> 3) << 17) | ((mma_m >> 4) << 24);
  p.idesc1 = (1u << 4) | (afmt << 7) | (bfmt << 10) | ((uint32_t)(p.w_bn1 >> 3) << 17) | ((mma_m >> 4) << 24);
  if (mx) {
    // block-scaled descriptor: A/B format 1 (e2m1, kind::mxf4), scale format 1 (UE8M0) at bit 23,
    // scale-factor ids 0, dense K = 64; no accumulator-format field (always f32)
    p.idesc = (1u << 7) | (1u << 10) | ((uint32_t)(PAIR_BN >> 3) << 17) | (1u << 23) | ((mma_m >> 4) << 24);
    p.idesc1 = (1u << 7) | (1u << 10) | ((uint32_t)(p.w_bn1 >> 3) << 17) | (1u << 23) | ((mma_m >> 4) << 24);
  }
  p.timeout_ns = g_timeout_ns;
  p.epoch = next_epoch();
  p.debug_skip_first_load = g_debug_skip_first_load;
  p.sk_mt = mt;
  p.kb_elems = kb_elems;
  p.sk_stages = p.sk_cs = p.sk_tmem_cols = 0;
  p.tma_store = 0;
  CUtensorMap md;
  memset(&md, 0, sizeof(md));
  CUtensorMap mb1 = mb;  // the wide kernel's second B block: w_bn1 / 2 rows per CTA
  if (wide) {
    if (int rc = make_out_map(&md, D, M, N, ldd, esz)) return rc;
    p.tma_store = 1;
    if (p.w_bn1 != PAIR_BN)
      if (int rc = make_kmajor_map(&mb1, B, N, K, ldb, p.w_bn1 / 2, b_mode)) return rc;
  }
  int sk_smem = 0;
  if (skinny) {
    // swapped operands: the weights (B) are the MMA's A (M=128), the rows of A its N (= mt)
    p.idesc = (1u << 4) | (bfmt << 7) | (afmt << 10) | ((uint32_t)(mt >> 3) << 17) | ((uint32_t)(SK_BN >> 4) << 24);
    const int stage_bytes = SK_B_BYTES + mt * BK;
    p.sk_stages = std::min(SK_MAX_STAGES, SK_RING_LIMIT / stage_bytes);
    int cols = 32;
    while (cols < mt) cols *= 2;
    p.sk_tmem_cols = cols;
    sk_smem = p.sk_stages * stage_bytes + 1024 + SK_MAX_MT * 4 + 256;
  }

  if (skinny) {
    p.sk_cs = skinny_cluster_size<false>(dev, p.num_tiles, p.num_kb, sk_smem);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.sk_cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(p.num_tiles * p.sk_cs), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)sk_smem;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = p.sk_cs > 1 ? 2 : 1;
    cudaLaunchKernelEx(&cfg, scaled_mm_skinny_kernel<false>, ma, mb, p);
  } else if (wide) {
    const int clusters = std::min(p.num_tiles, pair_clusters(dev, true));
    if (mx) scaled_mm_wide_kernel<2><<<2 * clusters, W_THREADS, W_SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, mb1, md, p);
    else scaled_mm_wide_kernel<0><<<2 * clusters, W_THREADS, W_SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, mb1, md, p);
  } else if (pair) {
    const int clusters = std::min(p.num_tiles, pair_clusters(dev, false));
    scaled_mm_pair_kernel<<<2 * clusters, THREADS, SMEM2_BYTES, (cudaStream_t)stream>>>(ma, mb, p);
  } else {
    const int grid = std::min(p.num_tiles, current_sm_count());
    scaled_mm_kernel<<<grid, THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, p);
  }
  count_launch();
  return check_launch("scaled_mm");
}

extern "C" int fp8b200_gemm_status(uint32_t *status_out, int reset) {
  unsigned long long w = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&w, g_status, sizeof(w));
  if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "gemm status read: %s", cudaGetErrorString(e));
  const uint32_t v = (uint32_t)w;  // the site code; the launch epoch is internal
  if (status_out) *status_out = v;
  if (reset) {
    const unsigned long long z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "gemm status reset: %s", cudaGetErrorString(e));
  }
  return v ? FP8B200_ETIMEOUT : FP8B200_OK;
}

extern "C" int fp8b200_debug_gemm(int skip_first_load, unsigned long long wait_timeout_ns) {
  g_debug_skip_first_load = skip_first_load ? 1 : 0;
  g_timeout_ns = wait_timeout_ns ? wait_timeout_ns : 2000000000ull;
  return FP8B200_OK;
}

extern "C" int fp8b200_gemm_set_path(int path) {
  if (path < 0 || path > 4) return set_error(FP8B200_EINVAL, "gemm path must be 0 (auto), 1, 2, 3 or 4");
  g_path = path;
  return FP8B200_OK;
}

namespace fp8b200 {
namespace gemm {
// 2-D tensor map of `outer` rows x `inner` elements (row pitch ld_bytes) with
// the given box and swizzle; no caching (used by the fp8-weight linear).
int make_map_2d(CUtensorMap *m, const void *ptr, CUtensorMapDataType dt, int64_t inner, int64_t outer,
                int64_t ld_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_error(FP8B200_ELAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FP8B200_EINVAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FP8B200_OK;
}
}  // namespace gemm
}  // namespace fp8b200

extern "C" int fp8b200_linear_fp8w(const void *x, int x_dtype, int64_t ldx, const void *w, int w_dtype, int64_t ldw,
                                   int64_t M, int64_t N, int64_t K, const float *w_scale, int w_scale_layout,
                                   const void *bias, int bias_dtype, void *D, int out_dtype, int64_t ldd,
                                   void *stream) {
  if (x_dtype != FP8B200_BF16 && x_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "linear_fp8w: activations must be bf16 or f16");
  if (w_dtype != FP8B200_E4M3 && w_dtype != FP8B200_E5M2)
    return set_error(FP8B200_EINVAL, "linear_fp8w: weights must be e4m3fn or e5m2");
  if (out_dtype != FP8B200_F32 && out_dtype != FP8B200_BF16 && out_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "linear_fp8w: output must be f32, bf16 or f16");
  if (M < 0 || N < 0 || K < 0) return set_error(FP8B200_EINVAL, "linear_fp8w: negative size");
  if (M == 0 || N == 0) return FP8B200_OK;
  if (K == 0) return set_error(FP8B200_EINVAL, "linear_fp8w: K must be positive");
  if (M > 0x7FFFFFFFLL || N > 0x7FFFFFFFLL || K > 0x7FFFFFFFLL)
    return set_error(FP8B200_EINVAL, "linear_fp8w: dimension too large");
  if (ldx < K || ldw < K || ldx % 8 || ldw % 16)
    return set_error(FP8B200_EINVAL, "linear_fp8w: row strides must be >= K and 16-byte multiples");
  if (ldd < N) return set_error(FP8B200_EINVAL, "linear_fp8w: output row stride < N");
  if (!x || !w || !D || !w_scale) return set_error(FP8B200_EINVAL, "linear_fp8w: null pointer");
  if (!aligned16(x) || !aligned16(w)) return set_error(FP8B200_EINVAL, "linear_fp8w: x and w must be 16-byte aligned");
  if (w_scale_layout != FP8B200_SCALE_TENSOR && w_scale_layout != FP8B200_SCALE_ROWWISE)
    return set_error(FP8B200_EINVAL, "linear_fp8w: unknown weight-scale layout");
  if (bias && bias_dtype != FP8B200_F32 && bias_dtype != FP8B200_BF16 && bias_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "linear_fp8w: bias must be f32/bf16/f16");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  static std::atomic<bool> attr_done[64];  // set-once flags; concurrent first calls both set the attribute
  if (dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(linear_fp8w_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LW_SMEM_BYTES);
    if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "linear_fp8w: smem attribute: %s", cudaGetErrorString(e));
    attr_done[dev].store(true, std::memory_order_release);
  }
  if (M <= 64 && K % GV_BK == 0 && K <= 0x7FFFFFFFLL - GV_BK && g_path != 3) {
    // very few rows: weights and x streamed by TMA, weights converted in registers for warp-level
    // MMAs; CTAs of 64 or 112 channels, K split over a cluster of ks CTAs (gv_plan: each K slice a
    // multiple of the 128-value block)
    const int nt = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8;  // 8-row tiles of x
    const bool f16 = x_dtype == FP8B200_F16;
    using GvKernel = void (*)(const CUtensorMap, const CUtensorMap, int, int, int, const Params);
#define GV_K(WF, F16, NT) linear_fp8w_gemv_kernel<WF, F16, NT, 4>, linear_fp8w_gemv_kernel<WF, F16, NT, 7>
#define GV_K4(WF, F16) GV_K(WF, F16, 1), GV_K(WF, F16, 2), GV_K(WF, F16, 4), GV_K(WF, F16, 8)
    static const GvKernel kernels[32] = {GV_K4(FP8B200_E4M3, false), GV_K4(FP8B200_E4M3, true),
                                         GV_K4(FP8B200_E5M2, false), GV_K4(FP8B200_E5M2, true)};
#undef GV_K4
#undef GV_K
    auto kindex = [&](int nrg) {
      const int nti = nt == 1 ? 0 : nt == 2 ? 1 : nt == 4 ? 2 : 3;
      return (w_dtype == FP8B200_E4M3 ? 0 : 16) + (f16 ? 8 : 0) + 2 * nti + (nrg == 7 ? 1 : 0);
    };
    const GvPlan plan = gv_plan(N, K, current_sm_count());
    const int nrg = plan.nrg, ks = plan.ks;
    const int64_t nb = (N + gv_bn(nrg) - 1) / gv_bn(nrg);
    const int64_t kslice = K / ks;
    const int64_t smem = gv_smem(nt, nrg);
    if (nb <= 65535) {
      CUtensorMap mw, mx;
      if (int rc = make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, GV_BK, (uint32_t)gv_bn(nrg),
                               CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
      // x: M rows of K 16-bit values; boxes of 64 values x 8 NT rows (rows past M read as zeros)
      if (int rc = make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_UINT16, K, M, ldx * 2, 64, (uint32_t)(8 * nt),
                               CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
      Params p;
      memset(&p, 0, sizeof(p));
      p.M = (int)M; p.N = (int)N; p.K = (int)K;
      p.sb = w_scale; p.sb_rowwise = w_scale_layout == FP8B200_SCALE_ROWWISE;
      p.bias = bias; p.bias_dtype = bias_dtype;
      p.D = D; p.ldd = ldd; p.out_dtype = out_dtype;
      p.sk_cs = ks;
      p.timeout_ns = g_timeout_ns;
      p.epoch = next_epoch();
      p.debug_skip_first_load = g_debug_skip_first_load;
      const int ki = kindex(nrg);
      const GvKernel kern = kernels[ki];
      {  // dynamic shared-memory limit per kernel, only ever raised
        static std::mutex mu;
        static int limit[32][64] = {};
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && limit[ki][dev] < smem) {
          cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "linear_fp8w: smem attribute: %s", cudaGetErrorString(e));
          limit[ki][dev] = (int)smem;
        }
      }
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)ks;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.gridDim = dim3((unsigned)ks, (unsigned)nb, 1);
      cfg.blockDim = dim3((unsigned)gv_threads(nrg), 1, 1);
      cfg.dynamicSmemBytes = (size_t)smem;
      cfg.stream = (cudaStream_t)stream;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      cudaLaunchKernelEx(&cfg, kern, mw, mx, (int)M, (int)N, (int)kslice, p);
      count_launch();
      return check_launch("linear_fp8w");
    }
  }
  // 16 < M <= 256: the small-M kernel (K split over a cluster) unless the CTA-pair kernel's
  // 256-wide column tiles alone occupy at least half of the resident CTA pairs (large N),
  // where its four converter groups move the weights faster (N = 14336: 52 against 92 us)
  const bool pair_mid = M > 16 && (N + PAIR_BN - 1) / PAIR_BN >= (int64_t)(pair_clusters(dev, false) / 2) &&
                        g_path != 3;
  if (M <= SK_MAX_MT && !pair_mid) {
    // few rows: the small-M kernel with weights dequantised on load (128
    // weight rows per tile on the MMA's M, K split over a cluster)
    static std::atomic<bool> sk_attr[64];
    if (dev < 64 && !sk_attr[dev].load(std::memory_order_acquire)) {
      cudaError_t e = cudaFuncSetAttribute(scaled_mm_skinny_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           SK_SMEM_MAX);
      if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "linear_fp8w: smem attribute: %s", cudaGetErrorString(e));
      sk_attr[dev].store(true, std::memory_order_release);
    }
    const int mt = (int)((M + 15) / 16 * 16);
    CUtensorMap mx, mw;
    if (int rc = make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_UINT16, K, M, ldx * 2, LW_BK, mt, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, LW_BK, SK_BN, CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
    Params p;
    memset(&p, 0, sizeof(p));
    p.M = (int)M; p.N = (int)N; p.K = (int)K;
    p.kb_elems = LW_BK;
    p.num_kb = (int)((K + LW_BK - 1) / LW_BK);
    p.tiles_m = 1;
    p.tiles_n = (int)((N + SK_BN - 1) / SK_BN);
    p.num_tiles = p.tiles_n;
    p.sa = nullptr; p.sa_rowwise = 0;
    p.sb = w_scale; p.sb_rowwise = w_scale_layout == FP8B200_SCALE_ROWWISE;
    p.bias = bias; p.bias_dtype = bias_dtype;
    p.D = D; p.ldd = ldd; p.out_dtype = out_dtype;
    p.vec_store = aligned16(D) && ((ldd * dtype_size(out_dtype)) % 16 == 0);
    p.w_fp8 = w_dtype;
    p.act_f16 = x_dtype == FP8B200_F16;
    const uint32_t fmt = p.act_f16 ? 0u : 1u;
    p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(mt >> 3) << 17) | ((uint32_t)(SK_BN >> 4) << 24);
    p.timeout_ns = g_timeout_ns;
    p.epoch = next_epoch();
    p.debug_skip_first_load = g_debug_skip_first_load;
    p.sk_mt = mt;
    const int stage_bytes = SK_B_BYTES + mt * BK + SK_B_BYTES / 2;
    // This path is bound by the converters' hand-off latency, not by ring
    // depth: a ring of about 104 KiB lets two CTAs share an SM (more k-block
    // streams at once), as long as it still holds the fp32 partial tile.
    const int need = (mt * SK_BN * 4 + stage_bytes - 1) / stage_bytes;
    p.sk_stages = std::max(need, std::min(SK_MAX_STAGES, (104 * 1024) / stage_bytes));
    p.sk_stages = std::max(p.sk_stages, 2);
    int cols = 32;
    while (cols < mt) cols *= 2;
    p.sk_tmem_cols = cols;
    const int sk_smem = p.sk_stages * stage_bytes + 1024 + SK_MAX_MT * 4 + 256;
    p.sk_cs = skinny_cluster_size<true>(dev, p.num_tiles, p.num_kb, sk_smem);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.sk_cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(p.num_tiles * p.sk_cs), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = (size_t)sk_smem;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = p.sk_cs > 1 ? 2 : 1;
    cudaLaunchKernelEx(&cfg, scaled_mm_skinny_kernel<true>, mx, mw, p);
    count_launch();
    return check_launch("linear_fp8w");
  }
  CUtensorMap mx, mw;
  if (int rc = make_map_2d(&mx, x, CU_TENSOR_MAP_DATA_TYPE_UINT16, K, M, ldx * 2, LW_BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = make_map_2d(&mw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, ldw, LW_BK, HALF_B, CU_TENSOR_MAP_SWIZZLE_64B))
    return rc;
  Params p;
  memset(&p, 0, sizeof(p));
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.num_kb = (int)((K + LW_BK - 1) / LW_BK);
  p.tiles_m = (int)((M + 2 * BM - 1) / (2 * BM));
  p.tiles_n = (int)((N + PAIR_BN - 1) / PAIR_BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.sa = nullptr; p.sa_rowwise = 0;
  p.sb = w_scale; p.sb_rowwise = w_scale_layout == FP8B200_SCALE_ROWWISE;
  p.bias = bias; p.bias_dtype = bias_dtype;
  p.scale_result = nullptr;
  p.D = D; p.ldd = ldd; p.out_dtype = out_dtype;
  p.vec_store = aligned16(D) && ((ldd * dtype_size(out_dtype)) % 16 == 0);
  p.w_fp8 = w_dtype;
  p.act_f16 = x_dtype == FP8B200_F16;
  const uint32_t fmt = p.act_f16 ? 0u : 1u;  // kind::f16 operand type: 0 = f16, 1 = bf16
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(PAIR_BN >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
  p.timeout_ns = g_timeout_ns;
  p.epoch = next_epoch();
  p.debug_skip_first_load = g_debug_skip_first_load;
  const int clusters = std::min(p.num_tiles, current_sm_count() / 2);
  linear_fp8w_kernel<<<2 * clusters, LW_THREADS, LW_SMEM_BYTES, (cudaStream_t)stream>>>(mx, mw, p);
  count_launch();
  return check_launch("linear_fp8w");
}

extern "C" int fp8b200_gemm_16bit(const void *A, const void *B, int dtype, int64_t lda, int64_t ldb, int64_t M,
                                  int64_t N, int64_t K, const float *scale_b, int scale_b_layout, const void *bias,
                                  int bias_dtype, void *D, int out_dtype, int64_t ldd, void *stream) {
  if (dtype != FP8B200_BF16 && dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "gemm_16bit: operands must be bf16 or f16");
  if (out_dtype != FP8B200_F32 && out_dtype != FP8B200_BF16 && out_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "gemm_16bit: output must be f32, bf16 or f16");
  if (M < 0 || N < 0 || K < 0) return set_error(FP8B200_EINVAL, "gemm_16bit: negative size");
  if (M == 0 || N == 0) return FP8B200_OK;
  if (K == 0) return set_error(FP8B200_EINVAL, "gemm_16bit: K must be positive");
  if (M > 0x7FFFFFFFLL || N > 0x7FFFFFFFLL || K > 0x7FFFFFFFLL)
    return set_error(FP8B200_EINVAL, "gemm_16bit: dimension too large");
  if (lda < K || ldb < K || lda % 8 || ldb % 8)
    return set_error(FP8B200_EINVAL, "gemm_16bit: row strides must be >= K and multiples of 8 elements");
  if (ldd < N) return set_error(FP8B200_EINVAL, "gemm_16bit: output row stride < N");
  if (!A || !B || !D || !scale_b) return set_error(FP8B200_EINVAL, "gemm_16bit: null pointer");
  if (!aligned16(A) || !aligned16(B)) return set_error(FP8B200_EINVAL, "gemm_16bit: operands must be 16-byte aligned");
  const int esz = dtype_size(out_dtype);
  if (!aligned16(D) || (ldd * esz) % 16)
    return set_error(FP8B200_EINVAL, "gemm_16bit: output rows must be 16-byte aligned");
  if (scale_b_layout != FP8B200_SCALE_TENSOR && scale_b_layout != FP8B200_SCALE_ROWWISE)
    return set_error(FP8B200_EINVAL, "gemm_16bit: unknown scale layout");
  if (bias && bias_dtype != FP8B200_F32 && bias_dtype != FP8B200_BF16 && bias_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "gemm_16bit: bias must be f32/bf16/f16");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  static std::atomic<bool> attr_done[64];  // set-once flags; concurrent first calls both set the attribute
  if (dev < 64 && !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(scaled_mm_wide_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         W_SMEM_BYTES);
    if (e != cudaSuccess) return set_error(FP8B200_ELAUNCH, "gemm_16bit: smem attribute: %s", cudaGetErrorString(e));
    attr_done[dev].store(true, std::memory_order_release);
  }
  CUtensorMap ma, mb, md;
  if (int rc = make_map_2d(&ma, A, CU_TENSOR_MAP_DATA_TYPE_UINT16, K, M, lda * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = make_map_2d(&mb, B, CU_TENSOR_MAP_DATA_TYPE_UINT16, K, N, ldb * 2, 64, HALF_B,
                           CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int rc = make_out_map(&md, D, M, N, ldd, esz)) return rc;
  Params p;
  memset(&p, 0, sizeof(p));
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.kb_elems = 64;
  p.tx_bytes = 2 * W_STAGE_BYTES;
  p.num_kb = (int)((K + 63) / 64);
  p.tiles_m = (int)((M + 2 * BM - 1) / (2 * BM));
  p.tiles_n = (int)((N + WIDE_BN - 1) / WIDE_BN);
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.sa = nullptr; p.sa_rowwise = 0;
  p.sb = scale_b; p.sb_rowwise = scale_b_layout == FP8B200_SCALE_ROWWISE;
  p.bias = bias; p.bias_dtype = bias_dtype;
  p.D = D; p.ldd = ldd; p.out_dtype = out_dtype;
  p.vec_store = 1;
  p.tma_store = 1;
  const uint32_t fmt = dtype == FP8B200_BF16 ? 1u : 0u;
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(PAIR_BN >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
  p.w_bn1 = PAIR_BN;
  p.idesc1 = p.idesc;
  p.timeout_ns = g_timeout_ns;
  p.epoch = next_epoch();
  p.debug_skip_first_load = g_debug_skip_first_load;
  const int clusters = std::min(p.num_tiles, pair_clusters(dev, true));
  scaled_mm_wide_kernel<1><<<2 * clusters, W_THREADS, W_SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, mb, md, p);
  count_launch();
  return check_launch("gemm_16bit");
}

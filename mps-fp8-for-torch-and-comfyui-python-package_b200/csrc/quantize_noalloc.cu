// Allocation-free per-tensor FP8 quantisation.
//
// fp8b200_quantize_fp8 needs one word of device scratch (the amax
// accumulator) that its caller must allocate. Some callers cannot allocate
// device memory at the point where they quantise: a host runtime or plugin
// ABI that owns a fixed device arena and only hands this library the tensors
// it should read and write, or code that must not enter the CUDA allocator on
// that path. For them, fp8b200_quantize_fp8_noalloc keeps its scratch in a
// fixed array in this library's own device memory instead.
//
// Scratch layout: one max-|x| partial per slice of input elements, kSlices
// slots (16 KiB). A call's slice length is the smallest multiple of
// kSliceUnit that needs at most kSlices slices (4096 elements up to 2^24
// elements, growing to kMaxSliceElems at the limit), so small inputs still
// spread over many blocks. Every slot a call reads was written
// earlier in the same call, so nothing has to be cleared between calls; the
// array keeps the last call's partials. Two calls that run at the same time
// on the GPU (different streams, or different host threads) share the array
// and race: serialise them.
#include "common.cuh"

#include <cuda_fp16.h>

#include <algorithm>


namespace fp8b200 {
namespace noalloc {

constexpr int64_t kSliceUnit = 4096;       // slice lengths are multiples of this (16-byte aligned slices)
constexpr int64_t kMaxSliceElems = 65536;
constexpr int kSlices = 4096;
constexpr int64_t kMaxElems = kMaxSliceElems * kSlices;  // 2^28 elements
constexpr int kThreads = 256;

// The scratch. In host code this name is only a stand-in for the symbol: the
// device address comes from cudaGetSymbolAddress (scratch_ptr below).
static __device__ __align__(256) uint32_t g_amax_partials[kSlices];

template <int SRC>
__device__ __forceinline__ uint32_t abs_bits(const void *src, int64_t i) {
  if constexpr (SRC == FP8B200_F32) {
    return reinterpret_cast<const uint32_t *>(src)[i] & 0x7FFFFFFFu;
  } else if constexpr (SRC == FP8B200_BF16) {
    return ((uint32_t)reinterpret_cast<const uint16_t *>(src)[i] << 16) & 0x7FFFFFFFu;
  } else {
    const float f = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t *>(src)[i]));
    return __float_as_uint(f) & 0x7FFFFFFFu;
  }
}

// |x| bits of the 16-byte unit q: f32 as float bits; 16-bit formats as their
// own magnitude bits (bf16 << 16 is its float; f16 bits order like values,
// NaN above inf), converted to float bits once per thread at the end.
template <int SRC>
__device__ __forceinline__ uint32_t unit_abs_max(const uint4 q) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if constexpr (SRC == FP8B200_F32) {
      m = max(m, w[j] & 0x7FFFFFFFu);
    } else {
      m = max(m, max(w[j] & 0x7FFFu, (w[j] >> 16) & 0x7FFFu));
    }
  }
  return m;
}

template <int SRC>
__device__ __forceinline__ uint32_t to_float_bits(uint32_t m16_or_f32) {
  if constexpr (SRC == FP8B200_F32) return m16_or_f32;
  else if constexpr (SRC == FP8B200_BF16) return m16_or_f32 << 16;
  else return __float_as_uint(__half2float(__ushort_as_half((uint16_t)m16_or_f32))) & 0x7FFFFFFFu;
}

// One block per slice: partials[b] = max |x| over slice b, as float bits
// (NaN sorts above inf, so a NaN anywhere wins, as in the allocating path).
// VEC: 16-byte loads, four in flight per thread (the slice starts on a
// 16-byte boundary when src does: a multiple of 4096 elements), scalar
// loads for the last partial unit; otherwise element by element.
template <int SRC, bool VEC>
__global__ void __launch_bounds__(kThreads)
slice_amax_kernel(const void *__restrict__ src, int64_t n, int64_t slice, uint32_t *__restrict__ partials) {
  const int64_t begin = (int64_t)blockIdx.x * slice;
  const int64_t end = min(n, begin + slice);
  uint32_t m = 0;  // magnitude bits in the source format
  if constexpr (VEC) {
    constexpr int per = SRC == FP8B200_F32 ? 4 : 8;  // elements per 16-byte unit
    constexpr int esz = SRC == FP8B200_F32 ? 4 : 2;
    const uint4 *v = reinterpret_cast<const uint4 *>(static_cast<const char *>(src) + begin * esz);
    const int nvec = (int)((end - begin) / per);
    int j = threadIdx.x;
    for (; j + 3 * kThreads < nvec; j += 4 * kThreads) {
      const uint4 q0 = __ldg(v + j), q1 = __ldg(v + j + kThreads), q2 = __ldg(v + j + 2 * kThreads),
                  q3 = __ldg(v + j + 3 * kThreads);
      m = max(max(m, unit_abs_max<SRC>(q0)), max(unit_abs_max<SRC>(q1), max(unit_abs_max<SRC>(q2),
                                                                               unit_abs_max<SRC>(q3))));
    }
    for (; j < nvec; j += kThreads) m = max(m, unit_abs_max<SRC>(__ldg(v + j)));
    for (int64_t i = begin + (int64_t)nvec * per + threadIdx.x; i < end; i += kThreads) {
      const uint32_t b = SRC == FP8B200_F32 ? reinterpret_cast<const uint32_t *>(src)[i] & 0x7FFFFFFFu
                                            : reinterpret_cast<const uint16_t *>(src)[i] & 0x7FFFu;
      m = max(m, b);
    }
    m = to_float_bits<SRC>(m);
  } else {
    for (int64_t i = begin + threadIdx.x; i < end; i += kThreads) m = max(m, abs_bits<SRC>(src, i));
  }
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[kThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t r = threadIdx.x < kThreads / 32 ? warp_max[threadIdx.x] : 0u;
    r = __reduce_max_sync(0xFFFFFFFFu, r);
    if (threadIdx.x == 0) partials[blockIdx.x] = r;
  }
}

// One block: amax over the first `nslices` partials, then scale = fmax/amax
// (1 when amax is 0 or NaN) and its reciprocal, in double as the allocating
// path computes them.
__global__ void __launch_bounds__(1024)
scale_from_partials_kernel(const uint32_t *__restrict__ partials, int nslices, float fmax,
                           float *__restrict__ scale_out) {
  uint32_t m = 0;
  for (int i = threadIdx.x; i < nslices; i += blockDim.x) m = max(m, partials[i]);
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t warp_max[32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t r = threadIdx.x < blockDim.x / 32 ? warp_max[threadIdx.x] : 0u;
    r = __reduce_max_sync(0xFFFFFFFFu, r);
    if (threadIdx.x == 0) {
      const double a = (double)__uint_as_float(r);
      const double sd = (a > 0.0) ? (double)fmax / a : 1.0;
      scale_out[0] = (float)sd;
      scale_out[1] = (float)(1.0 / sd);
    }
  }
}

// Device address of the scratch array on the current device. Looked up on
// every call: after the first call on a device (which loads this library's
// device code there, and so must come before any stream capture) the lookup
// is a cheap host query, and it stays right if the context is ever
// recreated (cudaDeviceReset) and the array lands at another address.
int scratch_ptr(uint32_t **out) {
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_amax_partials);
  if (e != cudaSuccess || p == nullptr)
    return set_error(FP8B200_ELAUNCH, "quantize_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  *out = static_cast<uint32_t *>(p);
  return FP8B200_OK;
}

}  // namespace noalloc
}  // namespace fp8b200

using namespace fp8b200;

extern "C" int fp8b200_quantize_fp8_noalloc(const void *src, int src_dtype, void *dst, int fp8_dtype, int64_t n,
                                            float *scale_out, void *stream) {
  using namespace fp8b200::noalloc;
  if (n < 0) return set_error(FP8B200_EINVAL, "quantize_noalloc: negative element count");
  if (n > kMaxElems)
    return set_error(FP8B200_EINVAL,
                     "quantize_noalloc: %lld elements exceed the limit of %lld (its fixed scratch holds %d "
                     "partials of %lld elements); use fp8b200_quantize_fp8 with caller-provided scratch",
                     (long long)n, (long long)kMaxElems, kSlices, (long long)kMaxSliceElems);
  if (src_dtype != FP8B200_F32 && src_dtype != FP8B200_BF16 && src_dtype != FP8B200_F16)
    return set_error(FP8B200_EINVAL, "quantize_noalloc: source dtype %d is not f32/bf16/f16", src_dtype);
  if (fp8_dtype != FP8B200_E4M3 && fp8_dtype != FP8B200_E5M2)
    return set_error(FP8B200_EINVAL, "quantize_noalloc: target dtype %d is not e4m3fn/e5m2", fp8_dtype);
  if (!scale_out) return set_error(FP8B200_EINVAL, "quantize_noalloc: null scale pointer");
  if (n > 0 && (!src || !dst)) return set_error(FP8B200_EINVAL, "quantize_noalloc: null pointer");
  int dev;
  if (int rc = check_device(&dev)) return rc;
  uint32_t *partials;
  if (int rc = scratch_ptr(&partials)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t per = (n + kSlices - 1) / kSlices;
  const int64_t slice = std::max<int64_t>(kSliceUnit, (per + kSliceUnit - 1) / kSliceUnit * kSliceUnit);
  const int nslices = (int)((n + slice - 1) / slice);
  if (nslices > 0) {
    const bool vec = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    if (src_dtype == FP8B200_F32) {
      if (vec) slice_amax_kernel<FP8B200_F32, true><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
      else slice_amax_kernel<FP8B200_F32, false><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
    } else if (src_dtype == FP8B200_BF16) {
      if (vec) slice_amax_kernel<FP8B200_BF16, true><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
      else slice_amax_kernel<FP8B200_BF16, false><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
    } else {
      if (vec) slice_amax_kernel<FP8B200_F16, true><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
      else slice_amax_kernel<FP8B200_F16, false><<<nslices, kThreads, 0, st>>>(src, n, slice, partials);
    }
    count_launch();
    if (int rc = check_launch("quantize_noalloc amax")) return rc;
  }
  const float fmax = fp8_dtype == FP8B200_E4M3 ? 448.0f : 57344.0f;
  scale_from_partials_kernel<<<1, 1024, 0, st>>>(partials, nslices, fmax, scale_out);
  count_launch();
  if (int rc = check_launch("quantize_noalloc scale")) return rc;
  // the encode pass is the library's ordinary encoder, reading the scale the
  // previous kernel wrote on the same stream
  return fp8b200_encode_fp8(src, src_dtype, dst, fp8_dtype, n, scale_out, stream);
}

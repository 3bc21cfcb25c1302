// Shared host/device helpers for libfp8_b200.so (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/fp8_b200.h"

namespace fp8b200 {

// ---------------------------------------------------------------- errors
int set_error(int code, const char *fmt, ...);
int check_launch(const char *what);
// Returns FP8B200_OK if the current device is a compute-capability 10.0 part.
int check_device(int *device_out);
void count_launch(uint64_t k = 1);

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dt) {
  switch (dt) {
    case FP8B200_F32: return 4;
    case FP8B200_BF16: case FP8B200_F16: return 2;
    case FP8B200_E4M3: case FP8B200_E5M2: return 1;
    default: return 0;
  }
}

// Grid size for grid-stride kernels: at most blocks_per_sm x the SM count of
// the current device, fewer when there is less work.
int grid_for(int64_t work_items, int threads_per_block, int blocks_per_sm);

// SM count of the device last passed through check_device on this thread.
int current_sm_count();

// ---------------------------------------------------------------- device bit helpers
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

}  // namespace fp8b200

// Library-wide plumbing for the C ABI: error reporting, device checks,
// grid sizing and the launch counter.
#include "common.cuh"

#include <atomic>
#include <mutex>

namespace fp8b200 {

static thread_local char g_err[512] = {0};
static std::atomic<uint64_t> g_launches{0};

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(FP8B200_ELAUNCH, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return FP8B200_OK;
}

void count_launch(uint64_t k) { g_launches.fetch_add(k, std::memory_order_relaxed); }

namespace {
constexpr int kMaxDevices = 64;
struct DevInfo {
  std::once_flag once;
  int ok = 0;  // 1 = sm_100
  int sms = 148;
  int major = 0, minor = 0;
};
DevInfo g_dev[kMaxDevices];
thread_local int t_sms = 148;
}  // namespace

int check_device(int *device_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FP8B200_EDEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(FP8B200_EDEVICE, "device index %d out of range", dev);
  DevInfo &d = g_dev[dev];
  std::call_once(d.once, [&] {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) {
      d.major = p.major;
      d.minor = p.minor;
      d.sms = p.multiProcessorCount;
      d.ok = (p.major == 10 && p.minor == 0) ? 1 : 0;
    }
  });
  if (!d.ok)
    return set_error(FP8B200_EDEVICE,
                     "device %d has compute capability %d.%d; this library is built for sm_100a (B200) only",
                     dev, d.major, d.minor);
  t_sms = d.sms;
  if (device_out) *device_out = dev;
  return FP8B200_OK;
}

int current_sm_count() { return t_sms; }

int grid_for(int64_t work_items, int threads_per_block, int blocks_per_sm) {
  const int64_t full = (int64_t)t_sms * blocks_per_sm;
  const int64_t need = (work_items + threads_per_block - 1) / threads_per_block;
  if (need >= full) return (int)full;
  return (int)(need < 1 ? 1 : need);
}

}  // namespace fp8b200

extern "C" int fp8b200_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" const char *fp8b200_last_error(void) { return fp8b200::g_err; }

extern "C" uint64_t fp8b200_launch_count(void) {
  return fp8b200::g_launches.load(std::memory_order_relaxed);
}

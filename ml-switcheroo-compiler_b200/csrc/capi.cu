// ABI-level helpers of libb200.so: version, error text, launch counter, device error flag.
#include <stdarg.h>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace b200 {

static thread_local char t_err[1024] = "";
static std::atomic<uint64_t> g_launches{0};
__device__ int g_device_error = 0;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return B200_ERR_CUDA;
  }
  count_launch();
  return B200_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

}  // namespace b200

extern "C" {

int b200_abi_version(void) { return 1; }

const char* b200_last_error(void) { return b200::t_err; }

uint64_t b200_launch_count(void) { return b200::g_launches.load(); }

int b200_check_device_error(void* stream) {
  cudaError_t e = cudaStreamSynchronize(b200::as_stream(stream));
  if (e != cudaSuccess) {
    b200::set_error("stream sync: %s", cudaGetErrorString(e));
    return B200_ERR_CUDA;
  }
  int code = 0;
  e = cudaMemcpyFromSymbol(&code, b200::g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    b200::set_error("read device error flag: %s", cudaGetErrorString(e));
    return B200_ERR_CUDA;
  }
  if (code != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(b200::g_device_error, &zero, sizeof(int));
    b200::set_error("device-side check failed (code %d)", code);
    return code;
  }
  return B200_OK;
}

}  // extern "C"

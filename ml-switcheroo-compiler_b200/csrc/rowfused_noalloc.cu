// b200_rowfused_fwd_bwd_noalloc: the fused row chain (b200_rowfused_fwd_bwd) for callers
// that cannot allocate device memory per call. Its scratch (the per-CTA column partials
// of da, db, dgamma, dbeta) lives in a file-scope device array of fixed size instead of a
// caller workspace. Host code cannot use the array's name as a device address, so its
// address is looked up once per device (cudaGetSymbolAddress, with that device current)
// and cached; every later call is allocation-free. Nothing in the scratch has to start at
// zero: each call writes every partial it reads. Calls that overlap in time on the GPU
// (on different streams, or from several host threads) share the one array and race;
// serialise them.
#include <mutex>

#include "common.cuh"

extern "C" size_t b200_rowfused_workspace_bytes(int64_t rows, int64_t cols);
extern "C" int b200_rowfused_fwd_bwd(const float* x, const float* a, const float* b, const float* gamma, const float* beta,
                                     const float* cot, float* y, int64_t* am, float* dx, float* da, float* db, float* dgamma,
                                     float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace,
                                     size_t workspace_bytes, void* stream);

namespace b200 {
namespace noalloc {

constexpr size_t kRowfusedScratchBytes = (size_t)16 << 20;  // 16 MiB, held by every GPU that loads the library
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_rowfused_scratch[kRowfusedScratchBytes];

std::mutex g_mu;
void* g_scratch[kMaxDevices] = {nullptr};

}  // namespace noalloc
}  // namespace b200

using namespace b200;

extern "C" int b200_rowfused_fwd_bwd_noalloc(const float* x, const float* a, const float* b, const float* gamma,
                                             const float* beta, const float* cot, float* y, int64_t* am, float* dx, float* da,
                                             float* db, float* dgamma, float* dbeta, int64_t rows, int64_t cols, float eps,
                                             void* stream) {
  using namespace b200::noalloc;
  B200_REQUIRE(rows >= 0 && cols >= 1, "rowfused_noalloc: bad sizes");
  B200_REQUIRE(cols <= 16384, "rowfused_noalloc: cols %lld > 16384", (long long)cols);
  const size_t need = b200_rowfused_workspace_bytes(rows, cols);
  if (need > kRowfusedScratchBytes) {
    set_error("rowfused_noalloc: %lld x %lld needs %zu bytes of scratch, above the %zu-byte static maximum "
              "(use b200_rowfused_fwd_bwd with a caller workspace)",
              (long long)rows, (long long)cols, need, kRowfusedScratchBytes);
    return B200_ERR_ARG;
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("rowfused_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return B200_ERR_CUDA;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch[dev]) {
      // first call on this device: resolve the array's device address (no allocation)
      e = cudaGetSymbolAddress(&scratch, g_rowfused_scratch);
      if (e != cudaSuccess || !scratch) {
        set_error("rowfused_noalloc: cudaGetSymbolAddress failed on device %d (%s)", dev, cudaGetErrorString(e));
        return B200_ERR_CUDA;
      }
      g_scratch[dev] = scratch;
    }
    scratch = g_scratch[dev];
  }
  return b200_rowfused_fwd_bwd(x, a, b, gamma, beta, cot, y, am, dx, da, db, dgamma, dbeta, rows, cols, eps, scratch,
                               kRowfusedScratchBytes, stream);
}

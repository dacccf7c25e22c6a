// Fused LogSoftmax -> TakeAlongAxis (pick the label column) forward and backward.
// Forward:  picked[r] = x[r, label[r]] - max_j x[r, j] - log(sum_j exp(x[r, j] - max))
// Backward: with d[r] the cotangent of picked (already computed by the small ops of the
//           loss reduction), the VJP graph ScatterAdd(ZerosLike(ls), label, d) followed by
//           the LogSoftmax rule g - exp(ls) * sum(g) collapses to
//           dx[r, j] = d[r] * ([j == label[r]] - softmax(x)[r, j]).
// Replaces LogSoftmax (numpy/eager/math_advanced/math_log_exp.py:87-104), TakeAlongAxis
// (numpy/eager/advanced_indexing.py:163-177), ZerosLike, ScatterAdd
// (advanced_indexing.py:309-326), ReduceSum/Exp/Multiply/Subtract of the LogSoftmax VJP.
// One CTA per row: an online max/sum-exp pass, then one write pass (the row is re-read
// from L2). Out-of-range labels set the device error flag.
#include "common.cuh"

namespace b200 {

constexpr int XE_T = 512;

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }

template <typename T>
__global__ void __launch_bounds__(XE_T) xent_kernel(const T* __restrict__ x, const int64_t* __restrict__ label,
                                                    const float* __restrict__ d, float* __restrict__ picked,
                                                    float* __restrict__ ls_out, float* __restrict__ dx, int64_t V) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const T* xr = x + r * V;
  float m = -INFINITY, s = 0.f;
  for (int64_t j = threadIdx.x; j < V; j += XE_T) {
    const float v = ldf(xr, j);
    if (v > m) {
      s = s * expf(m - v);
      m = v;
    }
    s += expf(v - m);
  }
  // merge (m, s) across the block
  const float M = block_max(m, red);
  s = (m == -INFINITY) ? 0.f : s * expf(m - M);
  const float S = block_sum(s, red);
  const float lse = M + logf(S);
  int64_t lab = label[r];
  if (lab < 0) lab += V;
  const bool ok = lab >= 0 && lab < V;
  if (threadIdx.x == 0) {
    if (!ok) raise_device_error(B200_ERR_ARG);
    if (picked) picked[r] = ok ? ldf(xr, lab) - lse : 0.f;
  }
  if (ls_out) {
    float* lr = ls_out + r * V;
    for (int64_t j = threadIdx.x; j < V; j += XE_T) lr[j] = ldf(xr, j) - lse;
  }
  if (dx) {
    const float dr = d[r];
    float* dr_out = dx + r * V;
    for (int64_t j = threadIdx.x; j < V; j += XE_T) {
      const float sm = expf(ldf(xr, j) - lse);
      dr_out[j] = dr * ((j == lab ? 1.f : 0.f) - sm);
    }
  }
}

}  // namespace b200

using namespace b200;

extern "C" int b200_logsoftmax_pick(int x_dtype, const void* x, const int64_t* label, const float* d, float* picked,
                                    float* ls, float* dx, int64_t rows, int64_t cols, void* stream) {
  B200_REQUIRE(x && label, "logsoftmax_pick: null input");
  B200_REQUIRE(!dx || d, "logsoftmax_pick: dx needs the cotangent d");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL, "logsoftmax_pick: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  if (x_dtype == B200_F32)
    xent_kernel<float><<<(unsigned)rows, XE_T, 0, s>>>((const float*)x, label, d, picked, ls, dx, cols);
  else if (x_dtype == B200_BF16)
    xent_kernel<__nv_bfloat16><<<(unsigned)rows, XE_T, 0, s>>>((const __nv_bfloat16*)x, label, d, picked, ls, dx, cols);
  else {
    set_error("logsoftmax_pick: dtype %d", x_dtype);
    return B200_ERR_DTYPE;
  }
  return check_launch("logsoftmax_pick");
}

// Backward of a tanh-approximation GELU fed by a bias add, in one pass over HBM:
//     dp = g * gelu'(p)       gelu'(p) = 0.5 (1 + t) + 0.5 p (1 - t^2) k (1 + 3 c p^2),
//                             t = tanh(k (p + c p^3)), k = sqrt(2 / pi), c = 0.044715
//     dbias = sum_rows(dp)    (BroadcastReduce to the bias vector)
// The derivative is evaluated in the operation order of the VJP graph the AD pass emits
// for Gelu (the elementwise chain the reference evaluates op by op with
// numpy/eager/math_binary.py:9-51 and np.tanh). dp is written in bf16 when it only
// feeds tensor-core GEMMs (and/or fp32); the column sums go through per-CTA partials
// reduced in a fixed order, so they are deterministic.
#include <math.h>

#include "common.cuh"

namespace b200 {
namespace gb {

constexpr int T = 256, V = 8;

__device__ __forceinline__ float gelu_deriv(float p) {
  const float k = 0.7978845608028654f, c = 0.044715f;
  const float p2 = p * p;
  const float p3 = p2 * p;
  const float t = tanhf((p + p3 * c) * k);
  const float left = (t + 1.f) * 0.5f;
  const float sech2 = 1.f - t * t;
  const float dinner = (p2 * 0.134145f + 1.f) * k;  // 3 c, rounded once as the graph constant is
  const float right = ((p * sech2) * dinner) * 0.5f;
  return left + right;
}

__global__ void __launch_bounds__(T) gelu_bwd_colsum_kernel(const float* __restrict__ g, const float* __restrict__ p,
                                                            __nv_bfloat16* __restrict__ ybf, float* __restrict__ yf,
                                                            float* __restrict__ part, int64_t R, int64_t C, int64_t rows_per,
                                                            int vec_ok) {
  const int64_t c0 = ((int64_t)blockIdx.x * T + threadIdx.x) * V;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = min(R, r0 + rows_per);
  if (c0 >= C) return;
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  const bool vec = vec_ok && (c0 + V <= C);
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t off = r * C + c0;
    if (vec) {
      const float4 g0 = __ldcs(reinterpret_cast<const float4*>(g + off));
      const float4 g1 = __ldcs(reinterpret_cast<const float4*>(g + off + 4));
      const float4 p0 = __ldcs(reinterpret_cast<const float4*>(p + off));
      const float4 p1 = __ldcs(reinterpret_cast<const float4*>(p + off + 4));
      const float gv[V] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float pv[V] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      float v[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[i] = gv[i] * gelu_deriv(pv[i]);
        acc[i] += v[i];
      }
      if (ybf) {
        __align__(16) __nv_bfloat162 t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        __stcs(reinterpret_cast<uint4*>(ybf + off), *reinterpret_cast<uint4*>(t));
      }
      if (yf) {
        __stcs(reinterpret_cast<float4*>(yf + off), make_float4(v[0], v[1], v[2], v[3]));
        __stcs(reinterpret_cast<float4*>(yf + off + 4), make_float4(v[4], v[5], v[6], v[7]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        if (c0 + i >= C) break;
        const float x = g[off + i] * gelu_deriv(p[off + i]);
        acc[i] += x;
        if (ybf) ybf[off + i] = __float2bfloat16_rn(x);
        if (yf) yf[off + i] = x;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i)
    if (c0 + i < C) part[(int64_t)blockIdx.y * C + c0 + i] = acc[i];
}

__global__ void colsum_parts_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t G, int64_t C) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (col >= C) return;
  float s = 0.f;
  for (int64_t k = 0; k < G; ++k) s += part[k * C + col];
  out[col] = s;
}

static void grid_for(int64_t R, int64_t C, int64_t& gx, int64_t& gy, int64_t& rows_per) {
  gx = ceil_div(ceil_div(C, V), T);
  const int64_t want = (int64_t)num_sms() * 8;
  gy = std::max<int64_t>(1, std::min<int64_t>(R, ceil_div(want, gx)));
  rows_per = ceil_div(R, gy);
  gy = ceil_div(R, rows_per);
}

}  // namespace gb
}  // namespace b200

using namespace b200;
using namespace b200::gb;

extern "C" size_t b200_gelu_bwd_colsum_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  int64_t gx, gy, rp;
  grid_for(rows, cols, gx, gy, rp);
  return (size_t)gy * (size_t)cols * sizeof(float);
}

extern "C" int b200_gelu_bwd_colsum(const float* g, const float* p, void* y_bf16, float* y_f32, float* colsum, int64_t rows,
                                    int64_t cols, void* workspace, size_t workspace_bytes, void* stream) {
  B200_REQUIRE(g && p, "gelu_bwd_colsum: null input");
  B200_REQUIRE(y_bf16 || y_f32 || colsum, "gelu_bwd_colsum: no output");
  B200_REQUIRE(rows >= 0 && cols >= 1, "gelu_bwd_colsum: bad sizes");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (colsum) cudaMemsetAsync(colsum, 0, cols * 4, s);
    return check_launch("gelu_bwd_colsum(empty)");
  }
  const size_t need = b200_gelu_bwd_colsum_workspace_bytes(rows, cols);
  B200_REQUIRE(workspace && workspace_bytes >= need, "gelu_bwd_colsum: workspace %zu < %zu", workspace_bytes, need);
  int64_t gx, gy, rp;
  grid_for(rows, cols, gx, gy, rp);
  B200_REQUIRE(gx <= 2147483647LL && gy <= 65535, "gelu_bwd_colsum: grid too large");
  const bool al = ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(y_f32) |
                    reinterpret_cast<uintptr_t>(y_bf16)) & 15) == 0;
  const int vec_ok = (al && cols % V == 0) ? 1 : 0;
  float* part = reinterpret_cast<float*>(workspace);
  dim3 grid((unsigned)gx, (unsigned)gy);
  gelu_bwd_colsum_kernel<<<grid, T, 0, s>>>(g, p, (__nv_bfloat16*)y_bf16, y_f32, part, rows, cols, rp, vec_ok);
  int rc = check_launch("gelu_bwd_colsum");
  if (rc || !colsum) return rc;
  colsum_parts_kernel<<<(unsigned)ceil_div(cols, 256), 256, 0, s>>>(part, colsum, gy, cols);
  return check_launch("gelu_bwd_colsum(colsum)");
}

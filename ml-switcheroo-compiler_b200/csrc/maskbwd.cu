// Backward of a ReLU + bias epilogue in one pass over HBM:
//     gp = g * mask            (Multiply(cot, Greater(pre, 0)), the ReLU VJP)
//     dbias = sum_rows(gp)     (BroadcastReduce to the bias vector)
// gp is written in bf16 when it only feeds tensor-core GEMMs (and/or in fp32), and the
// column sums go through per-CTA partials reduced in a fixed order (deterministic).
#include "common.cuh"

namespace b200 {

constexpr int MB_T = 256, MB_V = 8;

__global__ void __launch_bounds__(MB_T) mask_mul_colsum_kernel(const float* __restrict__ g, const uint8_t* __restrict__ mask,
                                                               __nv_bfloat16* __restrict__ ybf, float* __restrict__ yf,
                                                               float* __restrict__ part, int64_t R, int64_t C,
                                                               int64_t rows_per) {
  const int64_t c0 = ((int64_t)blockIdx.x * MB_T + threadIdx.x) * MB_V;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = min(R, r0 + rows_per);
  float acc[MB_V];
#pragma unroll
  for (int i = 0; i < MB_V; ++i) acc[i] = 0.f;
  if (c0 < C) {
    const bool vec = (c0 + MB_V <= C) && (C % MB_V == 0);
    for (int64_t r = r0; r < r1; ++r) {
      const int64_t off = r * C + c0;
      float v[MB_V];
      if (vec) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(g + off));
        const float4 b = __ldcs(reinterpret_cast<const float4*>(g + off + 4));
        const uint2 m = __ldcs(reinterpret_cast<const uint2*>(mask + off));
        v[0] = (m.x & 0xff) ? a.x : 0.f;
        v[1] = (m.x & 0xff00) ? a.y : 0.f;
        v[2] = (m.x & 0xff0000) ? a.z : 0.f;
        v[3] = (m.x & 0xff000000) ? a.w : 0.f;
        v[4] = (m.y & 0xff) ? b.x : 0.f;
        v[5] = (m.y & 0xff00) ? b.y : 0.f;
        v[6] = (m.y & 0xff0000) ? b.z : 0.f;
        v[7] = (m.y & 0xff000000) ? b.w : 0.f;
#pragma unroll
        for (int i = 0; i < MB_V; ++i) acc[i] += v[i];
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
        for (int i = 0; i < MB_V; ++i) {
          if (c0 + i >= C) break;
          const float x = mask[off + i] ? g[off + i] : 0.f;
          acc[i] += x;
          if (ybf) ybf[off + i] = __float2bfloat16_rn(x);
          if (yf) yf[off + i] = x;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < MB_V; ++i)
      if (c0 + i < C) part[(int64_t)blockIdx.y * C + c0 + i] = acc[i];
  }
}

__global__ void colsum_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t G, int64_t C) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (col >= C) return;
  float s = 0.f;
  for (int64_t g = 0; g < G; ++g) s += part[g * C + col];
  out[col] = s;
}

static void mb_grid(int64_t R, int64_t C, int64_t& gx, int64_t& gy, int64_t& rows_per) {
  gx = ceil_div(ceil_div(C, MB_V), MB_T);
  const int64_t want = (int64_t)num_sms() * 8;
  gy = std::max<int64_t>(1, std::min<int64_t>(R, ceil_div(want, gx)));
  rows_per = ceil_div(R, gy);
  gy = ceil_div(R, rows_per);
}

}  // namespace b200

using namespace b200;

extern "C" size_t b200_mask_mul_colsum_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  int64_t gx, gy, rp;
  mb_grid(rows, cols, gx, gy, rp);
  return (size_t)gy * (size_t)cols * sizeof(float);
}

extern "C" int b200_mask_mul_colsum(const float* g, const uint8_t* mask, void* y_bf16, float* y_f32, float* colsum,
                                    int64_t rows, int64_t cols, void* workspace, size_t workspace_bytes, void* stream) {
  B200_REQUIRE(g && mask, "mask_mul_colsum: null input");
  B200_REQUIRE(y_bf16 || y_f32 || colsum, "mask_mul_colsum: no output");
  B200_REQUIRE(rows >= 0 && cols >= 1, "mask_mul_colsum: bad sizes");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (colsum) cudaMemsetAsync(colsum, 0, cols * 4, s);
    return check_launch("mask_mul_colsum(empty)");
  }
  const size_t need = b200_mask_mul_colsum_workspace_bytes(rows, cols);
  B200_REQUIRE(!colsum || (workspace && workspace_bytes >= need), "mask_mul_colsum: workspace %zu < %zu", workspace_bytes, need);
  int64_t gx, gy, rp;
  mb_grid(rows, cols, gx, gy, rp);
  B200_REQUIRE(gx <= 2147483647LL && gy <= 65535, "mask_mul_colsum: grid too large");
  float* part = colsum ? reinterpret_cast<float*>(workspace) : nullptr;
  if (!colsum) {
    // no column sums wanted: the partials go nowhere useful, give the kernel a dummy
    // that is never written past its rows (reuse y_f32 is not allowed) -> require workspace
    B200_REQUIRE(workspace && workspace_bytes >= need, "mask_mul_colsum: workspace %zu < %zu", workspace_bytes, need);
    part = reinterpret_cast<float*>(workspace);
  }
  dim3 grid((unsigned)gx, (unsigned)gy);
  mask_mul_colsum_kernel<<<grid, MB_T, 0, s>>>(g, mask, (__nv_bfloat16*)y_bf16, y_f32, part, rows, cols, rp);
  int rc = check_launch("mask_mul_colsum");
  if (rc || !colsum) return rc;
  colsum_rows_kernel<<<(unsigned)ceil_div(cols, 256), 256, 0, s>>>(part, colsum, gy, cols);
  return check_launch("mask_mul_colsum(colsum)");
}

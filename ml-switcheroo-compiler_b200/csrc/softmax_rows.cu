// Softmax / log-softmax over the last axis and the softmax VJP, with an optional scalar
// pre-scale read from device memory and fp32 and/or bf16 outputs:
//
//   fwd : t = x * s;  y = exp(t - max t) / sum exp(t - max t)      (log: t - max t - log sum)
//   bwd : dx = s * (y * (g - sum(g * y)))
//
// Rows up to 2048 columns (a multiple of 4) are held in registers, one warp per row:
// every element is read once and written once (128-bit loads, 64/128-bit stores). Longer
// or unaligned rows use one CTA per row and re-read the row from L2.
//
// Reference semantics: Softmax (numpy/eager/math_advanced/math_signal.py:450-467),
// LogSoftmax (math_advanced/math_log_exp.py:87-104); the VJP is the composition the AD
// pass emits for Softmax (Multiply, ReduceSum keepdims, Subtract, Multiply), and the
// scalar multiply folds the Multiply node that feeds an attention softmax.
#include <math.h>

#include "common.cuh"

namespace b200 {
namespace smx {

constexpr int WARPS = 8;  // rows per CTA in the warp-per-row kernels

__device__ __forceinline__ float4 ldg4_stream(const float* p) { return __ldcs(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}

// ---------------------------------------------------------------------------------
// warp per row, NC chunks of 4 columns per lane (cols <= NC * 128, cols % 4 == 0)
// ---------------------------------------------------------------------------------
template <int NC, bool LOG>
__global__ void __launch_bounds__(WARPS * 32) softmax_warp_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                                  float* __restrict__ y, __nv_bfloat16* __restrict__ yb,
                                                                  int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float s = scale ? __ldg(scale) : 1.f;
  const float* xr = x + row * cols;
  float v[NC][4];
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
      const float4 t = ldg4_stream(xr + col);
      v[c][0] = t.x * s; v[c][1] = t.y * s; v[c][2] = t.z * s; v[c][3] = t.w * s;
    } else {
      v[c][0] = v[c][1] = v[c][2] = v[c][3] = -INFINITY;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) m = fmaxf(m, v[c][k]);
  }
  m = warp_max(m);
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float e = (v[c][k] == -INFINITY) ? 0.f : __expf(v[c][k] - m);
      sum += e;
      if (!LOG) v[c][k] = e;
    }
  sum = warp_sum(sum);
  const float inv = 1.f / sum, lse = logf(sum);
  float* yr = y ? y + row * cols : nullptr;
  __nv_bfloat16* ybr = yb ? yb + row * cols : nullptr;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col >= cols) continue;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = LOG ? (v[c][k] - m - lse) : v[c][k] * inv;
    if (yr) *reinterpret_cast<float4*>(yr + col) = make_float4(o[0], o[1], o[2], o[3]);
    if (ybr) st_bf16x4(ybr + col, o[0], o[1], o[2], o[3]);
  }
}

template <int NC>
__global__ void __launch_bounds__(WARPS * 32) softmax_bwd_warp_kernel(const float* __restrict__ y, const float* __restrict__ g,
                                                                      const float* __restrict__ scale, float* __restrict__ dx,
                                                                      __nv_bfloat16* __restrict__ dxb, int64_t rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float s = scale ? __ldg(scale) : 1.f;
  const float* yr = y + row * cols;
  const float* gr = g + row * cols;
  float yv[NC][4], gv[NC][4];
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
      const float4 a = ldg4_stream(yr + col), b = ldg4_stream(gr + col);
      yv[c][0] = a.x; yv[c][1] = a.y; yv[c][2] = a.z; yv[c][3] = a.w;
      gv[c][0] = b.x; gv[c][1] = b.y; gv[c][2] = b.z; gv[c][3] = b.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) yv[c][k] = gv[c][k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc += gv[c][k] * yv[c][k];
  }
  const float S = warp_sum(acc);
  float* dr = dx ? dx + row * cols : nullptr;
  __nv_bfloat16* dbr = dxb ? dxb + row * cols : nullptr;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col >= cols) continue;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = (yv[c][k] * (gv[c][k] - S)) * s;
    if (dr) *reinterpret_cast<float4*>(dr + col) = make_float4(o[0], o[1], o[2], o[3]);
    if (dbr) st_bf16x4(dbr + col, o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------------
// CTA per row (any column count): the row is re-read from L2 on each pass
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) softmax_block_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                            float* __restrict__ y, __nv_bfloat16* __restrict__ yb,
                                                            int64_t cols, int logmode) {
  __shared__ float sred[32];
  const float s = scale ? __ldg(scale) : 1.f;
  const float* xr = x + blockIdx.x * cols;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, xr[i] * s);
  const float M = block_max(m, sred);
  float sum = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float t = xr[i] * s;
    sum += (t == -INFINITY) ? 0.f : __expf(t - M);
  }
  const float S = block_sum(sum, sred);
  const float inv = 1.f / S, lse = logf(S);
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float t = xr[i] * s;
    const float o = logmode ? (t - M - lse) : ((t == -INFINITY) ? 0.f : __expf(t - M)) * inv;
    if (y) y[blockIdx.x * cols + i] = o;
    if (yb) yb[blockIdx.x * cols + i] = __float2bfloat16_rn(o);
  }
}

__global__ void __launch_bounds__(512) softmax_bwd_block_kernel(const float* __restrict__ y, const float* __restrict__ g,
                                                                const float* __restrict__ scale, float* __restrict__ dx,
                                                                __nv_bfloat16* __restrict__ dxb, int64_t cols) {
  __shared__ float sred[32];
  const float s = scale ? __ldg(scale) : 1.f;
  const float* yr = y + blockIdx.x * cols;
  const float* gr = g + blockIdx.x * cols;
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) acc += gr[i] * yr[i];
  const float S = block_sum(acc, sred);
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float o = (yr[i] * (gr[i] - S)) * s;
    if (dx) dx[blockIdx.x * cols + i] = o;
    if (dxb) dxb[blockIdx.x * cols + i] = __float2bfloat16_rn(o);
  }
}

inline int chunks_for(int64_t cols) {
  if (cols % 4) return 0;
  const int64_t nc = ceil_div(cols, 128);
  if (nc <= 1) return 1;
  if (nc <= 2) return 2;
  if (nc <= 4) return 4;
  if (nc <= 8) return 8;
  if (nc <= 16) return 16;
  return 0;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

}  // namespace smx
}  // namespace b200

using namespace b200;
using namespace b200::smx;

extern "C" int b200_softmax_rows(const float* x, const float* scale, float* y, void* y_bf16, int64_t rows, int64_t cols, int log,
                                 void* stream) {
  B200_REQUIRE(x && (y || y_bf16), "softmax_rows: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL && cols <= 2147483647LL, "softmax_rows: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  auto* yb = reinterpret_cast<__nv_bfloat16*>(y_bf16);
  int nc = chunks_for(cols);
  if (nc && !(aligned16(x) && (!y || aligned16(y)) && (!yb || aligned8(yb)))) nc = 0;
  const unsigned grid = (unsigned)ceil_div(rows, (int64_t)WARPS);
  if (nc && ceil_div(rows, (int64_t)WARPS) <= 2147483647LL) {
#define B200_SMX_FWD(NC)                                                                                          \
  (log ? softmax_warp_kernel<NC, true><<<grid, WARPS * 32, 0, s>>>(x, scale, y, yb, rows, (int)cols)                \
       : softmax_warp_kernel<NC, false><<<grid, WARPS * 32, 0, s>>>(x, scale, y, yb, rows, (int)cols))
    switch (nc) {
      case 1: B200_SMX_FWD(1); break;
      case 2: B200_SMX_FWD(2); break;
      case 4: B200_SMX_FWD(4); break;
      case 8: B200_SMX_FWD(8); break;
      default: B200_SMX_FWD(16); break;
    }
#undef B200_SMX_FWD
    return check_launch("softmax_rows(warp)");
  }
  const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
  softmax_block_kernel<<<(unsigned)rows, threads, 0, s>>>(x, scale, y, yb, cols, log);
  return check_launch("softmax_rows(block)");
}

extern "C" int b200_softmax_bwd_rows(const float* y, const float* g, const float* scale, float* dx, void* dx_bf16, int64_t rows,
                                     int64_t cols, void* stream) {
  B200_REQUIRE(y && g && (dx || dx_bf16), "softmax_bwd_rows: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL && cols <= 2147483647LL, "softmax_bwd_rows: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  auto* db = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
  int nc = chunks_for(cols);
  if (nc && !(aligned16(y) && aligned16(g) && (!dx || aligned16(dx)) && (!db || aligned8(db)))) nc = 0;
  const unsigned grid = (unsigned)ceil_div(rows, (int64_t)WARPS);
  if (nc) {
    switch (nc) {
      case 1: softmax_bwd_warp_kernel<1><<<grid, WARPS * 32, 0, s>>>(y, g, scale, dx, db, rows, (int)cols); break;
      case 2: softmax_bwd_warp_kernel<2><<<grid, WARPS * 32, 0, s>>>(y, g, scale, dx, db, rows, (int)cols); break;
      case 4: softmax_bwd_warp_kernel<4><<<grid, WARPS * 32, 0, s>>>(y, g, scale, dx, db, rows, (int)cols); break;
      case 8: softmax_bwd_warp_kernel<8><<<grid, WARPS * 32, 0, s>>>(y, g, scale, dx, db, rows, (int)cols); break;
      default: softmax_bwd_warp_kernel<16><<<grid, WARPS * 32, 0, s>>>(y, g, scale, dx, db, rows, (int)cols); break;
    }
    return check_launch("softmax_bwd_rows(warp)");
  }
  const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
  softmax_bwd_block_kernel<<<(unsigned)rows, threads, 0, s>>>(y, g, scale, dx, db, cols);
  return check_launch("softmax_bwd_rows(block)");
}

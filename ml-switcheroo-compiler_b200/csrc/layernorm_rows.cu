// LayerNorm over the last axis and its input gradient, fp32 math, fp32 and/or bf16
// outputs (a LayerNorm whose output only feeds bf16 GEMMs is written in bf16 alone).
//
//   fwd : y = (x - mean) * rstd * gamma + beta,   rstd = 1 / sqrt(var + eps)
//   dx  : dx = rstd / C * (C * g - sum(g) - xhat * sum(g * xhat)),  g = dy * gamma
//
// mean and the biased variance are two-pass (sum, then the sum of squared deviations),
// as np.mean / np.var compute them. Rows up to 2048 columns (a multiple of 4) live in
// registers, one warp per row, so x (and dy) are read from HBM exactly once; other rows
// take one CTA per row.
//
// Reference: LayerNorm (numpy/eager/nn_ops.py:219-241), LayerNormInputGrad (nn_ops.py:244).
#include <math.h>

#include "common.cuh"

extern "C" int b200_layernorm_input_grad_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16,
                                              int64_t rows, int64_t cols, float eps, void* stream);
extern "C" int b200_layernorm_param_grad(const float* dy, const float* x, float* dgamma, float* dbeta, int64_t rows,
                                         int64_t cols, float eps, void* workspace, size_t workspace_bytes, void* stream);
extern "C" size_t b200_layernorm_param_grad_workspace_bytes(int64_t rows, int64_t cols);

namespace b200 {
namespace lnr {

constexpr int WARPS = 8;

__device__ __forceinline__ void st_bf16x4(__nv_bfloat16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

template <int NC>
__global__ void __launch_bounds__(WARPS * 32) ln_fwd_warp_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta, float* __restrict__ y,
                                                                 __nv_bfloat16* __restrict__ yb, int64_t rows, int cols,
                                                                 float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float v[NC][4];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
      const float4 t = __ldcs(reinterpret_cast<const float4*>(xr + col));
      v[c][0] = t.x; v[c][1] = t.y; v[c][2] = t.z; v[c][3] = t.w;
    } else {
      v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
    }
    s += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
  }
  const float mean = warp_sum(s) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float d = v[c][k] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = 1.f / sqrtf(warp_sum(q) / (float)cols + eps);
  float* yr = y ? y + row * cols : nullptr;
  __nv_bfloat16* ybr = yb ? yb + row * cols : nullptr;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col >= cols) continue;
    const float4 g = gamma ? ld4(gamma + col) : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 b = beta ? ld4(beta + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float o0 = g.x * ((v[c][0] - mean) * rstd) + b.x;
    const float o1 = g.y * ((v[c][1] - mean) * rstd) + b.y;
    const float o2 = g.z * ((v[c][2] - mean) * rstd) + b.z;
    const float o3 = g.w * ((v[c][3] - mean) * rstd) + b.w;
    if (yr) *reinterpret_cast<float4*>(yr + col) = make_float4(o0, o1, o2, o3);
    if (ybr) st_bf16x4(ybr + col, o0, o1, o2, o3);
  }
}

template <int NC>
__global__ void __launch_bounds__(WARPS * 32) ln_dx_warp_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                                const float* __restrict__ gamma, float* __restrict__ dx,
                                                                __nv_bfloat16* __restrict__ dxb, int64_t rows, int cols,
                                                                float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  const float* dr = dy + row * cols;
  float v[NC][4], gv[NC][4];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
      const float4 t = __ldcs(reinterpret_cast<const float4*>(xr + col));
      const float4 d = __ldcs(reinterpret_cast<const float4*>(dr + col));
      const float4 g = gamma ? ld4(gamma + col) : make_float4(1.f, 1.f, 1.f, 1.f);
      v[c][0] = t.x; v[c][1] = t.y; v[c][2] = t.z; v[c][3] = t.w;
      gv[c][0] = d.x * g.x; gv[c][1] = d.y * g.y; gv[c][2] = d.z * g.z; gv[c][3] = d.w * g.w;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[c][k] = gv[c][k] = 0.f;
    }
    s += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
  }
  const float mean = warp_sum(s) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < cols) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float d = v[c][k] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = 1.f / sqrtf(warp_sum(q) / (float)cols + eps);
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[c][k] = (v[c][k] - mean) * rstd;  // xhat (0 in the padding: gv is 0 there too)
      s1 += gv[c][k];
      s2 += gv[c][k] * v[c][k];
    }
  const float S1 = warp_sum(s1), S2 = warp_sum(s2);
  const float d = (float)cols, f = rstd / d;
  float* dxr = dx ? dx + row * cols : nullptr;
  __nv_bfloat16* dbr = dxb ? dxb + row * cols : nullptr;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col >= cols) continue;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = f * (d * gv[c][k] - S1 - v[c][k] * S2);
    if (dxr) *reinterpret_cast<float4*>(dxr + col) = make_float4(o[0], o[1], o[2], o[3]);
    if (dbr) st_bf16x4(dbr + col, o[0], o[1], o[2], o[3]);
  }
}

// ---------------- one CTA per row (any column count) ----------------
__device__ __forceinline__ void block_stats(const float* __restrict__ xr, int64_t cols, float eps, float* sred, float& mean,
                                            float& rstd) {
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) s += xr[i];
  mean = block_sum(s, sred) / (float)cols;
  float q = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float d = xr[i] - mean;
    q += d * d;
  }
  rstd = 1.f / sqrtf(block_sum(q, sred) / (float)cols + eps);
}

__global__ void __launch_bounds__(512) ln_fwd_block_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                           const float* __restrict__ beta, float* __restrict__ y,
                                                           __nv_bfloat16* __restrict__ yb, int64_t cols, float eps) {
  __shared__ float sred[32];
  const int64_t base = (int64_t)blockIdx.x * cols;
  float mean, rstd;
  block_stats(x + base, cols, eps, sred, mean, rstd);
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float o = (gamma ? gamma[i] : 1.f) * ((x[base + i] - mean) * rstd) + (beta ? beta[i] : 0.f);
    if (y) y[base + i] = o;
    if (yb) yb[base + i] = __float2bfloat16_rn(o);
  }
}

__global__ void __launch_bounds__(512) ln_dx_block_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                          const float* __restrict__ gamma, float* __restrict__ dx,
                                                          __nv_bfloat16* __restrict__ dxb, int64_t cols, float eps) {
  __shared__ float sred[32];
  const int64_t base = (int64_t)blockIdx.x * cols;
  float mean, rstd;
  block_stats(x + base, cols, eps, sred, mean, rstd);
  float s1 = 0.f, s2 = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float g = dy[base + i] * (gamma ? gamma[i] : 1.f);
    s1 += g;
    s2 += g * ((x[base + i] - mean) * rstd);
  }
  const float S1 = block_sum(s1, sred), S2 = block_sum(s2, sred);
  const float d = (float)cols, f = rstd / d;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float g = dy[base + i] * (gamma ? gamma[i] : 1.f);
    const float o = f * (d * g - S1 - ((x[base + i] - mean) * rstd) * S2);
    if (dx) dx[base + i] = o;
    if (dxb) dxb[base + i] = __float2bfloat16_rn(o);
  }
}

// Whole LayerNorm backward, warp per row, persistent: dx for every row, and per-CTA
// column partials of dgamma = sum dy * xhat and dbeta = sum dy (LayerNormGammaGrad /
// LayerNormBetaGrad, nn_ops.py:276-318) reduced across the CTA's warps in shared memory;
// a second kernel sums the CTA partials in a fixed order (deterministic).
template <int NC>
__global__ void __launch_bounds__(WARPS * 32) ln_bwd_warp_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                                 const float* __restrict__ gamma, float* __restrict__ dx,
                                                                 __nv_bfloat16* __restrict__ dxb, float* __restrict__ part,
                                                                 int64_t rows, int cols, float eps) {
  extern __shared__ float sp[];  // [WARPS][2][cols] per-warp column partials
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float pg[NC][4], pb[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int k = 0; k < 4; ++k) pg[c][k] = pb[c][k] = 0.f;
  float gm[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    const float4 g = (gamma && col < cols) ? ld4(gamma + col) : make_float4(1.f, 1.f, 1.f, 1.f);
    gm[c][0] = g.x; gm[c][1] = g.y; gm[c][2] = g.z; gm[c][3] = g.w;
  }
  for (int64_t row = (int64_t)blockIdx.x * WARPS + w; row < rows; row += (int64_t)gridDim.x * WARPS) {
    const float* xr = x + row * cols;
    const float* dr = dy + row * cols;
    float v[NC][4], d[NC][4];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < cols) {
        const float4 t = __ldcs(reinterpret_cast<const float4*>(xr + col));
        const float4 e = __ldcs(reinterpret_cast<const float4*>(dr + col));
        v[c][0] = t.x; v[c][1] = t.y; v[c][2] = t.z; v[c][3] = t.w;
        d[c][0] = e.x; d[c][1] = e.y; d[c][2] = e.z; d[c][3] = e.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[c][k] = d[c][k] = 0.f;
      }
      s += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
    }
    const float mean = warp_sum(s) / (float)cols;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < cols) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float t = v[c][k] - mean;
          q += t * t;
        }
      }
    }
    const float rstd = 1.f / sqrtf(warp_sum(q) / (float)cols + eps);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[c][k] = (v[c][k] - mean) * rstd;  // xhat
        const float gd = d[c][k] * gm[c][k];
        s1 += gd;
        s2 += gd * v[c][k];
        pg[c][k] += d[c][k] * v[c][k];
        pb[c][k] += d[c][k];
      }
    const float S1 = warp_sum(s1), S2 = warp_sum(s2);
    const float fc = (float)cols, f = rstd / fc;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col >= cols) continue;
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = f * (fc * (d[c][k] * gm[c][k]) - S1 - v[c][k] * S2);
      if (dx) *reinterpret_cast<float4*>(dx + row * cols + col) = make_float4(o[0], o[1], o[2], o[3]);
      if (dxb) st_bf16x4(dxb + row * cols + col, o[0], o[1], o[2], o[3]);
    }
  }
  // CTA partials: warps add their columns in a fixed order
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col >= cols) continue;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      sp[(w * 2 + 0) * cols + col + k] = pg[c][k];
      sp[(w * 2 + 1) * cols + col + k] = pb[c][k];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * cols; i += blockDim.x) {
    const int which = i / cols, col = i % cols;
    float acc = 0.f;
    for (int ww = 0; ww < WARPS; ++ww) acc += sp[(ww * 2 + which) * cols + col];
    part[((int64_t)blockIdx.x * 2 + which) * cols + col] = acc;
  }
}

// part[g][2][cols] -> (dgamma, dbeta): entry i of the 2 cols outputs is the sum over g in a
// fixed order (deterministic): warp w of a block adds g = w, w + 8, ... in increasing g for
// 32 adjacent entries, then the 8 warp sums are added in warp order.
constexpr int LN_CS_WARPS = 8;
__global__ void __launch_bounds__(32 * LN_CS_WARPS) ln_colsum_kernel(const float* __restrict__ part, float* __restrict__ dg,
                                                             float* __restrict__ db, int64_t G, int64_t cols) {
  __shared__ float sh[LN_CS_WARPS][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t i = (int64_t)blockIdx.x * 32 + lane;
  const bool live = i < 2 * cols;
  float acc = 0.f;
  if (live) {
#pragma unroll 4
    for (int64_t g = w; g < G; g += LN_CS_WARPS) acc += __ldg(part + g * 2 * cols + i);
  }
  sh[w][lane] = acc;
  __syncthreads();
  if (w == 0 && live) {
    float t = sh[0][lane];
#pragma unroll
    for (int k = 1; k < LN_CS_WARPS; ++k) t += sh[k][lane];
    if (i < cols) {
      if (dg) dg[i] = t;
    } else if (db) {
      db[i - cols] = t;
    }
  }
}

inline int64_t ln_bwd_grid(int64_t rows) {
  return std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, (int64_t)WARPS), (int64_t)num_sms()));
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
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

}  // namespace lnr
}  // namespace b200

using namespace b200;
using namespace b200::lnr;

extern "C" int b200_layernorm_rows(const float* x, const float* gamma, const float* beta, float* y, void* y_bf16, int64_t rows,
                                   int64_t cols, float eps, void* stream) {
  B200_REQUIRE(x && (y || y_bf16), "layernorm_rows: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL && cols <= 2147483647LL, "layernorm_rows: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  auto* yb = reinterpret_cast<__nv_bfloat16*>(y_bf16);
  int nc = chunks_for(cols);
  if (nc && !(al16(x) && (!gamma || al16(gamma)) && (!beta || al16(beta)) && (!y || al16(y)) && (!yb || al8(yb)))) nc = 0;
  const unsigned grid = (unsigned)ceil_div(rows, (int64_t)WARPS);
  switch (nc) {
    case 1: ln_fwd_warp_kernel<1><<<grid, WARPS * 32, 0, s>>>(x, gamma, beta, y, yb, rows, (int)cols, eps); break;
    case 2: ln_fwd_warp_kernel<2><<<grid, WARPS * 32, 0, s>>>(x, gamma, beta, y, yb, rows, (int)cols, eps); break;
    case 4: ln_fwd_warp_kernel<4><<<grid, WARPS * 32, 0, s>>>(x, gamma, beta, y, yb, rows, (int)cols, eps); break;
    case 8: ln_fwd_warp_kernel<8><<<grid, WARPS * 32, 0, s>>>(x, gamma, beta, y, yb, rows, (int)cols, eps); break;
    case 16: ln_fwd_warp_kernel<16><<<grid, WARPS * 32, 0, s>>>(x, gamma, beta, y, yb, rows, (int)cols, eps); break;
    default: {
      const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
      ln_fwd_block_kernel<<<(unsigned)rows, threads, 0, s>>>(x, gamma, beta, y, yb, cols, eps);
    }
  }
  return check_launch("layernorm_rows");
}

extern "C" int b200_layernorm_input_grad_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16,
                                              int64_t rows, int64_t cols, float eps, void* stream) {
  B200_REQUIRE(dy && x && (dx || dx_bf16), "layernorm_input_grad_rows: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL && cols <= 2147483647LL, "layernorm_input_grad_rows: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  auto* db = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
  int nc = chunks_for(cols);
  if (nc && !(al16(x) && al16(dy) && (!gamma || al16(gamma)) && (!dx || al16(dx)) && (!db || al8(db)))) nc = 0;
  const unsigned grid = (unsigned)ceil_div(rows, (int64_t)WARPS);
  switch (nc) {
    case 1: ln_dx_warp_kernel<1><<<grid, WARPS * 32, 0, s>>>(dy, x, gamma, dx, db, rows, (int)cols, eps); break;
    case 2: ln_dx_warp_kernel<2><<<grid, WARPS * 32, 0, s>>>(dy, x, gamma, dx, db, rows, (int)cols, eps); break;
    case 4: ln_dx_warp_kernel<4><<<grid, WARPS * 32, 0, s>>>(dy, x, gamma, dx, db, rows, (int)cols, eps); break;
    case 8: ln_dx_warp_kernel<8><<<grid, WARPS * 32, 0, s>>>(dy, x, gamma, dx, db, rows, (int)cols, eps); break;
    case 16: ln_dx_warp_kernel<16><<<grid, WARPS * 32, 0, s>>>(dy, x, gamma, dx, db, rows, (int)cols, eps); break;
    default: {
      const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
      ln_dx_block_kernel<<<(unsigned)rows, threads, 0, s>>>(dy, x, gamma, dx, db, cols, eps);
    }
  }
  return check_launch("layernorm_input_grad_rows");
}

extern "C" size_t b200_layernorm_bwd_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  // the fused kernel's CTA partials, or the separate parameter-gradient kernel's
  return std::max((size_t)ln_bwd_grid(rows) * 2 * (size_t)cols * sizeof(float),
                  b200_layernorm_param_grad_workspace_bytes(rows, cols));
}

extern "C" int b200_layernorm_bwd_rows(const float* dy, const float* x, const float* gamma, float* dx, void* dx_bf16,
                                       float* dgamma, float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  B200_REQUIRE(dy && x, "layernorm_bwd_rows: null input");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL && cols <= 2147483647LL, "layernorm_bwd_rows: bad sizes");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (dgamma) cudaMemsetAsync(dgamma, 0, cols * 4, s);
    if (dbeta) cudaMemsetAsync(dbeta, 0, cols * 4, s);
    return check_launch("layernorm_bwd_rows(empty)");
  }
  auto* db = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
  const int nc = chunks_for(cols);
  const bool fits = nc > 0 && nc <= 8 && al16(x) && al16(dy) && (!gamma || al16(gamma)) && (!dx || al16(dx)) && (!db || al8(db));
  if (!fits) {
    // general shapes: the separate input-gradient and parameter-gradient kernels
    int rc = B200_OK;
    if (dx || db) rc = b200_layernorm_input_grad_rows(dy, x, gamma, dx, dx_bf16, rows, cols, eps, stream);
    if (rc == B200_OK && (dgamma || dbeta))
      rc = b200_layernorm_param_grad(dy, x, dgamma, dbeta, rows, cols, eps, workspace, workspace_bytes, stream);
    return rc;
  }
  const size_t need = b200_layernorm_bwd_workspace_bytes(rows, cols);
  B200_REQUIRE(workspace && workspace_bytes >= need, "layernorm_bwd_rows: workspace %zu < %zu", workspace_bytes, need);
  const int64_t G = ln_bwd_grid(rows);
  const size_t smem = (size_t)WARPS * 2 * (size_t)cols * sizeof(float);
  B200_REQUIRE(smem <= 200 * 1024, "layernorm_bwd_rows: %lld columns too many", (long long)cols);
  float* part = reinterpret_cast<float*>(workspace);
#define B200_LNB(NCV)                                                                                              \
  case NCV: {                                                                                                      \
    static bool attr = false;                                                                                      \
    if (!attr) {                                                                                                   \
      cudaFuncSetAttribute(ln_bwd_warp_kernel<NCV>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);      \
      attr = true;                                                                                                 \
    }                                                                                                              \
    ln_bwd_warp_kernel<NCV><<<(unsigned)G, WARPS * 32, smem, s>>>(dy, x, gamma, dx, db, part, rows, (int)cols, eps); \
    break;                                                                                                         \
  }
  switch (nc) {
    B200_LNB(1)
    B200_LNB(2)
    B200_LNB(4)
    B200_LNB(8)
    default: break;
  }
#undef B200_LNB
  int rc = check_launch("layernorm_bwd_rows");
  if (rc) return rc;
  if (!dgamma && !dbeta) return B200_OK;
  ln_colsum_kernel<<<(unsigned)ceil_div(2 * cols, (int64_t)32), 32 * LN_CS_WARPS, 0, s>>>(part, dgamma, dbeta, G, cols);
  return check_launch("layernorm_bwd_rows(colsum)");
}

// Row reductions (subsystem 2): axis reductions, argmax, softmax / log-softmax,
// LayerNorm forward and its three VJPs. Warp-shuffle + shared-memory block reductions;
// one CTA per row for last-axis work, column-parallel loops for middle-axis work.
#include <math.h>

#include "common.cuh"

namespace b200 {

// ---------------------------------------------------------------------------------
// middle-axis reduce: x [outer, red, inner] -> y [outer, inner]
// ---------------------------------------------------------------------------------

// inner == 1: one CTA per outer row (row reduction)
template <int OP>
__global__ void __launch_bounds__(256) reduce_rows_kernel(const void* __restrict__ x, int dt, float* __restrict__ y,
                                                          int64_t red) {
  __shared__ float sred[32];
  const int64_t row = blockIdx.x;
  float acc = (OP == B200_RED_MAX) ? -INFINITY : 0.f;
  for (int64_t i = threadIdx.x; i < red; i += blockDim.x) {
    float v = load_as_f32(x, row * red + i, dt);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
  float t = (OP == B200_RED_MAX) ? block_max(acc, sred) : block_sum(acc, sred);
  if (threadIdx.x == 0) y[row] = (OP == B200_RED_MEAN) ? t / (float)red : t;
}

// inner == 1 with short rows (red <= 1024): one warp per row, lane l combines elements
// l, l + 32, ... in order, then a fixed xor-butterfly (the same result on every run)
template <int OP>
__global__ void __launch_bounds__(256) reduce_rows_warp_kernel(const void* __restrict__ x, int dt, float* __restrict__ y,
                                                               int64_t rows, int64_t red) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float acc = (OP == B200_RED_MAX) ? -INFINITY : 0.f;
  for (int64_t i = lane; i < red; i += 32) {
    const float v = load_as_f32(x, row * red + i, dt);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, acc, o);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
  if (lane == 0) y[row] = (OP == B200_RED_MEAN) ? acc / (float)red : acc;
}

// inner == 1 with very short rows (red <= 64): G = 8 lanes per row, four rows per warp
// (a warp reads four consecutive rows at once); lane l of a group combines elements l,
// l + 8, ... in order, then a fixed xor-butterfly over the group
template <int OP>
__global__ void __launch_bounds__(256) reduce_rows_group_kernel(const void* __restrict__ x, int dt, float* __restrict__ y,
                                                                int64_t rows, int64_t red) {
  constexpr int G = 8;
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / G;
  const int sub = threadIdx.x % G;
  const bool live = row < rows;
  float acc = (OP == B200_RED_MAX) ? -INFINITY : 0.f;
  if (live) {
    for (int64_t i = sub; i < red; i += G) {
      const float v = load_as_f32(x, row * red + i, dt);
      if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
      else acc += v;
    }
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, acc, o);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
  if (live && sub == 0) y[row] = (OP == B200_RED_MEAN) ? acc / (float)red : acc;
}

// inner > 1: each thread owns one (outer, inner) column over a chunk of `red`. With one
// chunk the result goes straight to y; with several, chunk z writes its partial to
// part[z][outer][inner] and reduce_splits_kernel combines them in chunk order, so the
// result does not depend on scheduling (no float atomics).
template <int OP>
__global__ void __launch_bounds__(256) reduce_cols_kernel(const void* __restrict__ x, int dt, float* __restrict__ y,
                                                          float* __restrict__ part, int64_t outer, int64_t red, int64_t inner,
                                                          int64_t chunk) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t o = blockIdx.y;
  if (col >= inner) return;
  const int64_t r0 = blockIdx.z * chunk;
  const int64_t r1 = min(red, r0 + chunk);
  float acc = (OP == B200_RED_MAX) ? -INFINITY : 0.f;
  const int64_t base = o * red * inner + col;
  for (int64_t r = r0; r < r1; ++r) {
    float v = load_as_f32(x, base + r * inner, dt);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
  if (!part) {
    y[o * inner + col] = (OP == B200_RED_MEAN) ? acc / (float)red : acc;
  } else {
    part[((int64_t)blockIdx.z * outer + o) * inner + col] = acc;
  }
}

// one warp per output: lane l combines chunks l, l + 32, ... in order, then a fixed
// xor-butterfly combines the lanes, so the result is the same on every run
template <int OP>
__global__ void __launch_bounds__(256) reduce_splits_kernel(const float* __restrict__ part, float* __restrict__ y, int64_t n,
                                                            int64_t split, int64_t red) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  float acc = (OP == B200_RED_MAX) ? -INFINITY : 0.f;
  for (int64_t z = lane; z < split; z += 32) {
    const float v = __ldg(part + z * n + i);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, acc, o);
    if (OP == B200_RED_MAX) acc = fmaxf(acc, v);
    else acc += v;
  }
  if (lane == 0) y[i] = (OP == B200_RED_MEAN) ? acc / (float)red : acc;
}

__global__ void fill_kernel(float* y, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) y[i] = v;
}

// ---------------------------------------------------------------------------------
// argmax over the middle axis; first maximum wins, NaN counts as the maximum
// ---------------------------------------------------------------------------------
__device__ __forceinline__ bool am_better(float v, int64_t i, float m, int64_t j) {
  // does (v,i) beat (m,j)? ties -> smaller index
  const bool vn = isnan(v), mn = isnan(m);
  if (vn || mn) {
    if (vn && !mn) return true;
    if (!vn && mn) return false;
    return i < j;
  }
  if (v > m) return true;
  if (v < m) return false;
  return i < j;
}

__global__ void __launch_bounds__(256) argmax_rows_kernel(const void* __restrict__ x, int dt, int64_t* __restrict__ idx,
                                                          int64_t red) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int64_t row = blockIdx.x;
  float m = -INFINITY;
  int64_t j = INT64_MAX;
  for (int64_t i = threadIdx.x; i < red; i += blockDim.x) {
    float v = load_as_f32(x, row * red + i, dt);
    if (am_better(v, i, m, j)) { m = v; j = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, m, o);
    int64_t j2 = __shfl_xor_sync(0xffffffffu, j, o);
    if (am_better(v2, j2, m, j)) { m = v2; j = j2; }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { sv[wid] = m; si[wid] = j; }
  __syncthreads();
  if (wid == 0) {
    m = lane < nw ? sv[lane] : -INFINITY;
    j = lane < nw ? si[lane] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float v2 = __shfl_xor_sync(0xffffffffu, m, o);
      int64_t j2 = __shfl_xor_sync(0xffffffffu, j, o);
      if (am_better(v2, j2, m, j)) { m = v2; j = j2; }
    }
    if (lane == 0) idx[row] = (j == INT64_MAX) ? 0 : j;
  }
}

__global__ void __launch_bounds__(256) argmax_cols_kernel(const void* __restrict__ x, int dt, int64_t* __restrict__ idx,
                                                          int64_t outer, int64_t red, int64_t inner) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t o = blockIdx.y;
  if (col >= inner) return;
  float m = -INFINITY;
  int64_t j = INT64_MAX;
  for (int64_t r = 0; r < red; ++r) {
    float v = load_as_f32(x, (o * red + r) * inner + col, dt);
    if (am_better(v, r, m, j)) { m = v; j = r; }
  }
  idx[o * inner + col] = (j == INT64_MAX) ? 0 : j;
}

// ---------------------------------------------------------------------------------
// softmax / log-softmax over the last axis (one CTA per row, online max/sum)
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t cols,
                                                      int logmode) {
  __shared__ float sred[32];
  const float* xr = x + blockIdx.x * cols;
  float* yr = y + blockIdx.x * cols;
  float m = -INFINITY, s = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float v = xr[i];
    if (v > m) { s = s * expf(m - v); m = v; }  // rescale running sum (v finite here)
    s += expf(v - m);
  }
  const float M = block_max(m, sred);
  s = (m == -INFINITY) ? 0.f : s * expf(m - M);
  const float S = block_sum(s, sred);
  if (logmode) {
    const float lse = logf(S);
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) yr[i] = xr[i] - M - lse;
  } else {
    const float inv = 1.f / S;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) yr[i] = expf(xr[i] - M) * inv;
  }
}

// ---------------------------------------------------------------------------------
// LayerNorm (biased variance, two-pass mean then variance like np.mean / np.var)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void row_stats(const float* __restrict__ xr, int64_t cols, float eps, float* sred,
                                          float& mean, float& rstd) {
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) s += xr[i];
  mean = block_sum(s, sred) / (float)cols;
  float q = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float d = xr[i] - mean;
    q += d * d;
  }
  const float var = block_sum(q, sred) / (float)cols;
  rstd = 1.f / sqrtf(var + eps);
}

__global__ void __launch_bounds__(512) layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                                        const float* __restrict__ b, float* __restrict__ y,
                                                        int64_t cols, float eps) {
  __shared__ float sred[32];
  const float* xr = x + blockIdx.x * cols;
  float* yr = y + blockIdx.x * cols;
  float mean, rstd;
  row_stats(xr, cols, eps, sred, mean, rstd);
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float v = (xr[i] - mean) * rstd;
    yr[i] = (g ? g[i] : 1.f) * v + (b ? b[i] : 0.f);
  }
}

__global__ void __launch_bounds__(512) layernorm_input_grad_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                                   const float* __restrict__ g, float* __restrict__ dx,
                                                                   int64_t cols, float eps) {
  __shared__ float sred[32];
  const float* xr = x + blockIdx.x * cols;
  const float* dyr = dy + blockIdx.x * cols;
  float* dxr = dx + blockIdx.x * cols;
  float mean, rstd;
  row_stats(xr, cols, eps, sred, mean, rstd);
  float s1 = 0.f, s2 = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float dyg = dyr[i] * (g ? g[i] : 1.f);
    float xh = (xr[i] - mean) * rstd;
    s1 += dyg;
    s2 += dyg * xh;
  }
  const float S1 = block_sum(s1, sred);
  const float S2 = block_sum(s2, sred);
  const float d = (float)cols;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float dyg = dyr[i] * (g ? g[i] : 1.f);
    float xh = (xr[i] - mean) * rstd;
    dxr[i] = (rstd / d) * (d * dyg - S1 - xh * S2);
  }
}

// dgamma[c] = sum_r dy[r,c] * xhat[r,c], dbeta[c] = sum_r dy[r,c].
// Each CTA takes LN_PG_ROWS rows, keeps column partials in shared memory and writes them
// to part[cta][2][cols]; ln_pg_colsum_kernel adds the CTA partials in order
// (deterministic, no float atomics).
constexpr int LN_PG_ROWS = 64;
__global__ void __launch_bounds__(256) layernorm_param_grad_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                                   float* __restrict__ part, int64_t rows, int64_t cols,
                                                                   float eps) {
  extern __shared__ float sm[];  // [2*cols] partials
  __shared__ float sred[32];
  float* pg = sm;
  float* pb = sm + cols;
  for (int64_t i = threadIdx.x; i < 2 * cols; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const int64_t r0 = blockIdx.x * (int64_t)LN_PG_ROWS;
  const int64_t r1 = min(rows, r0 + LN_PG_ROWS);
  for (int64_t r = r0; r < r1; ++r) {
    const float* xr = x + r * cols;
    const float* dyr = dy + r * cols;
    float mean, rstd;
    row_stats(xr, cols, eps, sred, mean, rstd);
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
      float d = dyr[i];
      pg[i] += d * (xr[i] - mean) * rstd;
      pb[i] += d;
    }
  }
  __syncthreads();
  float* out = part + (int64_t)blockIdx.x * 2 * cols;
  for (int64_t i = threadIdx.x; i < 2 * cols; i += blockDim.x) out[i] = sm[i];
}

// part[g][2][cols] -> (dgamma, dbeta): entry i of the 2 cols outputs is the sum over g in a
// fixed order (deterministic): warp w of a block adds g = w, w + 8, ... in increasing g for
// 32 adjacent entries, then the 8 warp sums are added in warp order.
constexpr int LN_CS_WARPS = 8;
__global__ void __launch_bounds__(32 * LN_CS_WARPS) ln_pg_colsum_kernel(const float* __restrict__ part, float* __restrict__ dg,
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

}  // namespace b200

using namespace b200;

static void reduce_plan(int64_t outer, int64_t red, int64_t inner, int64_t& split, int64_t& chunk) {
  // split `red` across CTAs when there are too few columns to fill the GPU
  const int64_t cols_blocks = ceil_div(inner, 256);
  split = 1;
  const int64_t want = (int64_t)num_sms() * 4;
  if (cols_blocks * outer < want) split = std::min<int64_t>(ceil_div(want, cols_blocks * outer), ceil_div(red, 32));
  if (split < 1) split = 1;
  if (split > 65535) split = 65535;
  chunk = ceil_div(std::max<int64_t>(red, 1), split);
  split = ceil_div(std::max<int64_t>(red, 1), chunk);
}

extern "C" size_t b200_reduce_workspace_bytes(int64_t outer, int64_t red, int64_t inner) {
  if (outer <= 0 || red <= 0 || inner <= 1) return 0;
  int64_t split, chunk;
  reduce_plan(outer, red, inner, split, chunk);
  return split > 1 ? (size_t)split * (size_t)outer * (size_t)inner * sizeof(float) : 0;
}

extern "C" int b200_reduce(int dt, const void* x, float* y, int64_t outer, int64_t red, int64_t inner, int op,
                           void* workspace, size_t workspace_bytes, void* stream) {
  B200_REQUIRE(x && y, "reduce: null pointer");
  B200_REQUIRE(outer >= 0 && red >= 0 && inner >= 0, "reduce: negative size");
  B200_REQUIRE(op == B200_RED_SUM || op == B200_RED_MEAN || op == B200_RED_MAX, "reduce: bad op %d", op);
  if (dt != B200_F32 && dt != B200_BF16) {
    set_error("reduce: dtype %d", dt);
    return B200_ERR_DTYPE;
  }
  B200_REQUIRE(outer <= 2147483647LL && outer <= 65535 || inner == 1, "reduce: outer too large for column mode");
  if (outer == 0 || inner == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  if (red == 0) {
    // numpy: sum of nothing = 0, mean = nan, max raises
    B200_REQUIRE(op != B200_RED_MAX, "reduce: max over an empty axis");
    fill_kernel<<<64, 256, 0, s>>>(y, outer * inner, op == B200_RED_SUM ? 0.f : NAN);
    return check_launch("reduce(fill)");
  }
  if (inner == 1) {
    B200_REQUIRE(outer <= 2147483647LL, "reduce: too many rows");
    if (red <= 64) {
      const unsigned g = (unsigned)ceil_div(outer * 8, (int64_t)256);
      switch (op) {
        case B200_RED_SUM: reduce_rows_group_kernel<B200_RED_SUM><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
        case B200_RED_MEAN: reduce_rows_group_kernel<B200_RED_MEAN><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
        default: reduce_rows_group_kernel<B200_RED_MAX><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
      }
      return check_launch("reduce(short rows)");
    }
    if (red <= 1024) {
      const unsigned g = (unsigned)ceil_div(outer * 32, (int64_t)256);
      switch (op) {
        case B200_RED_SUM: reduce_rows_warp_kernel<B200_RED_SUM><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
        case B200_RED_MEAN: reduce_rows_warp_kernel<B200_RED_MEAN><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
        default: reduce_rows_warp_kernel<B200_RED_MAX><<<g, 256, 0, s>>>(x, dt, y, outer, red); break;
      }
      return check_launch("reduce(rows)");
    }
    switch (op) {
      case B200_RED_SUM: reduce_rows_kernel<B200_RED_SUM><<<(unsigned)outer, 256, 0, s>>>(x, dt, y, red); break;
      case B200_RED_MEAN: reduce_rows_kernel<B200_RED_MEAN><<<(unsigned)outer, 256, 0, s>>>(x, dt, y, red); break;
      default: reduce_rows_kernel<B200_RED_MAX><<<(unsigned)outer, 256, 0, s>>>(x, dt, y, red); break;
    }
    return check_launch("reduce(rows)");
  }
  int64_t split, chunk;
  reduce_plan(outer, red, inner, split, chunk);
  // without room for the chunk partials, one chunk per column (slower, same result)
  if (split > 1 && (!workspace || workspace_bytes < b200_reduce_workspace_bytes(outer, red, inner))) {
    split = 1;
    chunk = red;
  }
  float* part = split > 1 ? reinterpret_cast<float*>(workspace) : nullptr;
  dim3 grid((unsigned)ceil_div(inner, 256), (unsigned)outer, (unsigned)split);
  switch (op) {
    case B200_RED_SUM: reduce_cols_kernel<B200_RED_SUM><<<grid, 256, 0, s>>>(x, dt, y, part, outer, red, inner, chunk); break;
    case B200_RED_MEAN: reduce_cols_kernel<B200_RED_MEAN><<<grid, 256, 0, s>>>(x, dt, y, part, outer, red, inner, chunk); break;
    default: reduce_cols_kernel<B200_RED_MAX><<<grid, 256, 0, s>>>(x, dt, y, part, outer, red, inner, chunk); break;
  }
  int rc = check_launch("reduce(cols)");
  if (rc || split == 1) return rc;
  const int64_t n = outer * inner;
  const unsigned g2 = (unsigned)ceil_div(n * 32, 256);
  switch (op) {
    case B200_RED_SUM: reduce_splits_kernel<B200_RED_SUM><<<g2, 256, 0, s>>>(part, y, n, split, red); break;
    case B200_RED_MEAN: reduce_splits_kernel<B200_RED_MEAN><<<g2, 256, 0, s>>>(part, y, n, split, red); break;
    default: reduce_splits_kernel<B200_RED_MAX><<<g2, 256, 0, s>>>(part, y, n, split, red); break;
  }
  return check_launch("reduce(splits)");
}

extern "C" int b200_argmax(int dt, const void* x, int64_t* idx, int64_t outer, int64_t red, int64_t inner, void* stream) {
  B200_REQUIRE(x && idx, "argmax: null pointer");
  B200_REQUIRE(outer >= 0 && red >= 1 && inner >= 0, "argmax: bad sizes (red must be >= 1)");
  if (dt != B200_F32 && dt != B200_BF16) {
    set_error("argmax: dtype %d", dt);
    return B200_ERR_DTYPE;
  }
  if (outer == 0 || inner == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  if (inner == 1) {
    B200_REQUIRE(outer <= 2147483647LL, "argmax: too many rows");
    argmax_rows_kernel<<<(unsigned)outer, 256, 0, s>>>(x, dt, idx, red);
  } else {
    B200_REQUIRE(outer <= 65535, "argmax: outer too large");
    dim3 grid((unsigned)ceil_div(inner, 256), (unsigned)outer);
    argmax_cols_kernel<<<grid, 256, 0, s>>>(x, dt, idx, outer, red, inner);
  }
  return check_launch("argmax");
}

extern "C" int b200_softmax(const float* x, float* y, int64_t rows, int64_t cols, int log, void* stream) {
  B200_REQUIRE(x && y, "softmax: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL, "softmax: bad sizes");
  if (rows == 0) return B200_OK;
  const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
  softmax_kernel<<<(unsigned)rows, threads, 0, as_stream(stream)>>>(x, y, cols, log);
  return check_launch("softmax");
}

extern "C" int b200_layernorm(const float* x, const float* g, const float* b, float* y, int64_t rows, int64_t cols,
                              float eps, void* stream) {
  B200_REQUIRE(x && y, "layernorm: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL, "layernorm: bad sizes");
  if (rows == 0) return B200_OK;
  const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
  layernorm_kernel<<<(unsigned)rows, threads, 0, as_stream(stream)>>>(x, g, b, y, cols, eps);
  return check_launch("layernorm");
}

extern "C" int b200_layernorm_input_grad(const float* dy, const float* x, const float* g, float* dx, int64_t rows,
                                         int64_t cols, float eps, void* stream) {
  B200_REQUIRE(dy && x && dx, "layernorm_input_grad: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL, "layernorm_input_grad: bad sizes");
  if (rows == 0) return B200_OK;
  const int threads = cols >= 4096 ? 512 : (cols >= 1024 ? 256 : 128);
  layernorm_input_grad_kernel<<<(unsigned)rows, threads, 0, as_stream(stream)>>>(dy, x, g, dx, cols, eps);
  return check_launch("layernorm_input_grad");
}

extern "C" size_t b200_layernorm_param_grad_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)ceil_div(rows, (int64_t)LN_PG_ROWS) * 2 * (size_t)cols * sizeof(float);
}

extern "C" int b200_layernorm_param_grad(const float* dy, const float* x, float* dg, float* db, int64_t rows, int64_t cols,
                                         float eps, void* workspace, size_t workspace_bytes, void* stream) {
  B200_REQUIRE(dy && x, "layernorm_param_grad: null pointer");
  B200_REQUIRE(dg || db, "layernorm_param_grad: no output");
  B200_REQUIRE(rows >= 0 && cols >= 1, "layernorm_param_grad: bad sizes");
  B200_REQUIRE(cols <= 16384, "layernorm_param_grad: cols %lld > 16384", (long long)cols);
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (dg) cudaMemsetAsync(dg, 0, cols * sizeof(float), s);
    if (db) cudaMemsetAsync(db, 0, cols * sizeof(float), s);
    return check_launch("layernorm_param_grad(zero)");
  }
  const size_t need = b200_layernorm_param_grad_workspace_bytes(rows, cols);
  B200_REQUIRE(workspace && workspace_bytes >= need, "layernorm_param_grad: workspace %zu < %zu", workspace_bytes, need);
  const int64_t G = ceil_div(rows, (int64_t)LN_PG_ROWS);
  B200_REQUIRE(G <= 2147483647LL, "layernorm_param_grad: too many rows");
  const size_t smem = 2 * cols * sizeof(float);
  if (smem > 48 * 1024) cudaFuncSetAttribute(layernorm_param_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  float* part = reinterpret_cast<float*>(workspace);
  layernorm_param_grad_kernel<<<(unsigned)G, 256, smem, s>>>(dy, x, part, rows, cols, eps);
  int rc = check_launch("layernorm_param_grad");
  if (rc) return rc;
  ln_pg_colsum_kernel<<<(unsigned)ceil_div(2 * cols, (int64_t)32), 32 * LN_CS_WARPS, 0, s>>>(part, dg, db, G, cols);
  return check_launch("layernorm_param_grad(colsum)");
}

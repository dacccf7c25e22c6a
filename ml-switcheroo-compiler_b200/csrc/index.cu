// Indexing kernels: TakeAlongAxis / ScatterAdd on the last axis (cross-entropy pick and
// its VJP), row gather (embedding lookup, np.take axis 0) and row scatter-add
// (TensorScatterAdd, the embedding VJP). Out-of-range indices set the device error flag
// and the element is skipped (never read or written out of bounds).
#include "common.cuh"

namespace b200 {

__global__ void take_along_last_kernel(const float* __restrict__ x, const int64_t* __restrict__ idx, float* __restrict__ y,
                                       int64_t rows, int64_t cols, int64_t k) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < rows * k; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / k;
    int64_t j = idx[e];
    if (j < 0) j += cols;  // numpy negative index
    if (j < 0 || j >= cols) {
      raise_device_error(B200_ERR_ARG);
      y[e] = 0.f;
      continue;
    }
    y[e] = x[r * cols + j];
  }
}

// one thread per row: copy the row, then apply the k updates in order (last write wins
// for a repeated index, like put_along_axis of take + src)
__global__ void scatter_add_last_kernel(const float* __restrict__ base, const int64_t* __restrict__ idx,
                                        const float* __restrict__ src, float* __restrict__ y, int64_t rows, int64_t cols,
                                        int64_t k) {
  const int64_t r = blockIdx.x;
  float* yr = y + r * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = base ? base[r * cols + c] : 0.f;
  __syncthreads();
  if (threadIdx.x == 0) {
    // put_along_axis(out, idx, take_along_axis(out, idx) + src): all reads happen before writes
    for (int64_t j = 0; j < k; ++j) {
      int64_t c = idx[r * k + j];
      if (c < 0) c += cols;
      if (c < 0 || c >= cols) {
        raise_device_error(B200_ERR_ARG);
        continue;
      }
      const float old = base ? base[r * cols + c] : 0.f;
      yr[c] = old + src[r * k + j];
    }
  }
}

template <typename T>
__global__ void take_rows_kernel(const T* __restrict__ table, const int64_t* __restrict__ ids, T* __restrict__ y, int64_t n,
                                 int64_t V, int64_t D) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * D; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / D, d = e % D;
    int64_t v = ids[i];
    if (v < 0) v += V;
    if (v < 0 || v >= V) {
      raise_device_error(B200_ERR_ARG);
      continue;
    }
    y[e] = table[v * D + d];
  }
}

// fp32 rows of D % 4 == 0 (16-byte aligned): one warp per output row, 16-byte accesses
__global__ void __launch_bounds__(256) take_rows4_kernel(const float* __restrict__ table, const int64_t* __restrict__ ids,
                                                         float* __restrict__ y, int64_t n, int64_t V, int64_t D) {
  const int64_t i = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (i >= n) return;
  const int lane = threadIdx.x & 31;
  int64_t v = ids[i];
  if (v < 0) v += V;
  if (v < 0 || v >= V) {
    if (lane == 0) raise_device_error(B200_ERR_ARG);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(table + v * D);
  float4* dst = reinterpret_cast<float4*>(y + i * D);
  for (int64_t c = lane; c < D / 4; c += 32) dst[c] = __ldg(src + c);
}

// Deterministic row scatter-add: positions are bucketed by their row id with a stable
// counting sort (integer atomics only; stable order from in-block ranks), then every
// output row sums its source rows in increasing position order. Float results therefore
// do not depend on scheduling, unlike an atomic accumulation.
constexpr int SA_B = 1024;  // positions per counting block

// ranks / block histogram: rank[i] = earlier positions of block g with the same id,
// cnt[g][v] = positions of block g with id v (cnt zeroed by the caller)
__global__ void __launch_bounds__(SA_B) sa_rank_kernel(const int64_t* __restrict__ ids, int* __restrict__ rank,
                                                       int* __restrict__ cnt, int64_t n, int64_t V) {
  __shared__ int sid[SA_B];
  const int64_t i = (int64_t)blockIdx.x * SA_B + threadIdx.x;
  int v = -1;
  if (i < n) {
    int64_t x = ids[i];
    if (x < 0) x += V;
    if (x < 0 || x >= V) raise_device_error(B200_ERR_ARG);
    else v = (int)x;
  }
  sid[threadIdx.x] = v;
  __syncthreads();
  if (v < 0) return;
  int r = 0, tot = 0;
  const int lim = (int)min((int64_t)SA_B, n - (int64_t)blockIdx.x * SA_B);
  for (int j = 0; j < lim; ++j) {
    const int same = sid[j] == v;
    tot += same;
    if (j < (int)threadIdx.x) r += same;
  }
  rank[i] = r;
  if (r == 0) cnt[(int64_t)blockIdx.x * V + v] = tot;
}

// per row id v: total count, and cnt[g][v] turned into the start of block g's run
__global__ void sa_colscan_kernel(int* __restrict__ cnt, int* __restrict__ tot, int64_t G, int64_t V) {
  const int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (v >= V) return;
  int run = 0;
  for (int64_t g = 0; g < G; ++g) {
    const int c = cnt[g * V + v];
    cnt[g * V + v] = run;
    run += c;
  }
  tot[v] = run;
}

// exclusive scan of tot[V] into off[V + 1] (one CTA, chunked)
__global__ void __launch_bounds__(1024) sa_scan_kernel(const int* __restrict__ tot, int* __restrict__ off, int64_t V) {
  __shared__ int part[1024];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < V; base += 1024) {
    const int64_t v = base + threadIdx.x;
    const int x = v < V ? tot[v] : 0;
    part[threadIdx.x] = x;
    __syncthreads();
    for (int d = 1; d < 1024; d <<= 1) {  // inclusive Hillis-Steele scan
      const int y = threadIdx.x >= d ? part[threadIdx.x - d] : 0;
      __syncthreads();
      part[threadIdx.x] += y;
      __syncthreads();
    }
    if (v < V) off[v] = carry + part[threadIdx.x] - x;
    __syncthreads();
    if (threadIdx.x == 1023) carry += part[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) off[V] = carry;
}

__global__ void sa_place_kernel(const int64_t* __restrict__ ids, const int* __restrict__ rank, const int* __restrict__ cnt,
                                const int* __restrict__ off, int* __restrict__ perm, int64_t n, int64_t V) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  int64_t x = ids[i];
  if (x < 0) x += V;
  if (x < 0 || x >= V) return;
  const int64_t g = i / SA_B;
  perm[off[x] + cnt[g * V + x] + rank[i]] = (int)i;
}

// y[v, :] = (accumulate ? y[v, :] : 0) + sum over v's positions, in position order;
// block (v, column chunk) = blockIdx.x / dblocks, blockIdx.x % dblocks
__global__ void __launch_bounds__(256) sa_sum_kernel(const float* __restrict__ src, const int* __restrict__ perm,
                                                     const int* __restrict__ off, float* __restrict__ y, int64_t D,
                                                     int64_t dblocks, int accumulate) {
  const int64_t v = blockIdx.x / dblocks;
  const int64_t d = (blockIdx.x % dblocks) * 256 + threadIdx.x;
  if (d >= D) return;
  const int a = off[v], b = off[v + 1];
  float acc = accumulate ? y[v * D + d] : 0.f;
  for (int k = a; k < b; ++k) acc += __ldg(src + (int64_t)perm[k] * D + d);
  y[v * D + d] = acc;
}

// the same sums, one warp per row v with 16-byte accesses (D % 4 == 0, 16-byte aligned
// rows): each float4 column group is summed over v's positions in position order, so the
// result is bit-identical to sa_sum_kernel
__global__ void __launch_bounds__(256) sa_sum4_kernel(const float* __restrict__ src, const int* __restrict__ perm,
                                                      const int* __restrict__ off, float* __restrict__ y, int64_t V, int64_t D,
                                                      int accumulate) {
  const int64_t v = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (v >= V) return;
  const int lane = threadIdx.x & 31;
  const int a = off[v], b = off[v + 1];
  float4* yr = reinterpret_cast<float4*>(y + v * D);
  for (int64_t c = lane; c < D / 4; c += 32) {
    float4 acc = accumulate ? yr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = a; k < b; ++k) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src + (int64_t)perm[k] * D) + c);
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    yr[c] = acc;
  }
}

inline int64_t sa_blocks(int64_t n) { return ceil_div(n, (int64_t)SA_B); }

static unsigned grid_for(int64_t n, int threads) {
  int64_t b = ceil_div(n, threads);
  int64_t cap = (int64_t)num_sms() * 16;
  return (unsigned)std::max<int64_t>(1, std::min(b, cap));
}

}  // namespace b200

using namespace b200;

extern "C" int b200_take_along_last(const float* x, const int64_t* idx, float* y, int64_t rows, int64_t cols, int64_t k,
                                    void* stream) {
  B200_REQUIRE(x && idx && y, "take_along_last: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && k >= 0, "take_along_last: bad sizes");
  if (rows * k == 0) return B200_OK;
  take_along_last_kernel<<<grid_for(rows * k, 256), 256, 0, as_stream(stream)>>>(x, idx, y, rows, cols, k);
  return check_launch("take_along_last");
}

extern "C" int b200_scatter_add_last(const float* base, const int64_t* idx, const float* src, float* y, int64_t rows,
                                     int64_t cols, int64_t k, void* stream) {
  B200_REQUIRE(idx && src && y, "scatter_add_last: null pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1 && k >= 0 && rows <= 2147483647LL, "scatter_add_last: bad sizes");
  B200_REQUIRE(base != y, "scatter_add_last: base and output must not alias");
  if (rows == 0) return B200_OK;
  scatter_add_last_kernel<<<(unsigned)rows, 128, 0, as_stream(stream)>>>(base, idx, src, y, rows, cols, k);
  return check_launch("scatter_add_last");
}

extern "C" int b200_take_rows(int dt, const void* table, const int64_t* ids, void* y, int64_t n, int64_t V, int64_t D,
                              void* stream) {
  B200_REQUIRE(table && ids && y, "take_rows: null pointer");
  B200_REQUIRE(n >= 0 && V >= 1 && D >= 0, "take_rows: bad sizes");
  if (n * D == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  if (dt == B200_F32 && D % 4 == 0 && (reinterpret_cast<uintptr_t>(table) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0)
    take_rows4_kernel<<<(unsigned)ceil_div(n, (int64_t)8), 256, 0, s>>>((const float*)table, ids, (float*)y, n, V, D);
  else if (dt == B200_F32)
    take_rows_kernel<float><<<grid_for(n * D, 256), 256, 0, s>>>((const float*)table, ids, (float*)y, n, V, D);
  else if (dt == B200_BF16)
    take_rows_kernel<__nv_bfloat16><<<grid_for(n * D, 256), 256, 0, s>>>((const __nv_bfloat16*)table, ids,
                                                                          (__nv_bfloat16*)y, n, V, D);
  else {
    set_error("take_rows: dtype %d", dt);
    return B200_ERR_DTYPE;
  }
  return check_launch("take_rows");
}

static size_t sa_al(size_t v) { return (v + 255) & ~size_t(255); }

extern "C" size_t b200_scatter_add_rows_workspace_bytes(int64_t n, int64_t V) {
  if (n <= 0 || V <= 0) return 0;
  const size_t G = (size_t)sa_blocks(n);
  // rank[n], cnt[G][V], tot[V], off[V + 1], perm[n]
  return sa_al(n * 4) + sa_al(G * V * 4) + sa_al(V * 4) + sa_al((V + 1) * 4) + sa_al(n * 4);
}

extern "C" int b200_scatter_add_rows(const float* src, const int64_t* ids, float* y, int64_t n, int64_t V, int64_t D,
                                     int accumulate, void* workspace, size_t workspace_bytes, void* stream) {
  B200_REQUIRE(src && ids && y, "scatter_add_rows: null pointer");
  B200_REQUIRE(n >= 0 && V >= 1 && D >= 0, "scatter_add_rows: bad sizes");
  B200_REQUIRE(n < 2147483647LL && V < 2147483647LL, "scatter_add_rows: too many rows");
  B200_REQUIRE(V * ceil_div(std::max<int64_t>(D, 1), (int64_t)256) < 2147483647LL, "scatter_add_rows: output too large");
  cudaStream_t s = as_stream(stream);
  if (n == 0 || D == 0) {
    if (!accumulate) cudaMemsetAsync(y, 0, (size_t)V * D * sizeof(float), s);
    return check_launch("scatter_add_rows(zero)");
  }
  const size_t need = b200_scatter_add_rows_workspace_bytes(n, V);
  B200_REQUIRE(workspace && workspace_bytes >= need, "scatter_add_rows: workspace %zu < %zu", workspace_bytes, need);
  const int64_t G = sa_blocks(n);
  uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
  int* rank = reinterpret_cast<int*>(w);
  w += sa_al(n * 4);
  int* cnt = reinterpret_cast<int*>(w);
  w += sa_al((size_t)G * V * 4);
  int* tot = reinterpret_cast<int*>(w);
  w += sa_al(V * 4);
  int* off = reinterpret_cast<int*>(w);
  w += sa_al((V + 1) * 4);
  int* perm = reinterpret_cast<int*>(w);
  cudaMemsetAsync(cnt, 0, (size_t)G * V * 4, s);
  sa_rank_kernel<<<(unsigned)G, SA_B, 0, s>>>(ids, rank, cnt, n, V);
  int rc = check_launch("scatter_add_rows(rank)");
  if (rc) return rc;
  sa_colscan_kernel<<<(unsigned)ceil_div(V, (int64_t)256), 256, 0, s>>>(cnt, tot, G, V);
  if ((rc = check_launch("scatter_add_rows(colscan)"))) return rc;
  sa_scan_kernel<<<1, 1024, 0, s>>>(tot, off, V);
  if ((rc = check_launch("scatter_add_rows(scan)"))) return rc;
  sa_place_kernel<<<(unsigned)ceil_div(n, (int64_t)256), 256, 0, s>>>(ids, rank, cnt, off, perm, n, V);
  if ((rc = check_launch("scatter_add_rows(place)"))) return rc;
  if (D % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    sa_sum4_kernel<<<(unsigned)ceil_div(V, (int64_t)8), 256, 0, s>>>(src, perm, off, y, V, D, accumulate);
    return check_launch("scatter_add_rows(sum)");
  }
  const int64_t dblocks = ceil_div(D, (int64_t)256);
  sa_sum_kernel<<<(unsigned)(V * dblocks), 256, 0, s>>>(src, perm, off, y, D, dblocks, accumulate);
  return check_launch("scatter_add_rows(sum)");
}

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

__global__ void scatter_add_rows_kernel(const float* __restrict__ src, const int64_t* __restrict__ ids, float* __restrict__ y,
                                        int64_t n, int64_t V, int64_t D) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n * D; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / D, d = e % D;
    int64_t v = ids[i];
    if (v < 0) v += V;
    if (v < 0 || v >= V) {
      raise_device_error(B200_ERR_ARG);
      continue;
    }
    atomicAdd(y + v * D + d, src[e]);
  }
}

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
  if (dt == B200_F32)
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

extern "C" int b200_scatter_add_rows(const float* src, const int64_t* ids, float* y, int64_t n, int64_t V, int64_t D,
                                     int accumulate, void* stream) {
  B200_REQUIRE(src && ids && y, "scatter_add_rows: null pointer");
  B200_REQUIRE(n >= 0 && V >= 1 && D >= 0, "scatter_add_rows: bad sizes");
  cudaStream_t s = as_stream(stream);
  if (!accumulate) cudaMemsetAsync(y, 0, (size_t)V * D * sizeof(float), s);
  if (n * D == 0) return check_launch("scatter_add_rows(zero)");
  scatter_add_rows_kernel<<<grid_for(n * D, 256), 256, 0, s>>>(src, ids, y, n, V, D);
  return check_launch("scatter_add_rows");
}

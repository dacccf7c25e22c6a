// Gather along any axis (np.take_along_axis with broadcasting of the other axes) and
// OneHot. Both walk the output index space with one thread per element over a strided
// view of at most B200_GATHER_MAX_DIM axes. Indices follow numpy: a negative index counts
// from the end of the axis; one outside [-len, len) sets the device error flag and the
// element is written as zero, never read out of bounds.
#include <algorithm>

#include "common.cuh"

namespace b200 {
namespace gat {

struct View {
  int ndim;
  int64_t shape[B200_GATHER_MAX_DIM];
  int64_t xs[B200_GATHER_MAX_DIM];  // element strides of x (0: broadcast); the axis entry is the axis stride
  int64_t is[B200_GATHER_MAX_DIM];  // element strides of the indices (0: broadcast)
};

template <typename T>
__global__ void gather_axis_kernel(const T* __restrict__ x, const int64_t* __restrict__ idx, T* __restrict__ y, int64_t n,
                                   int axis, int64_t axis_len, const __grid_constant__ View v) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, xo = 0, io = 0;
    for (int d = v.ndim - 1; d >= 0; --d) {
      const int64_t c = rem % v.shape[d];
      rem /= v.shape[d];
      io += c * v.is[d];
      if (d != axis) xo += c * v.xs[d];
    }
    int64_t j = idx[io];
    if (j < 0) j += axis_len;
    if (j < 0 || j >= axis_len) {
      raise_device_error(B200_ERR_ARG);
      y[e] = T(0);
      continue;
    }
    y[e] = x[xo + j * v.xs[axis]];
  }
}

// out[o, c, i] = (idx[o, i] == c ? on : off) as numpy computes eye(depth)[idx] * (on - off)
// + off in the output's arithmetic, then casts: fp32 output rounds (on - off) and off to
// fp32 and computes in fp32; every other output computes in fp64.
template <typename T>
__global__ void one_hot_kernel(const int64_t* __restrict__ idx, T* __restrict__ y, int64_t outer, int64_t depth,
                               int64_t inner, double diff, double off, int f32_math) {
  const int64_t n = outer * depth * inner;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e % inner, c = (e / inner) % depth, o = e / (inner * depth);
    int64_t j = idx[o * inner + i];
    if (j < 0) j += depth;
    if (j < 0 || j >= depth) {
      raise_device_error(B200_ERR_ARG);
      y[e] = T(0);
      continue;
    }
    const bool hot = j == c;
    double val;
    if (f32_math) {
      const float d32 = (float)diff, o32 = (float)off;
      val = (double)(__fadd_rn(__fmul_rn(hot ? 1.0f : 0.0f, d32), o32));
    } else {
      val = __dadd_rn(__dmul_rn(hot ? 1.0 : 0.0, diff), off);
    }
    y[e] = (T)val;
  }
}

template <>
__global__ void one_hot_kernel<uint8_t>(const int64_t* __restrict__ idx, uint8_t* __restrict__ y, int64_t outer, int64_t depth,
                                        int64_t inner, double diff, double off, int) {
  const int64_t n = outer * depth * inner;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e % inner, c = (e / inner) % depth, o = e / (inner * depth);
    int64_t j = idx[o * inner + i];
    if (j < 0) j += depth;
    if (j < 0 || j >= depth) {
      raise_device_error(B200_ERR_ARG);
      y[e] = 0;
      continue;
    }
    y[e] = (__dadd_rn(__dmul_rn(j == c ? 1.0 : 0.0, diff), off) != 0.0) ? 1 : 0;
  }
}

// dst[i] = src[i] over a strided index space (either side may be a strided view; src
// strides of 0 broadcast): the value write of IndexPut into a view of its cloned base
template <typename T>
__global__ void copy_strided_kernel(const T* __restrict__ src, T* __restrict__ dst, int64_t n, const __grid_constant__ View v) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, so = 0, dof = 0;
    for (int d = v.ndim - 1; d >= 0; --d) {
      const int64_t c = rem % v.shape[d];
      rem /= v.shape[d];
      so += c * v.xs[d];
      dof += c * v.is[d];
    }
    dst[dof] = src[so];
  }
}

inline int grid_for(int64_t n) {
  const int64_t want = ceil_div(n, 256);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 16));
}

}  // namespace gat
}  // namespace b200

using namespace b200;

extern "C" int b200_gather_axis(int elem_bytes, const void* x, const int64_t* x_strides, const int64_t* idx,
                                const int64_t* idx_strides, void* y, const int64_t* shape, int ndim, int axis,
                                int64_t axis_len, void* stream) {
  B200_REQUIRE(ndim >= 1 && ndim <= B200_GATHER_MAX_DIM, "gather_axis: ndim %d not in [1, %d]", ndim, B200_GATHER_MAX_DIM);
  B200_REQUIRE(axis >= 0 && axis < ndim, "gather_axis: axis %d out of range", axis);
  B200_REQUIRE(x_strides && idx_strides && shape, "gather_axis: null table");
  gat::View v;
  v.ndim = ndim;
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    B200_REQUIRE(shape[d] >= 0, "gather_axis: negative extent");
    v.shape[d] = shape[d];
    v.xs[d] = x_strides[d];
    v.is[d] = idx_strides[d];
    n *= shape[d];
  }
  if (n == 0) return B200_OK;
  B200_REQUIRE(x && idx && y, "gather_axis: null pointer");
  B200_REQUIRE(axis_len >= 1, "gather_axis: empty gather axis with a non-empty output");
  const int grid = gat::grid_for(n);
  cudaStream_t s = as_stream(stream);
  switch (elem_bytes) {
    case 1: gat::gather_axis_kernel<uint8_t><<<grid, 256, 0, s>>>((const uint8_t*)x, idx, (uint8_t*)y, n, axis, axis_len, v); break;
    case 2: gat::gather_axis_kernel<uint16_t><<<grid, 256, 0, s>>>((const uint16_t*)x, idx, (uint16_t*)y, n, axis, axis_len, v); break;
    case 4: gat::gather_axis_kernel<uint32_t><<<grid, 256, 0, s>>>((const uint32_t*)x, idx, (uint32_t*)y, n, axis, axis_len, v); break;
    case 8: gat::gather_axis_kernel<uint64_t><<<grid, 256, 0, s>>>((const uint64_t*)x, idx, (uint64_t*)y, n, axis, axis_len, v); break;
    default: B200_REQUIRE(false, "gather_axis: element size %d not in {1, 2, 4, 8}", elem_bytes);
  }
  return check_launch("gather_axis");
}

extern "C" int b200_one_hot(const int64_t* idx, void* y, int out_dtype, int64_t outer, int64_t depth, int64_t inner,
                            double on_value, double off_value, void* stream) {
  B200_REQUIRE(outer >= 0 && inner >= 0 && depth >= 0, "one_hot: negative extent");
  const int64_t n = outer * depth * inner;
  if (n == 0) return B200_OK;
  B200_REQUIRE(idx && y, "one_hot: null pointer");
  const double diff = on_value - off_value;
  const int grid = gat::grid_for(n);
  cudaStream_t s = as_stream(stream);
  switch (out_dtype) {
    case B200_F32: gat::one_hot_kernel<float><<<grid, 256, 0, s>>>(idx, (float*)y, outer, depth, inner, diff, off_value, 1); break;
    case B200_F64: gat::one_hot_kernel<double><<<grid, 256, 0, s>>>(idx, (double*)y, outer, depth, inner, diff, off_value, 0); break;
    case B200_I64:
      gat::one_hot_kernel<long long><<<grid, 256, 0, s>>>(idx, (long long*)y, outer, depth, inner, diff, off_value, 0);
      break;
    case B200_I32: gat::one_hot_kernel<int><<<grid, 256, 0, s>>>(idx, (int*)y, outer, depth, inner, diff, off_value, 0); break;
    case B200_BOOL: gat::one_hot_kernel<uint8_t><<<grid, 256, 0, s>>>(idx, (uint8_t*)y, outer, depth, inner, diff, off_value, 0); break;
    default: B200_REQUIRE(false, "one_hot: output dtype %d has no kernel", out_dtype);
  }
  return check_launch("one_hot");
}

extern "C" int b200_copy_strided(int elem_bytes, const void* src, const int64_t* src_strides, void* dst,
                                 const int64_t* dst_strides, const int64_t* shape, int ndim, void* stream) {
  B200_REQUIRE(ndim >= 1 && ndim <= B200_GATHER_MAX_DIM, "copy_strided: ndim %d not in [1, %d]", ndim, B200_GATHER_MAX_DIM);
  B200_REQUIRE(src_strides && dst_strides && shape, "copy_strided: null table");
  gat::View v;
  v.ndim = ndim;
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    B200_REQUIRE(shape[d] >= 0, "copy_strided: negative extent");
    v.shape[d] = shape[d];
    v.xs[d] = src_strides[d];
    v.is[d] = dst_strides[d];
    n *= shape[d];
  }
  if (n == 0) return B200_OK;
  B200_REQUIRE(src && dst, "copy_strided: null pointer");
  const int grid = gat::grid_for(n);
  cudaStream_t s = as_stream(stream);
  switch (elem_bytes) {
    case 1: gat::copy_strided_kernel<uint8_t><<<grid, 256, 0, s>>>((const uint8_t*)src, (uint8_t*)dst, n, v); break;
    case 2: gat::copy_strided_kernel<uint16_t><<<grid, 256, 0, s>>>((const uint16_t*)src, (uint16_t*)dst, n, v); break;
    case 4: gat::copy_strided_kernel<uint32_t><<<grid, 256, 0, s>>>((const uint32_t*)src, (uint32_t*)dst, n, v); break;
    case 8: gat::copy_strided_kernel<uint64_t><<<grid, 256, 0, s>>>((const uint64_t*)src, (uint64_t*)dst, n, v); break;
    default: B200_REQUIRE(false, "copy_strided: element size %d not in {1, 2, 4, 8}", elem_bytes);
  }
  return check_launch("copy_strided");
}

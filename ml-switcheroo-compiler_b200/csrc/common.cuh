// Shared host/device helpers for libb200.so: status codes, per-thread error text,
// launch accounting, the device error flag and small numeric helpers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/b200.h"

namespace b200 {

// Per-host-thread message of the last failing call.
void set_error(const char* fmt, ...);
// Count of kernel launches issued through this library.
void count_launch(uint64_t n = 1);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Check the launch that was just issued; returns B200_OK or B200_ERR_CUDA.
int check_launch(const char* what);

// Device-side error flag (index out of range, bounded wait gave up). Written with
// atomicCAS so the first error code wins; read and cleared by b200_check_device_error.
extern __device__ int g_device_error;
__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f32_to_bf16(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case B200_F32: return reinterpret_cast<const float*>(p)[i];
    case B200_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case B200_I64: return (float)reinterpret_cast<const long long*>(p)[i];
    case B200_BOOL: return reinterpret_cast<const uint8_t*>(p)[i] ? 1.0f : 0.0f;
    case B200_I32: return (float)reinterpret_cast<const int*>(p)[i];
    case B200_F64: return (float)reinterpret_cast<const double*>(p)[i];
  }
  return 0.0f;
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, int dtype, float v) {
  switch (dtype) {
    case B200_F32: reinterpret_cast<float*>(p)[i] = v; break;
    case B200_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case B200_I64: reinterpret_cast<long long*>(p)[i] = (long long)v; break;
    case B200_BOOL: reinterpret_cast<uint8_t*>(p)[i] = (v != 0.0f) ? 1 : 0; break;
    case B200_I32: reinterpret_cast<int*>(p)[i] = (int)v; break;
    case B200_F64: reinterpret_cast<double*>(p)[i] = (double)v; break;
  }
}

// tanh-approximation GELU, same formula as the reference forward
// (backends/eager/core_math_ops/math_nn.py:184-199).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

// Warp / block reductions (fp32).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over a whole block; `red` is >= 32 floats of shared memory. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.0f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : -INFINITY;
  return warp_max(t);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// number of SMs of the current device (cached per device)
int num_sms();

}  // namespace b200

#define B200_REQUIRE(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::b200::set_error(__VA_ARGS__);      \
      return B200_ERR_ARG;                 \
    }                                      \
  } while (0)

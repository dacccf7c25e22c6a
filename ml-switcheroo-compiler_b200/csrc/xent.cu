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
#include <algorithm>

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

// Rows whose columns fit in registers (V % 4 == 0, V <= XR_T * VPT, fp32 logits): the row
// is read from HBM once, exp(x - max) is evaluated once per element and kept, and dx is
// written in fp32 and/or bf16 (bf16 when it only feeds the output-projection GEMMs).
constexpr int XR_T = 512;

__device__ __forceinline__ void xr_cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void xr_cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void xr_cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Persistent over rows (one CTA per SM): while a row is reduced and its gradient written
// from registers, the CTA's next row streams into shared memory with cp.async, so HBM
// reads overlap the math and the stores. Thread t copies and later reads only its own
// float4 slots, so the staging buffer needs no barrier. Each thread keeps its own
// (max m_t, sum of exp(x - m_t)) over its columns and the exponentials themselves; one
// block-wide merge of the (m, s) pairs gives the row's max M and sum S, and the gradient
// is then e * exp(m_t - M) / S per element: one exp2 per element and two barriers per row.
constexpr float XR_LOG2E = 1.4426950408889634f;

// (m, s) pairs: s sums exp(x - m); merged with the larger maximum
__device__ __forceinline__ void xr_merge(float& m, float& s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  const float a = m == -INFINITY ? 0.f : s * exp2f((m - M) * XR_LOG2E);
  const float b = m2 == -INFINITY ? 0.f : s2 * exp2f((m2 - M) * XR_LOG2E);
  m = M;
  s = a + b;
}

template <int VPT>
__global__ void __launch_bounds__(XR_T, 1) xent_reg_kernel(const float* __restrict__ x, const int64_t* __restrict__ label,
                                                           const float* __restrict__ d, float* __restrict__ picked,
                                                           float* __restrict__ dx, __nv_bfloat16* __restrict__ dxb, int64_t V,
                                                           int64_t rows) {
  __shared__ float redm[32], reds[32], fin[2];
  extern __shared__ float4 stage[];  // [NC][XR_T]: the next row
  constexpr int NC = VPT / 4;
  const int64_t G = gridDim.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  auto prefetch = [&](int64_t r) {
    if (r < rows) {
      const float* xr = x + r * V;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int64_t col = ((int64_t)c * XR_T + threadIdx.x) * 4;
        if (col < V) xr_cp_async16(&stage[c * XR_T + threadIdx.x], xr + col);
      }
    }
    xr_cp_async_commit();
  };
  prefetch(blockIdx.x);
  for (int64_t r = blockIdx.x; r < rows; r += G) {
    int64_t lab = label[r];
    if (lab < 0) lab += V;
    const bool ok = lab >= 0 && lab < V;
    xr_cp_async_wait_all();
    float v[NC][4];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int64_t col = ((int64_t)c * XR_T + threadIdx.x) * 4;
      if (col < V) {
        const float4 t = stage[c * XR_T + threadIdx.x];
        v[c][0] = t.x; v[c][1] = t.y; v[c][2] = t.z; v[c][3] = t.w;
      } else {
        v[c][0] = v[c][1] = v[c][2] = v[c][3] = -INFINITY;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) m = fmaxf(m, v[c][k]);
    }
    prefetch(r + G);  // this thread's slots are in registers now
    // e = exp(x - m_t), kept in place of x
    float s = 0.f;
    const float ml = m * XR_LOG2E;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float e = v[c][k] == -INFINITY ? 0.f : exp2f(fmaf(v[c][k], XR_LOG2E, -ml));
        v[c][k] = e;
        s += e;
      }
    // block merge of the (m, s) pairs
    float bm = m, bs = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, bm, o), s2 = __shfl_xor_sync(0xffffffffu, bs, o);
      xr_merge(bm, bs, m2, s2);
    }
    if (lane == 0) {
      redm[wid] = bm;
      reds[wid] = bs;
    }
    __syncthreads();
    if (wid == 0) {
      constexpr int NW = XR_T / 32;
      bm = lane < NW ? redm[lane] : -INFINITY;
      bs = lane < NW ? reds[lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, bm, o), s2 = __shfl_xor_sync(0xffffffffu, bs, o);
        xr_merge(bm, bs, m2, s2);
      }
      if (lane == 0) {
        fin[0] = bm;
        fin[1] = bs;
      }
    }
    __syncthreads();
    const float M = fin[0], S = fin[1];
    const float lse = M + logf(S);
    // the label's logit, read back by one thread (the row is in L2)
    if (threadIdx.x == 0) {
      if (!ok) raise_device_error(B200_ERR_ARG);
      if (picked) picked[r] = ok ? __ldg(x + r * V + lab) - lse : 0.f;
    }
    if (!dx && !dxb) continue;
    // softmax = e * exp(m_t - M) / S; dx = d * ([j == label] - softmax)
    const float dr = d[r];
    const float sc = m == -INFINITY ? 0.f : exp2f((m - M) * XR_LOG2E) / S;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int64_t col = ((int64_t)c * XR_T + threadIdx.x) * 4;
      if (col >= V) continue;
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = dr * ((col + k == lab ? 1.f : 0.f) - v[c][k] * sc);
      if (dx) __stcs(reinterpret_cast<float4*>(dx + r * V + col), make_float4(o[0], o[1], o[2], o[3]));
      if (dxb) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&lo);
        u.y = *reinterpret_cast<uint32_t*>(&hi);
        __stcs(reinterpret_cast<uint2*>(dxb + r * V + col), u);
      }
    }
  }
  xr_cp_async_wait_all();
}

template <int VPT>
void launch_xent_reg(const float* x, const int64_t* label, const float* d, float* picked, float* dx, __nv_bfloat16* dxb,
                     int64_t V, int64_t rows, cudaStream_t s) {
  const size_t smem = (size_t)VPT * XR_T * sizeof(float);
  static bool attr = false;
  if (!attr && smem > 48 * 1024) {
    cudaFuncSetAttribute(xent_reg_kernel<VPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  const int64_t grid = std::min<int64_t>(rows, (int64_t)num_sms());
  xent_reg_kernel<VPT><<<(unsigned)grid, XR_T, smem, s>>>(x, label, d, picked, dx, dxb, V, rows);
}

}  // namespace b200

using namespace b200;

extern "C" int b200_logsoftmax_pick(int x_dtype, const void* x, const int64_t* label, const float* d, float* picked,
                                    float* ls, float* dx, void* dx_bf16, int64_t rows, int64_t cols, void* stream) {
  B200_REQUIRE(x && label, "logsoftmax_pick: null input");
  B200_REQUIRE(!(dx || dx_bf16) || d, "logsoftmax_pick: dx needs the cotangent d");
  B200_REQUIRE(rows >= 0 && cols >= 1 && rows <= 2147483647LL, "logsoftmax_pick: bad sizes");
  if (rows == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  auto al = [](const void* p, int b) { return (reinterpret_cast<uintptr_t>(p) % b) == 0; };
  const bool reg = x_dtype == B200_F32 && !ls && cols % 4 == 0 && cols <= (int64_t)XR_T * 64 && al(x, 16) &&
                   (!dx || al(dx, 16)) && (!dx_bf16 || al(dx_bf16, 8));
  if (reg) {
    const int vpt = (int)ceil_div(ceil_div(cols, (int64_t)XR_T), (int64_t)4) * 4;
    auto* db = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
    const float* xf = (const float*)x;
    if (vpt <= 4) launch_xent_reg<4>(xf, label, d, picked, dx, db, cols, rows, s);
    else if (vpt <= 8) launch_xent_reg<8>(xf, label, d, picked, dx, db, cols, rows, s);
    else if (vpt <= 16) launch_xent_reg<16>(xf, label, d, picked, dx, db, cols, rows, s);
    else if (vpt <= 32) launch_xent_reg<32>(xf, label, d, picked, dx, db, cols, rows, s);
    else launch_xent_reg<64>(xf, label, d, picked, dx, db, cols, rows, s);
    return check_launch("logsoftmax_pick(rows in registers)");
  }
  B200_REQUIRE(!dx_bf16, "logsoftmax_pick: bf16 dx needs fp32 logits with cols %% 4 == 0");
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

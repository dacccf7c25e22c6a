// Optimizer update steps on the device: ApplyAdam, ApplyAdagrad, ApplyFtrl, ApplyRMSProp
// as the reference's numpy backend computes them (numpy/eager/optimizers_ops.py:11-103;
// that registry wins over the generic one for these names, numpy/eager/__init__.py:110-115).
// The hyperparameters the numpy kernels fix are fixed here too: Adam beta1 0.9, beta2
// 0.999, eps 1e-8, no bias correction; Adagrad eps 1e-10; RMSProp rho 0.9, momentum 0,
// eps 1e-8; FTRL in the numpy form (p - lr g; linear - g + sigma p).
//
// numpy evaluates these expressions in fp32 (a Python-float scalar takes the array's
// dtype), one IEEE rounding per operation, in source order, without fused multiply-adds.
// Every operation below is the matching round-to-nearest intrinsic (__fmul_rn, __fadd_rn,
// __fsub_rn, __fdiv_rn, __fsqrt_rn), so the compiler cannot contract or reorder them and
// the results are bit-identical to the reference's. The scalar constants are the fp32
// roundings of the same double values (1.0 - 0.9 and so on), computed on the host.
//
// One element = one read of param, the state arrays and grad and one write of param and
// the states: HBM-bound (Adam 28 bytes per element). Outputs may alias inputs (in-place
// update): each element is read and written by the same thread.
#include <algorithm>

#include "optim_math.cuh"

namespace b200 {
namespace opt {

struct Tensor {
  const float *p, *s1, *s2, *g;
  float *po, *s1o, *s2o;
  int64_t n;
};

constexpr int OT = 256;
constexpr int MAXT = 128;  // tensors per launch (8 KB of kernel parameters)

struct Batch {
  Tensor t[MAXT];
};

// grid.y = tensor; each thread walks its elements 4 at a time (float4 when aligned)
__global__ void __launch_bounds__(OT) apply_kernel(const __grid_constant__ Batch B, int kind, Consts k) {
  const Tensor& t = B.t[blockIdx.y];
  const bool two = kind != ADAGRAD;  // a second state array
  const bool vec = ((reinterpret_cast<uintptr_t>(t.p) | reinterpret_cast<uintptr_t>(t.s1) | reinterpret_cast<uintptr_t>(t.g) |
                     reinterpret_cast<uintptr_t>(t.po) | reinterpret_cast<uintptr_t>(t.s1o) |
                     (two ? (reinterpret_cast<uintptr_t>(t.s2) | reinterpret_cast<uintptr_t>(t.s2o)) : 0)) & 15) == 0;
  const int64_t stride = (int64_t)gridDim.x * OT * 4;
  for (int64_t i0 = ((int64_t)blockIdx.x * OT + threadIdx.x) * 4; i0 < t.n; i0 += stride) {
    if (vec && i0 + 4 <= t.n) {
      const float4 p = *reinterpret_cast<const float4*>(t.p + i0);
      const float4 a = *reinterpret_cast<const float4*>(t.s1 + i0);
      const float4 b = two ? *reinterpret_cast<const float4*>(t.s2 + i0) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 g = *reinterpret_cast<const float4*>(t.g + i0);
      float4 po, ao, bo;
      update(kind, k, p.x, a.x, b.x, g.x, po.x, ao.x, bo.x);
      update(kind, k, p.y, a.y, b.y, g.y, po.y, ao.y, bo.y);
      update(kind, k, p.z, a.z, b.z, g.z, po.z, ao.z, bo.z);
      update(kind, k, p.w, a.w, b.w, g.w, po.w, ao.w, bo.w);
      __stcs(reinterpret_cast<float4*>(t.po + i0), po);
      __stcs(reinterpret_cast<float4*>(t.s1o + i0), ao);
      if (two) __stcs(reinterpret_cast<float4*>(t.s2o + i0), bo);
    } else {
      for (int64_t i = i0; i < min(i0 + 4, t.n); ++i) {
        float po, ao, bo;
        update(kind, k, t.p[i], t.s1[i], two ? t.s2[i] : 0.f, t.g[i], po, ao, bo);
        t.po[i] = po;
        t.s1o[i] = ao;
        if (two) t.s2o[i] = bo;
      }
    }
  }
}


}  // namespace opt
}  // namespace b200

using namespace b200;

extern "C" double b200_optimizer_default_lr(int kind) {
  switch (kind) {
    case opt::ADAM: return 0.001;
    case opt::ADAGRAD: return 0.01;
    case opt::FTRL: return 0.001;
    case opt::RMSPROP: return 0.001;
    default: return 0.0;
  }
}

extern "C" int b200_apply_optimizer_f32(int kind, int count, const float* const* param, const float* const* s1,
                                        const float* const* s2, const float* const* grad, float* const* param_out,
                                        float* const* s1_out, float* const* s2_out, const int64_t* n, float lr, void* stream) {
  B200_REQUIRE(kind >= 0 && kind <= 3, "apply_optimizer: kind %d not in [0, 3]", kind);
  B200_REQUIRE(count >= 0, "apply_optimizer: count %d", count);
  if (count == 0) return B200_OK;
  B200_REQUIRE(param && s1 && grad && param_out && s1_out && n, "apply_optimizer: null pointer table");
  const bool two = kind != opt::ADAGRAD;
  B200_REQUIRE(!two || (s2 && s2_out), "apply_optimizer: this optimizer has a second state array");
  cudaStream_t st = as_stream(stream);
  const opt::Consts k = opt::consts_for(kind, lr);
  for (int base = 0; base < count; base += opt::MAXT) {
    opt::Batch B;
    int64_t max_n = 0;
    const int m = std::min(opt::MAXT, count - base);
    for (int i = 0; i < m; ++i) {
      const int j = base + i;
      B200_REQUIRE(n[j] >= 0, "apply_optimizer: negative size of tensor %d", j);
      B200_REQUIRE(n[j] == 0 || (param[j] && s1[j] && grad[j] && param_out[j] && s1_out[j] && (!two || (s2[j] && s2_out[j]))),
                   "apply_optimizer: null pointer for tensor %d", j);
      B.t[i] = {param[j], s1[j], two ? s2[j] : nullptr, grad[j], param_out[j], s1_out[j], two ? s2_out[j] : nullptr, n[j]};
      max_n = std::max(max_n, n[j]);
    }
    if (max_n == 0) continue;
    const int64_t per = (int64_t)opt::OT * 4;
    const int64_t gx = std::min<int64_t>(ceil_div(max_n, per), (int64_t)num_sms() * 8);
    opt::apply_kernel<<<dim3((unsigned)gx, (unsigned)m), opt::OT, 0, st>>>(B, kind, k);
    const int rc = check_launch("apply_optimizer");
    if (rc) return rc;
  }
  return B200_OK;
}

// Per-element optimizer updates shared by the optimizer kernel (optim.cu) and the fused
// all-reduce + optimizer epilogue (peer.cu): the reference numpy backend's formulas
// (numpy/eager/optimizers_ops.py:11-103) with one IEEE round-to-nearest intrinsic per
// operation in the same order, so both kernels and the reference agree bit for bit.
#pragma once
#include "common.cuh"

namespace b200 {
namespace opt {

enum Kind { ADAM = 0, ADAGRAD = 1, FTRL = 2, RMSPROP = 3 };

struct Consts {
  float lr, c0, c1, c2, c3, eps;
};

// one element; s1, s2 are the state values (unused ones ignored)
__device__ __forceinline__ void update(int kind, const Consts& k, float p, float s1, float s2, float g, float& po, float& s1o,
                                       float& s2o) {
  if (kind == ADAM) {  // c0 beta1, c1 1 - beta1, c2 beta2, c3 1 - beta2
    const float m = __fadd_rn(__fmul_rn(s1, k.c0), __fmul_rn(g, k.c1));
    const float v = __fadd_rn(__fmul_rn(s2, k.c2), __fmul_rn(__fmul_rn(g, g), k.c3));
    const float u = __fdiv_rn(m, __fadd_rn(__fsqrt_rn(v), k.eps));
    po = __fsub_rn(p, __fmul_rn(k.lr, u));
    s1o = m;
    s2o = v;
  } else if (kind == ADAGRAD) {
    const float a = __fadd_rn(s1, __fmul_rn(g, g));
    const float u = __fdiv_rn(g, __fadd_rn(__fsqrt_rn(a), k.eps));
    po = __fsub_rn(p, __fmul_rn(k.lr, u));
    s1o = a;
    s2o = s2;
  } else if (kind == FTRL) {  // s1 accum, s2 linear
    const float a = __fadd_rn(s1, __fmul_rn(g, g));
    const float sigma = __fdiv_rn(__fsub_rn(__fsqrt_rn(a), __fsqrt_rn(s1)), k.lr);
    s2o = __fadd_rn(__fsub_rn(s2, g), __fmul_rn(sigma, p));
    po = __fsub_rn(p, __fmul_rn(k.lr, g));
    s1o = a;
  } else {  // RMSProp: c0 rho, c1 1 - rho, c2 momentum; s1 ms, s2 mom
    const float m = __fadd_rn(__fmul_rn(s1, k.c0), __fmul_rn(__fmul_rn(g, g), k.c1));
    const float mo = __fadd_rn(__fmul_rn(s2, k.c2), __fdiv_rn(g, __fadd_rn(__fsqrt_rn(m), k.eps)));
    po = __fsub_rn(p, __fmul_rn(k.lr, mo));
    s1o = m;
    s2o = mo;
  }
}

inline Consts consts_for(int kind, float lr) {
  Consts k{lr, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (kind == ADAM) {
    k.c0 = (float)0.9; k.c1 = (float)(1.0 - 0.9); k.c2 = (float)0.999; k.c3 = (float)(1.0 - 0.999); k.eps = (float)1e-8;
  } else if (kind == ADAGRAD) {
    k.eps = (float)1e-10;
  } else if (kind == RMSPROP) {
    k.c0 = (float)0.9; k.c1 = (float)(1.0 - 0.9); k.c2 = 0.f; k.eps = (float)1e-8;
  }
  return k;
}

}  // namespace opt
}  // namespace b200

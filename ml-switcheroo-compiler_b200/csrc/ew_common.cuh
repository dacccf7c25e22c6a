// Shared by the elementwise program kernels: launch parameters and fast division.
#pragma once
#include "common.cuh"

namespace b200 {

struct EwParams {
  b200_ew_program p;
  const void* in[B200_EW_MAX_IN];
  void* out[B200_EW_MAX_OUT];
  int64_t n;
  // 32-bit strided path: per-dim size, fast-division multiplier and shift, 32-bit strides
  uint32_t dsz[B200_EW_MAX_DIM], dmul[B200_EW_MAX_DIM], dshr[B200_EW_MAX_DIM];
  int32_t st32[B200_EW_MAX_IN][B200_EW_MAX_DIM];
  // flat path: per-input mode (0 dense, 1 scalar, 2 vector along the last dim, 3 one
  // value per row of the last dim), the last-dim length (fast division), whether
  // 8-element groups never straddle rows (lastdim % 8 == 0), and which inputs / outputs
  // may use 128-bit accesses
  int32_t mode[B200_EW_MAX_IN];
  int64_t lastdim;
  uint32_t ld_mul, ld_shr;
  int32_t ld8;
  int32_t vin[B200_EW_MAX_IN], vout[B200_EW_MAX_OUT];
  // specialised straight-line programs: kind (0 generic, 1 copy/cast, 2 unary, 3 binary),
  // op, and the input feeding each operand
  int32_t kind, sop, sa, sb;
  // kind 4: a left fold of additions over inputs sumord[0 .. nsum) (in that order)
  int32_t nsum, sumord[B200_EW_MAX_IN];
  // kind 5: a chain of up to 4 unary / binary ops, t = op_k(x, y), each operand an input
  // (index >= 0), an immediate (-1, value in cimm) or the previous op's result (-2)
  int32_t nchain, cop[4], csrc[4][2];
  float cimm[4][2];
};

// n / d for 32-bit n with a precomputed (mul, shr): q = (umulhi(n, mul) + n) >> shr
__device__ __forceinline__ uint32_t fast_div(uint32_t n, uint32_t mul, uint32_t shr) {
  return (uint32_t)(((uint64_t)__umulhi(n, mul) + n) >> shr);
}
inline void fastdiv_params(uint32_t d, uint32_t& mul, uint32_t& shr) {
  uint32_t l = 0;
  while (((uint64_t)1 << l) < d) ++l;
  mul = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << l) - d)) / d + 1);
  if (d == 1) mul = 0;
  shr = l;
}


// Flat-path launch (every input dense, scalar, a last-dim vector or a row scalar);
// defined in elementwise_flat.cu.
int ew_flat_launch(EwParams& P, cudaStream_t s);

}  // namespace b200

// Flat-path elementwise programs: every input is dense over the output index space, a
// scalar, a vector along the last dim, or one value per row of the last dim. Each
// thread handles groups of 8 consecutive elements (two 128-bit fp32 accesses, one
// 128-bit bf16 access per operand).
//
// The register program runs from a register-resident file: registers are selected by
// a warp-uniform switch over compile-time indices (the file is sized to the program,
// 4 / 8 / 16 registers), and each instruction is dispatched once per 4 elements.
// Programs that are a single cast, unary or binary op run as straight-line kernels.
#include <math.h>

#include "ew_common.cuh"

namespace b200 {
namespace ewf {

constexpr int THREADS = 256;
constexpr int V = 8;   // elements per thread-group in the straight-line kernels
constexpr int VG = 4;  // elements per thread-group in the register-program kernel

__device__ __forceinline__ float bf2f(uint32_t h) { return __uint_as_float(h << 16); }

// VV (4 or 8) consecutive elements of a contiguous run starting at `idx` (dense / vector)
template <int VV>
__device__ __forceinline__ void load_run(const void* src, int dt, int vec, int64_t idx, float (&o)[VV]) {
  if (vec && dt == B200_F32) {
#pragma unroll
    for (int h = 0; h < VV / 4; ++h) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx + 4 * h));
      o[4 * h] = a.x; o[4 * h + 1] = a.y; o[4 * h + 2] = a.z; o[4 * h + 3] = a.w;
    }
  } else if (vec && dt == B200_BF16 && VV == 8) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src) + idx));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < VV / 2; ++h) {
      o[2 * h] = bf2f(w[h] & 0xFFFFu);
      o[2 * h + 1] = bf2f(w[h] >> 16);
    }
  } else if (vec && dt == B200_BF16) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(src) + idx));
    o[0] = bf2f(u.x & 0xFFFFu); o[1] = bf2f(u.x >> 16);
    o[2 % VV] = bf2f(u.y & 0xFFFFu); o[3 % VV] = bf2f(u.y >> 16);
  } else {
#pragma unroll
    for (int k = 0; k < VV; ++k) o[k] = load_as_f32(src, idx + k, dt);
  }
}

template <int VV>
__device__ __forceinline__ void loadv(const EwParams& P, int j, int64_t base, bool full, float (&o)[VV]) {
  const void* src = P.in[j];
  const int dt = P.p.in_dtype[j];
  const int mode = P.mode[j];
  if (mode == 1) {
    const float s = load_as_f32(src, 0, dt);
#pragma unroll
    for (int k = 0; k < VV; ++k) o[k] = s;
    return;
  }
  if (full && (mode == 0 || (VV == 8 ? P.ld8 : (P.lastdim % 4 == 0)))) {
    if (mode == 0) {
      load_run<VV>(src, dt, P.vin[j], base, o);
    } else {
      const uint32_t b32 = (uint32_t)base;
      const uint32_t row = fast_div(b32, P.ld_mul, P.ld_shr);
      if (mode == 2) {
        load_run<VV>(src, dt, P.vin[j], (int64_t)(b32 - row * (uint32_t)P.lastdim), o);
      } else {
        const float s = load_as_f32(src, row, dt);
#pragma unroll
        for (int k = 0; k < VV; ++k) o[k] = s;
      }
    }
    return;
  }
  // ragged tail, or rows that do not hold whole groups: element by element
#pragma unroll
  for (int k = 0; k < VV; ++k) {
    const int64_t e = base + k;
    if (e >= P.n) {
      o[k] = 0.f;
      continue;
    }
    int64_t idx = e;
    if (mode != 0) {
      const uint32_t e32 = (uint32_t)e;
      const uint32_t row = fast_div(e32, P.ld_mul, P.ld_shr);
      idx = (mode == 2) ? (int64_t)(e32 - row * (uint32_t)P.lastdim) : (int64_t)row;
    }
    o[k] = load_as_f32(src, idx, dt);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

template <int VV>
__device__ __forceinline__ void storev(const EwParams& P, int o, int64_t base, bool full, const float (&x)[VV]) {
  void* dst = P.out[o];
  const int dt = P.p.out_dtype[o];
  if (full && P.vout[o]) {
    if (dt == B200_F32) {
      float* d = reinterpret_cast<float*>(dst) + base;
#pragma unroll
      for (int h = 0; h < VV / 4; ++h) reinterpret_cast<float4*>(d)[h] = make_float4(x[4 * h], x[4 * h + 1], x[4 * h + 2], x[4 * h + 3]);
      return;
    }
    if (dt == B200_BF16) {
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst) + base;
      if (VV == 8)
        *reinterpret_cast<uint4*>(d) = make_uint4(pack2(x[0], x[1]), pack2(x[2 % VV], x[3 % VV]), pack2(x[4 % VV], x[5 % VV]),
                                                  pack2(x[6 % VV], x[7 % VV]));
      else
        *reinterpret_cast<uint2*>(d) = make_uint2(pack2(x[0], x[1]), pack2(x[2 % VV], x[3 % VV]));
      return;
    }
    if (dt == B200_BOOL && VV == 8) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        lo |= (x[k] != 0.f ? 1u : 0u) << (8 * k);
        hi |= (x[(k + 4) % VV] != 0.f ? 1u : 0u) << (8 * k);
      }
      *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(dst) + base) = make_uint2(lo, hi);
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < VV; ++k)
    if (base + k < P.n) store_from_f32(dst, base + k, dt, x[k]);
}

// ---------------- op semantics (fp32) ----------------
__device__ __forceinline__ float apply1(int op, float x) {
  switch (op) {
    case B200_EW_NEG: return -x;
    case B200_EW_EXP: return expf(x);
    case B200_EW_LOG: return logf(x);
    case B200_EW_TANH: return tanhf(x);
    case B200_EW_SQRT: return sqrtf(x);
    case B200_EW_RELU: return x > 0.f ? x : 0.f;
    case B200_EW_GELU: return gelu_tanh(x);
    case B200_EW_ABS: return fabsf(x);
    case B200_EW_SIGMOID: return 1.f / (1.f + expf(-x));
    case B200_EW_ERF: return erff(x);
    case B200_EW_RECIP: return 1.f / x;
    default: return x;  // MOV
  }
}

template <int OP>
__device__ __forceinline__ float apply2(float x, float y) {
  if (OP == B200_EW_ADD) return x + y;
  if (OP == B200_EW_SUB) return x - y;
  if (OP == B200_EW_MUL) return x * y;
  if (OP == B200_EW_DIV) return x / y;
  if (OP == B200_EW_MAX) return fmaxf(x, y);
  if (OP == B200_EW_MIN) return fminf(x, y);
  if (OP == B200_EW_POW) return powf(x, y);
  if (OP == B200_EW_GT) return (x > y) ? 1.f : 0.f;
  if (OP == B200_EW_GE) return (x >= y) ? 1.f : 0.f;
  if (OP == B200_EW_LT) return (x < y) ? 1.f : 0.f;
  return (x == y) ? 1.f : 0.f;  // EQ
}

// ---------------- register file (constant indices only) ----------------
template <int NREG>
__device__ __forceinline__ void rd(const float (&R)[NREG][VG], int k, float (&o)[VG]) {
#define B200_RD(i)                                     \
  case i:                                              \
    if constexpr (i < NREG) {                          \
      _Pragma("unroll") for (int v = 0; v < VG; ++v) o[v] = R[i][v]; \
    }                                                  \
    break;
  switch (k) {
    B200_RD(0) B200_RD(1) B200_RD(2) B200_RD(3) B200_RD(4) B200_RD(5) B200_RD(6) B200_RD(7)
    B200_RD(8) B200_RD(9) B200_RD(10) B200_RD(11) B200_RD(12) B200_RD(13) B200_RD(14) B200_RD(15)
    default: break;
  }
#undef B200_RD
}

template <int NREG>
__device__ __forceinline__ void wr(float (&R)[NREG][VG], int k, const float (&x)[VG]) {
#define B200_WR(i)                                     \
  case i:                                              \
    if constexpr (i < NREG) {                          \
      _Pragma("unroll") for (int v = 0; v < VG; ++v) R[i][v] = x[v]; \
    }                                                  \
    break;
  switch (k) {
    B200_WR(0) B200_WR(1) B200_WR(2) B200_WR(3) B200_WR(4) B200_WR(5) B200_WR(6) B200_WR(7)
    B200_WR(8) B200_WR(9) B200_WR(10) B200_WR(11) B200_WR(12) B200_WR(13) B200_WR(14) B200_WR(15)
    default: break;
  }
#undef B200_WR
}

// NIN: input slots held in registers (2, 4 or the maximum 8): the loaded-up-front inputs
// take NIN x VG registers, so small programs keep their register count (and the SM's
// occupancy) low
template <int NREG, int NIN>
__global__ void __launch_bounds__(THREADS) ew_prog_kernel(const __grid_constant__ EwParams P) {
  const b200_ew_program& p = P.p;
  float R[NREG][VG];
#pragma unroll
  for (int i = 0; i < NREG; ++i)
#pragma unroll
    for (int v = 0; v < VG; ++v) R[i][v] = 0.f;
  const int64_t ng = (P.n + VG - 1) / VG;
  const int nins = p.n_ins;
  const int nin = p.n_in;
  for (int64_t q = blockIdx.x * (int64_t)THREADS + threadIdx.x; q < ng; q += (int64_t)gridDim.x * THREADS) {
    const int64_t base = q * VG;
    const bool full = base + VG <= P.n;
    // every input of the group is loaded up front, so the loads of all inputs are in
    // flight together; LOAD instructions then read these registers
    float IN[NIN][VG];
#pragma unroll
    for (int j = 0; j < NIN; ++j)
      if (j < nin) loadv<VG>(P, j, base, full, IN[j]);
    for (int i = 0; i < nins; ++i) {
      const b200_ew_ins I = p.ins[i];
      float x[VG], y[VG], res[VG];
      if (I.op == B200_EW_LOAD) {
        switch (I.a) {
#define B200_LDIN(j)                                                                          \
  case j:                                                                                     \
    if constexpr (j < NIN) {                                                                  \
      _Pragma("unroll") for (int v = 0; v < VG; ++v) res[v] = IN[j][v];                       \
    }                                                                                         \
    break;
          B200_LDIN(0) B200_LDIN(1) B200_LDIN(2) B200_LDIN(3) B200_LDIN(4) B200_LDIN(5) B200_LDIN(6) B200_LDIN(7)
#undef B200_LDIN
          default: break;
        }
        wr<NREG>(R, I.dst, res);
        continue;
      }
      if (I.op == B200_EW_STORE) {
        rd<NREG>(R, I.a, x);
        storev<VG>(P, I.dst, base, full, x);
        continue;
      }
      if (I.op == B200_EW_IMM) {
#pragma unroll
        for (int v = 0; v < VG; ++v) res[v] = I.imm;
        wr<NREG>(R, I.dst, res);
        continue;
      }
      rd<NREG>(R, I.a, x);
      rd<NREG>(R, I.b, y);
      switch (I.op) {
#define B200_BIN(OPC)                                                         \
  case OPC:                                                                   \
    _Pragma("unroll") for (int v = 0; v < VG; ++v) res[v] = apply2<OPC>(x[v], y[v]); \
    break;
        B200_BIN(B200_EW_ADD) B200_BIN(B200_EW_SUB) B200_BIN(B200_EW_MUL) B200_BIN(B200_EW_DIV)
        B200_BIN(B200_EW_MAX) B200_BIN(B200_EW_MIN) B200_BIN(B200_EW_POW) B200_BIN(B200_EW_GT)
        B200_BIN(B200_EW_GE) B200_BIN(B200_EW_LT) B200_BIN(B200_EW_EQ)
#undef B200_BIN
        case B200_EW_WHERE:
        case B200_EW_FMA: {
          float z[VG];
          rd<NREG>(R, I.c, z);
          if (I.op == B200_EW_WHERE) {
#pragma unroll
            for (int v = 0; v < VG; ++v) res[v] = (x[v] != 0.f) ? y[v] : z[v];
          } else {
#pragma unroll
            for (int v = 0; v < VG; ++v) res[v] = fmaf(x[v], y[v], z[v]);
          }
          break;
        }
        default: {
          const int op = I.op;
#pragma unroll
          for (int v = 0; v < VG; ++v) res[v] = apply1(op, x[v]);
        }
      }
      wr<NREG>(R, I.dst, res);
    }
  }
}

// straight-line programs: y = op(in[sa]) or y = op(in[sa], in[sb]) stored to every output
template <int OP>
__global__ void __launch_bounds__(THREADS) ew_bin8_kernel(const __grid_constant__ EwParams P) {
  const int64_t ng = (P.n + V - 1) / V;
  const int nout = P.p.n_out;
  for (int64_t q = blockIdx.x * (int64_t)THREADS + threadIdx.x; q < ng; q += (int64_t)gridDim.x * THREADS) {
    const int64_t base = q * V;
    const bool full = base + V <= P.n;
    float x[V], y[V], r[V];
    loadv<V>(P, P.sa, base, full, x);
    loadv<V>(P, P.sb, base, full, y);
#pragma unroll
    for (int v = 0; v < V; ++v) r[v] = apply2<OP>(x[v], y[v]);
    for (int o = 0; o < nout; ++o) storev<V>(P, o, base, full, r);
  }
}

__global__ void __launch_bounds__(THREADS) ew_un8_kernel(const __grid_constant__ EwParams P) {
  const int64_t ng = (P.n + V - 1) / V;
  const int nout = P.p.n_out;
  const int op = P.sop;
  for (int64_t q = blockIdx.x * (int64_t)THREADS + threadIdx.x; q < ng; q += (int64_t)gridDim.x * THREADS) {
    const int64_t base = q * V;
    const bool full = base + V <= P.n;
    float x[V];
    loadv<V>(P, P.sa, base, full, x);
    if (op != B200_EW_MOV) {
#pragma unroll
      for (int v = 0; v < V; ++v) x[v] = apply1(op, x[v]);
    }
    for (int o = 0; o < nout; ++o) storev<V>(P, o, base, full, x);
  }
}

// a chain of up to 4 ops, each operand an input, an immediate or the previous result
// (e.g. (x > 0) * dy, or g * 1/36): straight-line per op (one warp-uniform dispatch per
// op and 8 elements), no register file
template <int OPK>
__device__ __forceinline__ void apply_rt(int op, const float (&x)[V], const float (&y)[V], float (&r)[V]) {
  switch (op) {
#define B200_CH2(OPC)                                         \
  case OPC:                                                   \
    _Pragma("unroll") for (int v = 0; v < V; ++v) r[v] = apply2<OPC>(x[v], y[v]); \
    return;
    B200_CH2(B200_EW_ADD) B200_CH2(B200_EW_SUB) B200_CH2(B200_EW_MUL) B200_CH2(B200_EW_DIV) B200_CH2(B200_EW_MAX)
    B200_CH2(B200_EW_MIN) B200_CH2(B200_EW_POW) B200_CH2(B200_EW_GT) B200_CH2(B200_EW_GE) B200_CH2(B200_EW_LT)
    B200_CH2(B200_EW_EQ)
#undef B200_CH2
    default:
#pragma unroll
      for (int v = 0; v < V; ++v) r[v] = apply1(op, x[v]);
  }
}

__global__ void __launch_bounds__(THREADS) ew_chain8_kernel(const __grid_constant__ EwParams P) {
  const int64_t ng = (P.n + V - 1) / V;
  const int nout = P.p.n_out, nch = P.nchain;
  for (int64_t q = blockIdx.x * (int64_t)THREADS + threadIdx.x; q < ng; q += (int64_t)gridDim.x * THREADS) {
    const int64_t base = q * V;
    const bool full = base + V <= P.n;
    float t[V];
#pragma unroll
    for (int v = 0; v < V; ++v) t[v] = 0.f;
    for (int k = 0; k < nch; ++k) {
      float xy[2][V];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int src = P.csrc[k][i];
        if (src >= 0) {
          loadv<V>(P, src, base, full, xy[i]);
        } else if (src == -1) {
          const float c = P.cimm[k][i];
#pragma unroll
          for (int v = 0; v < V; ++v) xy[i][v] = c;
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) xy[i][v] = t[v];
        }
      }
      apply_rt<0>(P.cop[k], xy[0], xy[1], t);
    }
    for (int o = 0; o < nout; ++o) storev<V>(P, o, base, full, t);
  }
}

// sum of inputs as a left fold, ((in[o0] + in[o1]) + in[o2]) + ..., stored to every output:
// all inputs of a group are loaded before the first addition
__global__ void __launch_bounds__(THREADS) ew_sum8_kernel(const __grid_constant__ EwParams P) {
  const int64_t ng = (P.n + V - 1) / V;
  const int nout = P.p.n_out, nsum = P.nsum;
  for (int64_t q = blockIdx.x * (int64_t)THREADS + threadIdx.x; q < ng; q += (int64_t)gridDim.x * THREADS) {
    const int64_t base = q * V;
    const bool full = base + V <= P.n;
    float x[B200_EW_MAX_IN][V];
#pragma unroll
    for (int k = 0; k < B200_EW_MAX_IN; ++k)
      if (k < nsum) loadv<V>(P, P.sumord[k], base, full, x[k]);
    float r[V];
#pragma unroll
    for (int v = 0; v < V; ++v) r[v] = x[0][v];
#pragma unroll
    for (int k = 1; k < B200_EW_MAX_IN; ++k)
      if (k < nsum) {
#pragma unroll
        for (int v = 0; v < V; ++v) r[v] = r[v] + x[k][v];
      }
    for (int o = 0; o < nout; ++o) storev<V>(P, o, base, full, r);
  }
}

// Recognise a program that adds its loaded inputs one after another (a left fold of ADD
// instructions) and stores only the final sum.
static bool classify_sum(EwParams& P) {
  const b200_ew_program& p = P.p;
  int reg_in[B200_EW_MAX_REG];
  for (int i = 0; i < B200_EW_MAX_REG; ++i) reg_in[i] = -1;
  int acc = -1, n = 0, stores = 0;
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins& I = p.ins[i];
    if (I.op == B200_EW_LOAD) {
      if (I.dst >= B200_EW_MAX_REG || I.dst == acc) return false;
      reg_in[I.dst] = I.a;
    } else if (I.op == B200_EW_ADD) {
      if (I.a >= B200_EW_MAX_REG || I.b >= B200_EW_MAX_REG || I.dst >= B200_EW_MAX_REG || stores) return false;
      if (acc < 0) {
        if (reg_in[I.a] < 0 || reg_in[I.b] < 0) return false;
        P.sumord[0] = reg_in[I.a];
        P.sumord[1] = reg_in[I.b];
        n = 2;
      } else {
        int other;
        if (I.a == acc && I.b != acc) other = I.b;
        else if (I.b == acc && I.a != acc) other = I.a;
        else return false;
        if (reg_in[other] < 0 || n >= B200_EW_MAX_IN) return false;
        P.sumord[n++] = reg_in[other];
      }
      acc = I.dst;
      reg_in[acc] = -1;
    } else if (I.op == B200_EW_STORE) {
      if (acc < 0 || I.a != acc) return false;
      ++stores;
    } else {
      return false;
    }
  }
  if (acc < 0 || stores == 0) return false;
  P.nsum = n;
  P.kind = 4;
  return true;
}

// Recognise a chain: every op reads inputs, immediates or the result of the op just
// before it (which nothing else reads), and the stores take the last op's result.
static bool classify_chain(EwParams& P) {
  const b200_ew_program& p = P.p;
  int kind_of[B200_EW_MAX_REG];  // >= 0 input, -1 immediate, -2 the current result, -3 dead / unset
  float imm_of[B200_EW_MAX_REG];
  for (int i = 0; i < B200_EW_MAX_REG; ++i) kind_of[i] = -3, imm_of[i] = 0.f;
  int n = 0, treg = -1;
  bool stored = false;
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins& I = p.ins[i];
    if (stored && I.op != B200_EW_STORE) return false;  // stores come last
    if (I.op == B200_EW_LOAD) {
      if ((int)I.dst == treg) return false;
      kind_of[I.dst] = I.a;
    } else if (I.op == B200_EW_IMM) {
      if ((int)I.dst == treg) return false;
      kind_of[I.dst] = -1;
      imm_of[I.dst] = I.imm;
    } else if (I.op == B200_EW_STORE) {
      if (treg < 0 || (int)I.a != treg) return false;
      stored = true;
    } else if (I.op == B200_EW_WHERE || I.op == B200_EW_FMA) {
      return false;
    } else {
      if (n >= 4) return false;
      const bool unary = !(I.op == B200_EW_ADD || I.op == B200_EW_SUB || I.op == B200_EW_MUL || I.op == B200_EW_DIV ||
                           I.op == B200_EW_MAX || I.op == B200_EW_MIN || I.op == B200_EW_POW || I.op == B200_EW_GT ||
                           I.op == B200_EW_GE || I.op == B200_EW_LT || I.op == B200_EW_EQ);
      const int regs[2] = {I.a, unary ? I.a : I.b};
      int uses_t = 0;
      for (int k = 0; k < 2; ++k) {
        const int kd = kind_of[regs[k]];
        if (kd == -3) return false;
        if (kd == -2) {
          if (regs[k] != treg) return false;
          ++uses_t;
        }
        P.csrc[n][k] = kd;
        P.cimm[n][k] = imm_of[regs[k]];
      }
      if (n > 0 && uses_t == 0) return false;  // the previous result would be lost
      if (treg >= 0) kind_of[treg] = -3;      // read once: the chain moves on
      P.cop[n++] = I.op;
      treg = I.dst;
      kind_of[treg] = -2;
    }
  }
  if (n == 0 || treg < 0) return false;
  P.nchain = n;
  P.kind = 5;
  return true;
}

// Recognise a program that is LOADs, one op, and STOREs of that op's result only (or
// LOADs and STOREs of a single loaded register: a copy / cast).
static void classify(EwParams& P) {
  const b200_ew_program& p = P.p;
  P.kind = 0;
  int reg_in[B200_EW_MAX_REG];
  for (int i = 0; i < B200_EW_MAX_REG; ++i) reg_in[i] = -1;
  int n_op = 0, op = -1, a_in = -1, b_in = -1, rdst = -1, copy_in = -1;
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins& I = p.ins[i];
    if (I.op == B200_EW_LOAD) {
      reg_in[I.dst] = I.a;
      if (I.dst == rdst) return;  // the op's result is overwritten
    } else if (I.op == B200_EW_STORE) {
      if (n_op == 0) {
        const int src = reg_in[I.a];
        if (src < 0 || (copy_in >= 0 && copy_in != src)) return;
        copy_in = src;
      } else if (I.a != rdst) {
        return;
      }
    } else {
      if (++n_op > 1 || copy_in >= 0) return;
      op = I.op;
      a_in = reg_in[I.a];
      b_in = reg_in[I.b];
      rdst = I.dst;
    }
  }
  if (n_op == 0) {
    if (copy_in < 0) return;
    P.kind = 1;
    P.sop = B200_EW_MOV;
    P.sa = copy_in;
    return;
  }
  const bool binary = op == B200_EW_ADD || op == B200_EW_SUB || op == B200_EW_MUL || op == B200_EW_DIV ||
                      op == B200_EW_MAX || op == B200_EW_MIN || op == B200_EW_GT || op == B200_EW_GE || op == B200_EW_LT ||
                      op == B200_EW_EQ;
  const bool unary = op == B200_EW_NEG || op == B200_EW_EXP || op == B200_EW_LOG || op == B200_EW_TANH ||
                     op == B200_EW_SQRT || op == B200_EW_RELU || op == B200_EW_GELU || op == B200_EW_ABS ||
                     op == B200_EW_SIGMOID || op == B200_EW_ERF || op == B200_EW_RECIP || op == B200_EW_MOV;
  if (binary && a_in >= 0 && b_in >= 0) {
    P.kind = 3;
    P.sop = op;
    P.sa = a_in;
    P.sb = b_in;
  } else if (unary && a_in >= 0) {
    P.kind = 2;
    P.sop = op;
    P.sa = a_in;
  }
}

}  // namespace ewf

int ew_flat_launch(EwParams& P, cudaStream_t s) {
  using namespace ewf;
  const b200_ew_program& p = P.p;
  classify(P);
  const int64_t groups = ceil_div(P.n, (int64_t)V);
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(groups, THREADS), (int64_t)num_sms() * 8));
  const unsigned gblocks =
      (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(ceil_div(P.n, (int64_t)VG), THREADS), (int64_t)num_sms() * 8));
  if (P.kind == 1 || P.kind == 2) {
    ew_un8_kernel<<<blocks, THREADS, 0, s>>>(P);
    return check_launch("ew_run(unary)");
  }
  if (P.kind == 0) classify_sum(P);
  if (P.kind == 0) classify_chain(P);
  if (P.kind == 5) {
    ew_chain8_kernel<<<blocks, THREADS, 0, s>>>(P);
    return check_launch("ew_run(chain)");
  }
  if (P.kind == 4) {
    ew_sum8_kernel<<<blocks, THREADS, 0, s>>>(P);
    return check_launch("ew_run(sum)");
  }
  if (P.kind == 3) {
    switch (P.sop) {
#define B200_LB(OPC) \
  case OPC: ew_bin8_kernel<OPC><<<blocks, THREADS, 0, s>>>(P); break;
      B200_LB(B200_EW_ADD) B200_LB(B200_EW_SUB) B200_LB(B200_EW_MUL) B200_LB(B200_EW_DIV) B200_LB(B200_EW_MAX)
      B200_LB(B200_EW_MIN) B200_LB(B200_EW_GT) B200_LB(B200_EW_GE) B200_LB(B200_EW_LT) B200_LB(B200_EW_EQ)
#undef B200_LB
      default: break;
    }
    return check_launch("ew_run(binary)");
  }
  int nreg = 0;
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins& I = p.ins[i];
    int hi = 0;
    if (I.op == B200_EW_LOAD || I.op == B200_EW_IMM) hi = I.dst;
    else if (I.op == B200_EW_STORE) hi = I.a;
    else hi = std::max<int>(std::max<int>(I.dst, I.a), std::max<int>(I.b, I.c));
    nreg = std::max(nreg, hi + 1);
  }
#define B200_PROG(NR)                                                                      \
  do {                                                                                     \
    if (p.n_in <= 2) ew_prog_kernel<NR, 2><<<gblocks, THREADS, 0, s>>>(P);                 \
    else if (p.n_in <= 4) ew_prog_kernel<NR, 4><<<gblocks, THREADS, 0, s>>>(P);            \
    else ew_prog_kernel<NR, B200_EW_MAX_IN><<<gblocks, THREADS, 0, s>>>(P);                \
  } while (0)
  if (nreg <= 4) B200_PROG(4);
  else if (nreg <= 8) B200_PROG(8);
  else B200_PROG(16);
#undef B200_PROG
  return check_launch("ew_run(program)");
}

}  // namespace b200

// Fused elementwise programs (subsystem 1).
//
// One launch evaluates a whole chain of elementwise graph nodes: every element of the
// output index space loads its inputs once (broadcast by zero strides), runs the
// register program in fp32 and stores the chain's live outputs once. HBM traffic is
// one read per distinct input and one write per output, however long the chain.
//
// Two paths:
//  * flat: every input is either dense over the output (strides == row-major strides)
//    or a scalar (all strides 0). Each thread handles 4 consecutive elements with
//    128-bit loads/stores for fp32 operands (16-byte aligned bases).
//  * strided: arbitrary per-input strides over up to 6 dims (broadcast, transposed
//    views); offsets come from one index decomposition per element.
#include "ew_common.cuh"

namespace b200 {

template <int V>
__device__ __forceinline__ void ew_exec(const b200_ew_program& p, float (&r)[B200_EW_MAX_REG][V],
                                        const float (&ld)[B200_EW_MAX_IN][V], float (&st)[B200_EW_MAX_OUT][V]) {
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins I = p.ins[i];
    const int d = I.dst, a = I.a, b = I.b, c = I.c;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float x = r[a][v], y = r[b][v], res;
      switch (I.op) {
        case B200_EW_LOAD: res = ld[a][v]; break;
        case B200_EW_STORE: st[d][v] = x; continue;
        case B200_EW_IMM: res = I.imm; break;
        case B200_EW_ADD: res = x + y; break;
        case B200_EW_SUB: res = x - y; break;
        case B200_EW_MUL: res = x * y; break;
        case B200_EW_DIV: res = x / y; break;
        case B200_EW_NEG: res = -x; break;
        case B200_EW_EXP: res = expf(x); break;
        case B200_EW_LOG: res = logf(x); break;
        case B200_EW_TANH: res = tanhf(x); break;
        case B200_EW_SQRT: res = sqrtf(x); break;
        case B200_EW_POW: res = powf(x, y); break;
        case B200_EW_MAX: res = fmaxf(x, y); break;
        case B200_EW_MIN: res = fminf(x, y); break;
        case B200_EW_GT: res = (x > y) ? 1.f : 0.f; break;
        case B200_EW_GE: res = (x >= y) ? 1.f : 0.f; break;
        case B200_EW_LT: res = (x < y) ? 1.f : 0.f; break;
        case B200_EW_EQ: res = (x == y) ? 1.f : 0.f; break;
        case B200_EW_WHERE: res = (x != 0.f) ? y : r[c][v]; break;
        case B200_EW_RELU: res = x > 0.f ? x : 0.f; break;
        case B200_EW_GELU: res = gelu_tanh(x); break;
        case B200_EW_ABS: res = fabsf(x); break;
        case B200_EW_SIGMOID: res = 1.f / (1.f + expf(-x)); break;
        case B200_EW_ERF: res = erff(x); break;
        case B200_EW_MOV: res = x; break;
        case B200_EW_RECIP: res = 1.f / x; break;
        case B200_EW_FMA: res = fmaf(x, y, r[c][v]); break;
        default: res = 0.f; break;
      }
      r[d][v] = res;
    }
  }
}

// strided path: 1 element per thread-iteration
__global__ void __launch_bounds__(256) ew_strided_kernel(const __grid_constant__ EwParams P) {
  const b200_ew_program& p = P.p;
  float r[B200_EW_MAX_REG][1];
  float ld[B200_EW_MAX_IN][1];
  float st[B200_EW_MAX_OUT][1];
#pragma unroll
  for (int i = 0; i < B200_EW_MAX_REG; ++i) r[i][0] = 0.f;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < P.n; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t off[B200_EW_MAX_IN];
#pragma unroll
    for (int j = 0; j < B200_EW_MAX_IN; ++j) off[j] = 0;
    int64_t rem = e;
    for (int d = p.ndim - 1; d >= 0; --d) {
      const int64_t sz = p.shape[d];
      const int64_t id = rem % sz;
      rem /= sz;
#pragma unroll
      for (int j = 0; j < B200_EW_MAX_IN; ++j)
        if (j < p.n_in) off[j] += id * p.in_strides[j][d];
    }
    for (int j = 0; j < p.n_in; ++j) ld[j][0] = load_as_f32(P.in[j], off[j], p.in_dtype[j]);
    ew_exec<1>(p, r, ld, st);
    for (int o = 0; o < p.n_out; ++o) store_from_f32(P.out[o], e, p.out_dtype[o], st[o][0]);
  }
}

// strided path with 32-bit index arithmetic (fast division per dim)
__global__ void __launch_bounds__(256) ew_strided32_kernel(const __grid_constant__ EwParams P) {
  const b200_ew_program& p = P.p;
  float r[B200_EW_MAX_REG][1];
  float ld[B200_EW_MAX_IN][1];
  float st[B200_EW_MAX_OUT][1];
#pragma unroll
  for (int i = 0; i < B200_EW_MAX_REG; ++i) r[i][0] = 0.f;
  const uint32_t n = (uint32_t)P.n;
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    int32_t off[B200_EW_MAX_IN];
#pragma unroll
    for (int j = 0; j < B200_EW_MAX_IN; ++j) off[j] = 0;
    uint32_t rem = e;
    for (int d = p.ndim - 1; d >= 0; --d) {
      const uint32_t q = fast_div(rem, P.dmul[d], P.dshr[d]);
      const int32_t id = (int32_t)(rem - q * P.dsz[d]);
      rem = q;
#pragma unroll
      for (int j = 0; j < B200_EW_MAX_IN; ++j)
        if (j < p.n_in) off[j] += id * P.st32[j][d];
    }
    for (int j = 0; j < p.n_in; ++j) ld[j][0] = load_as_f32(P.in[j], off[j], p.in_dtype[j]);
    ew_exec<1>(p, r, ld, st);
    for (int o = 0; o < p.n_out; ++o) store_from_f32(P.out[o], e, p.out_dtype[o], st[o][0]);
  }
}

// Merges adjacent dims of the index space wherever every input's strides allow it
// (stride[d] == stride[d + 1] * shape[d + 1], broadcast dims included) and drops size-1
// dims, so that e.g. a [N, C, 1, 1] operand broadcast over [N, C, H, W] becomes one value
// per row of H * W elements. The output is dense, so any merge keeps its addressing.
static void coalesce_dims(b200_ew_program& q) {
  int64_t sh[B200_EW_MAX_DIM], st[B200_EW_MAX_IN][B200_EW_MAX_DIM];
  int nd = 0;
  for (int d = 0; d < q.ndim; ++d) {
    if (q.shape[d] == 1) continue;
    if (nd > 0) {
      bool ok = true;
      for (int j = 0; j < q.n_in && ok; ++j) ok = st[j][nd - 1] == q.in_strides[j][d] * q.shape[d];
      if (ok) {
        sh[nd - 1] *= q.shape[d];
        for (int j = 0; j < q.n_in; ++j) st[j][nd - 1] = q.in_strides[j][d];
        continue;
      }
    }
    sh[nd] = q.shape[d];
    for (int j = 0; j < q.n_in; ++j) st[j][nd] = q.in_strides[j][d];
    ++nd;
  }
  if (nd == 0) {  // every dim is 1: one element
    sh[0] = 1;
    for (int j = 0; j < q.n_in; ++j) st[j][0] = 0;
    nd = q.ndim > 0 ? 1 : 0;
  }
  q.ndim = nd;
  for (int d = 0; d < nd; ++d) {
    q.shape[d] = sh[d];
    for (int j = 0; j < q.n_in; ++j) q.in_strides[j][d] = st[j][d];
  }
}

static bool dtype_ok(int dt) { return dt == B200_F32 || dt == B200_BF16 || dt == B200_I64 || dt == B200_BOOL || dt == B200_I32; }

}  // namespace b200

extern "C" int b200_ew_run(const b200_ew_program* prog, const void* const* inputs, void* const* outputs, void* stream) {
  using namespace b200;
  B200_REQUIRE(prog != nullptr, "ew_run: null program");
  const b200_ew_program& p0 = *prog;
  B200_REQUIRE(p0.ndim >= 0 && p0.ndim <= B200_EW_MAX_DIM, "ew_run: ndim %d out of range", p0.ndim);
  B200_REQUIRE(p0.n_in >= 0 && p0.n_in <= B200_EW_MAX_IN, "ew_run: n_in %d out of range", p0.n_in);
  B200_REQUIRE(p0.n_out >= 1 && p0.n_out <= B200_EW_MAX_OUT, "ew_run: n_out %d out of range", p0.n_out);
  B200_REQUIRE(p0.n_ins >= 1 && p0.n_ins <= B200_EW_MAX_INS, "ew_run: n_ins %d out of range", p0.n_ins);
  int64_t n = 1;
  for (int d = 0; d < p0.ndim; ++d) {
    B200_REQUIRE(p0.shape[d] >= 0, "ew_run: negative dim");
    n *= p0.shape[d];
  }
  EwParams P;
  P.p = p0;
  P.n = n;
  if (n > 0) coalesce_dims(P.p);
  const b200_ew_program& p = P.p;
  for (int j = 0; j < p.n_in; ++j) {
    B200_REQUIRE(inputs && inputs[j], "ew_run: null input %d", j);
    if (!dtype_ok(p.in_dtype[j])) {
      set_error("ew_run: input %d dtype %d", j, p.in_dtype[j]);
      return B200_ERR_DTYPE;
    }
    P.in[j] = inputs[j];
  }
  for (int j = p.n_in; j < B200_EW_MAX_IN; ++j) P.in[j] = nullptr;
  for (int o = 0; o < p.n_out; ++o) {
    B200_REQUIRE(outputs && outputs[o], "ew_run: null output %d", o);
    if (!dtype_ok(p.out_dtype[o])) {
      set_error("ew_run: output %d dtype %d", o, p.out_dtype[o]);
      return B200_ERR_DTYPE;
    }
    P.out[o] = outputs[o];
  }
  for (int o = p.n_out; o < B200_EW_MAX_OUT; ++o) P.out[o] = nullptr;
  for (int i = 0; i < p.n_ins; ++i) {
    const b200_ew_ins& I = p.ins[i];
    B200_REQUIRE(I.op <= B200_EW_FMA, "ew_run: bad opcode %d at %d", I.op, i);
    B200_REQUIRE(I.a < B200_EW_MAX_REG && I.b < B200_EW_MAX_REG && I.c < B200_EW_MAX_REG, "ew_run: bad register at %d", i);
    if (I.op == B200_EW_LOAD) B200_REQUIRE(I.a < p.n_in && I.dst < B200_EW_MAX_REG, "ew_run: bad load at %d", i);
    else if (I.op == B200_EW_STORE) B200_REQUIRE(I.dst < p.n_out, "ew_run: bad store at %d", i);
    else B200_REQUIRE(I.dst < B200_EW_MAX_REG, "ew_run: bad dst at %d", i);
  }
  if (n == 0) return B200_OK;

  // flat path when every input is dense over the output, a scalar, a vector along the
  // last dim or one value per row of the last dim
  bool flat = true;
  int64_t dense[B200_EW_MAX_DIM];
  {
    int64_t s = 1;
    for (int d = p.ndim - 1; d >= 0; --d) {
      dense[d] = s;
      s *= p.shape[d];
    }
  }
  const int64_t lastdim = p.ndim > 0 ? p.shape[p.ndim - 1] : 1;
  const bool small = n < ((int64_t)1 << 31) && lastdim >= 1;
  P.lastdim = lastdim;
  fastdiv_params((uint32_t)std::min<int64_t>(std::max<int64_t>(lastdim, 1), 0x7fffffff), P.ld_mul, P.ld_shr);
  P.ld8 = (lastdim % 8 == 0) ? 1 : 0;
  auto al = [](const void* q, int bytes) { return (reinterpret_cast<uintptr_t>(q) % bytes) == 0; };
  for (int j = 0; j < p.n_in && flat; ++j) {
    bool all0 = true, isdense = true, isvec = p.ndim > 0, isrow = p.ndim > 0 && lastdim > 1;
    for (int d = 0; d < p.ndim; ++d) {
      if (p.shape[d] == 1) continue;
      const int64_t st = p.in_strides[j][d];
      if (st != 0) all0 = false;
      if (st != dense[d]) isdense = false;
      if (d == p.ndim - 1 ? st != 1 : st != 0) isvec = false;
      if (d == p.ndim - 1 ? st != 0 : st != dense[d] / lastdim) isrow = false;
    }
    const int dt = p.in_dtype[j];
    P.vin[j] = ((dt == B200_F32 || dt == B200_BF16) && al(inputs[j], 16)) ? 1 : 0;
    if (all0) P.mode[j] = 1;
    else if (isdense) P.mode[j] = 0;
    else if (isvec && small) P.mode[j] = 2;
    else if (isrow && small) P.mode[j] = 3;
    else flat = false;
  }
  for (int o = 0; o < p.n_out; ++o) {
    const int dt = p.out_dtype[o];
    P.vout[o] = ((dt == B200_F32 || dt == B200_BF16) && al(outputs[o], 16)) || (dt == B200_BOOL && al(outputs[o], 8));
  }
  if (flat) return ew_flat_launch(P, as_stream(stream));

  const int threads = 256;
  const int64_t sms = num_sms();
  {
    // 32-bit index path when every offset fits
    bool fits = n < ((int64_t)1 << 31);
    for (int j = 0; j < p.n_in && fits; ++j) {
      int64_t ext = 0;
      for (int d = 0; d < p.ndim; ++d) ext += (p.shape[d] - 1) * (p.in_strides[j][d] < 0 ? -p.in_strides[j][d] : p.in_strides[j][d]);
      if (ext >= ((int64_t)1 << 31)) fits = false;
    }
    int64_t blocks = std::min<int64_t>(ceil_div(n, threads), sms * 8);
    if (fits) {
      for (int d = 0; d < p.ndim; ++d) {
        P.dsz[d] = (uint32_t)p.shape[d];
        fastdiv_params(P.dsz[d], P.dmul[d], P.dshr[d]);
        for (int j = 0; j < p.n_in; ++j) P.st32[j][d] = (int32_t)p.in_strides[j][d];
      }
      ew_strided32_kernel<<<(unsigned)blocks, threads, 0, as_stream(stream)>>>(P);
    } else {
      ew_strided_kernel<<<(unsigned)blocks, threads, 0, as_stream(stream)>>>(P);
    }
  }
  return check_launch("ew_run");
}

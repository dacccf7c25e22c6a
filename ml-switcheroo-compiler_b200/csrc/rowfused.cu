// Whole-row fused forward + backward of the chain
//     p = x * a + b ;  g = gelu_tanh(p) ;  n = LayerNorm(g; gamma, beta, eps) ;
//     y = softmax(n) ;  am = argmax(y)
// and of its VJP for an upstream gradient c on y:
//     dn = y * (c - sum(c*y)) ;  dg = LayerNormInputGrad(dn, g, gamma) ;
//     dp = dg * gelu_tanh'(p) ;  dx = dp * a ;  da = sum_rows(dp * x) ;  db = sum_rows(dp)
//     (optional) dgamma = sum_rows(dn * g_hat), dbeta = sum_rows(dn)
//
// These are the reference ops Multiply/Add (numpy/eager/math_binary.py:9-51),
// Gelu (eager/core_math_ops/math_nn.py:184-199), LayerNorm (numpy/eager/nn_ops.py:219-241),
// Softmax (numpy/eager/math_advanced/math_signal.py:450-467), Argmax
// (numpy/eager/math_reductions.py:129-140) and the VJP graph the AD emits for them
// (Softmax rule, LayerNormInputGrad nn_ops.py:244, tanh-GELU derivative, BroadcastReduce
// math_reduction.py:192 for the column vectors).
//
// One CTA per row at a time (persistent over rows); the row lives in registers, so HBM
// sees exactly one read of x and c and one write of y and dx per element. Column sums
// (da, db, dgamma, dbeta) are accumulated per CTA in registers, written once per CTA to a
// workspace, and reduced over CTAs by a second kernel in a fixed order (deterministic).
#include <math.h>

#include "common.cuh"

namespace b200 {
namespace rf {

constexpr float K_GELU = 0.7978845608028654f;  // sqrt(2/pi)
constexpr float C_GELU = 0.044715f;
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  const float *x, *a, *b, *gamma, *beta, *c;
  float *y, *dx;
  int64_t* am;
  float* part;  // [4][grid][cols] partial column sums: da, db, dgamma, dbeta
  int64_t rows, cols;
  float eps;
  int want_gb;    // accumulate dgamma / dbeta partials
  int aligned16;  // every row and column-vector pointer is 16-byte aligned (vector loads / cp.async allowed)
};

// ---- packed fp32x2 arithmetic (sm_100a): two lanes of a row per instruction -------
struct F2 {
  unsigned long long v;
};
__device__ __forceinline__ F2 pk(float a, float b) {
  F2 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r.v) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk(F2 r, float& a, float& b) { asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(r.v)); }
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) {
  F2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
__device__ __forceinline__ F2 mul2(F2 a, F2 b) {
  F2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 add2(F2 a, F2 b) {
  F2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 sub2(F2 a, F2 b) {
  F2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ F2 sp(float a) { return pk(a, a); }
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// cp.async (Ampere-style, per thread) into this thread's own shared-memory slot; the
// issuing thread is also the only reader, so completion needs no block barrier.
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async4(void* sdst, const void* gsrc, bool valid) {
  // src-size 0 zero-fills the destination without reading global memory
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)), "l"(gsrc),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// lanes 0-15 return sum(a), lanes 16-31 sum(b) over the warp (one shuffle tree for both)
__device__ __forceinline__ float warp_pair_sum(float a, float b, int lane) {
  const bool hi = lane >= 16;
  float keep = hi ? b : a;
  const float send = hi ? a : b;
  keep += __shfl_xor_sync(0xffffffffu, send, 16);
  keep += __shfl_xor_sync(0xffffffffu, keep, 8);
  keep += __shfl_xor_sync(0xffffffffu, keep, 4);
  keep += __shfl_xor_sync(0xffffffffu, keep, 2);
  keep += __shfl_xor_sync(0xffffffffu, keep, 1);
  return keep;
}
// order-preserving map of a float onto an unsigned key and back
__device__ __forceinline__ uint32_t ord_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_value(uint32_t o) { return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o); }

// Block reductions of one barrier each: every warp shuffles its partials down, lane 0 /
// lane 16 post them to the site's shared region, and after the barrier every warp combines
// the NW warp partials itself (same order in every warp, so every thread sees the same
// bits). A site is written again only in the next row, after later barriers every reader
// of its previous contents has passed.
template <int NW>
__device__ __forceinline__ float2 block_finish(const float* red, int lane) {
  if (NW > 16) {
    const float ra = lane < NW ? red[lane] : 0.f, rb = lane < NW ? red[32 + lane] : 0.f;
    const float t = warp_pair_sum(ra, rb, lane);
    return make_float2(__shfl_sync(0xffffffffu, t, 0), __shfl_sync(0xffffffffu, t, 16));
  }
  float t = (lane & 15) < NW ? red[(lane >> 4) * 32 + (lane & 15)] : 0.f;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return make_float2(__shfl_sync(0xffffffffu, t, 0), __shfl_sync(0xffffffffu, t, 16));
}
template <int NW>
__device__ __forceinline__ float2 block_pair_sum(float a, float b, float* red, int lane, int w) {
  const float v = warp_pair_sum(a, b, lane);
  if ((lane & 15) == 0) red[(lane >> 4) * 32 + w] = v;
  __syncthreads();
  return block_finish<NW>(red, lane);
}
// the same plus the maximum of an unsigned key (red[64 .. 64 + NW))
template <int NW>
__device__ __forceinline__ float2 block_pair_sum_max(float a, float b, uint32_t& m, float* red, int lane, int w) {
  const float v = warp_pair_sum(a, b, lane);
  const uint32_t wm = __reduce_max_sync(0xffffffffu, m);
  uint32_t* ured = reinterpret_cast<uint32_t*>(red);
  if ((lane & 15) == 0) red[(lane >> 4) * 32 + w] = v;
  if (lane == 0) ured[64 + w] = wm;
  __syncthreads();
  m = __reduce_max_sync(0xffffffffu, lane < NW ? ured[64 + lane] : 0u);
  return block_finish<NW>(red, lane);
}
template <int NW>
__device__ __forceinline__ uint32_t block_max_key(uint32_t m, float* red, int lane, int w) {
  uint32_t* ured = reinterpret_cast<uint32_t*>(red);
  const uint32_t wm = __reduce_max_sync(0xffffffffu, m);
  if (lane == 0) ured[64 + w] = wm;
  __syncthreads();
  return __reduce_max_sync(0xffffffffu, lane < NW ? ured[64 + lane] : 0u);
}

// V values of a column vector from column c0 on: past the row end 0, a null vector `if_null`
template <int V>
__device__ __forceinline__ void ldg_vals(float (&r)[V], const float* __restrict__ p, int c0, int64_t C, bool vec, float if_null) {
  if (p && vec) {
#pragma unroll
    for (int i = 0; i < V; i += 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p + c0 + i));
      r[i] = t.x; r[i + 1] = t.y; r[i + 2] = t.z; r[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = c0 + i < C ? (p ? p[c0 + i] : if_null) : 0.f;
  }
}

// This thread's V columns of the column vectors, from column c0 on: a and b as given,
// gamma log2e and (beta - shift) log2e for the softmax exponent; columns past the row end
// get a = b = 0, gamma = 0, beta' = -inf. Returns whether the fixed softmax shift applies
// (the same answer in every thread: each warp reduces the same partials in the same order).
// Contains one __syncthreads.
template <int NW, int V, bool RAGGED>
__device__ __forceinline__ bool load_columns(const Params& P, int c0, bool vec, float (&av)[V], float (&bv)[V], float (&glv)[V],
                                             float (&blv)[V], float (*sh)[32], int lane, int wid) {
  const int64_t C = P.cols;
  float gv[V], ev[V];
  ldg_vals<V>(av, P.a, c0, C, vec, 0.f);
  ldg_vals<V>(bv, P.b, c0, C, vec, 0.f);
  ldg_vals<V>(gv, P.gamma, c0, C, vec, 1.f);
  ldg_vals<V>(ev, P.beta, c0, C, vec, 0.f);
  // Softmax shift: for n = gamma * x_hat + beta with every gamma >= 0, each row max lies in
  // [min beta, max gamma * sqrt(C) + max beta] (|x_hat| <= sqrt(C), max x_hat >= 0). When
  // that interval is at most 80 wide, exp(n - S) with S its top never overflows and the
  // largest term never underflows, so the per-row max reduction is not needed.
  float gmin = INFINITY, gmx = -INFINITY, bmn = INFINITY, bmx = -INFINITY;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if (!RAGGED || c0 + i < C) {
      gmin = fminf(gmin, gv[i]); gmx = fmaxf(gmx, gv[i]);
      bmn = fminf(bmn, ev[i]); bmx = fmaxf(bmx, ev[i]);
    }
  }
  gmin = -warp_max(-gmin);
  gmx = warp_max(gmx);
  bmn = -warp_max(-bmn);
  bmx = warp_max(bmx);
  if (lane == 0) {
    sh[0][wid] = gmin; sh[1][wid] = gmx; sh[2][wid] = bmn; sh[3][wid] = bmx;
  }
  __syncthreads();
  const int l = lane < NW ? lane : 0;
  gmin = -warp_max(-sh[0][l]);
  gmx = warp_max(sh[1][l]);
  bmn = -warp_max(-sh[2][l]);
  bmx = warp_max(sh[3][l]);
  const float shiftS = gmx * sqrtf((float)C) + bmx;
  const bool use_shift = gmin >= 0.f && (shiftS - bmn) <= 80.f && isfinite(shiftS);
  const float sub = use_shift ? shiftS : 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    glv[i] = gv[i] * LOG2E;
    blv[i] = (!RAGGED || c0 + i < C) ? (ev[i] - sub) * LOG2E : -INFINITY;
  }
  return use_shift;
}

// gamma log2e and beta' log2e are read in two of the four passes only, so up to 8 columns
// per thread they wait in the thread's shared-memory slot (freeing registers for the rest)
constexpr bool gl_in_smem(int V) { return V <= 8; }

// T threads, V consecutive columns per thread (cols <= T*V), V/2 packed pairs, one row per
// CTA at a time. Registers hold this thread's slice of the column vectors a, b (and
// gamma log2e, (beta - shift) log2e above 8 columns per thread; loaded once per CTA), sigma(2u) of the current row,
// one working row array w and the column accumulators. x and c of the current and the
// next row sit in this thread's own shared-memory slot, prefetched with cp.async one row
// ahead (double-buffered). Per row three block reductions of one barrier each:
//   R1  sum g, sum g^2                       (LayerNorm statistics)
//   R2  sum e, sum c e, max e                (e = exp(n - shift); sum c y = sum(c e) / sum e)
//   R3  sum dn gamma, sum dn gamma g_hat     (LayerNormInputGrad)
// plus the row max of n before R2 when the fixed softmax shift does not apply.
// gelu_tanh(p) = 0.5 p (1 + tanh u) = p sigma(2u), u = k (p + c p^3). Columns past the
// row end have a = b = 0, gamma = 0, beta' = -inf and zero-filled x, c, so they add exact
// zeros to every row sum and never win a maximum; they are only kept out of the stores.
// argmax(y): y is a monotone function of e, so only threads whose largest e rounds to the
// row's largest y search their columns, and post the first match with a shared-memory
// atomicMin (an order-independent minimum).
template <int T, int V, bool GB, bool RAGGED>
__global__ void __launch_bounds__(T, (V == 4 ? 1024 : 512) / T > 0 ? (V == 4 ? 1024 : 512) / T : 1) rowfused_kernel(const __grid_constant__ Params P) {
  constexpr int NW = T / 32;
  constexpr int H = V / 2;
  __shared__ __align__(16) float sh[4][32];    // set-up reductions
  __shared__ __align__(16) float red[4][96];   // per-row reduction sites
  __shared__ int s_am;
  // [2 stages][x, c][T][V], then [gamma log2e, beta' log2e][T][V] when GLSM (a warp's slices are contiguous)
  extern __shared__ __align__(16) float sm[];
  constexpr bool GLSM = gl_in_smem(V);
  const int64_t C = P.cols;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c0 = threadIdx.x * V;
  const bool full = c0 + V <= C;
  const bool vec = full && ((C & 3) == 0) && P.aligned16;
  const bool any = c0 < C;
  const float invC = 1.f / (float)C;
  const int64_t G = gridDim.x;

  F2 a[H], b[H], glr[GLSM ? 1 : H], blr[GLSM ? 1 : H];
  float* const sgl = sm + ((size_t)4 * T + threadIdx.x) * V;  // this thread's gamma log2e (GLSM)
  float* const sbl = sgl + (size_t)T * V;                    // and beta' log2e
  if (threadIdx.x == 0) s_am = 0x7fffffff;
  bool use_shift;
  {
    float av[V], bv[V], glv[V], blv[V];
    use_shift = load_columns<NW, V, RAGGED>(P, c0, vec, av, bv, glv, blv, sh, lane, wid);
#pragma unroll
    for (int i = 0; i < H; ++i) {
      a[i] = pk(av[2 * i], av[2 * i + 1]);
      b[i] = pk(bv[2 * i], bv[2 * i + 1]);
      if (GLSM) {
        sgl[2 * i] = glv[2 * i]; sgl[2 * i + 1] = glv[2 * i + 1];
        sbl[2 * i] = blv[2 * i]; sbl[2 * i + 1] = blv[2 * i + 1];
      } else {
        glr[GLSM ? 0 : i] = pk(glv[2 * i], glv[2 * i + 1]);
        blr[GLSM ? 0 : i] = pk(blv[2 * i], blv[2 * i + 1]);
      }
    }
  }
  constexpr float CS0 = -2.f * LOG2E * K_GELU;  // sigma(2u) = 1 / (1 + 2^(p (CS0 + CS1 p^2)))
  constexpr float CS1 = -2.f * LOG2E * K_GELU * C_GELU;
  constexpr float D0 = 2.f * K_GELU, D1 = 6.f * K_GELU * C_GELU;  // gelu' = s + p (D0 + D1 p^2) s (1 - s)

  F2 acc_da[H], acc_db[H], acc_dg[GB ? H : 1], acc_dbe[GB ? H : 1];
#pragma unroll
  for (int i = 0; i < H; ++i) {
    acc_da[i] = acc_db[i] = sp(0.f);
    if (GB) acc_dg[i] = acc_dbe[i] = sp(0.f);
  }

  auto prefetch = [&](int64_t row, int stage) {
    if (row < P.rows) {
      float* dx_ = sm + ((size_t)stage * 2 * T + threadIdx.x) * V;
      float* dc_ = dx_ + (size_t)T * V;
      const float* xr = P.x + row * C + c0;
      const float* cr = P.c + row * C + c0;
      if (vec) {
#pragma unroll
        for (int i = 0; i < V; i += 4) {
          cp_async16(dx_ + i, xr + i);
          cp_async16(dc_ + i, cr + i);
        }
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const bool ok = c0 + i < C;
          cp_async4(dx_ + i, ok ? xr + i : P.x, ok);
          cp_async4(dc_ + i, ok ? cr + i : P.c, ok);
        }
      }
    }
    cp_async_commit();
  };
  auto lds_pairs = [&](const float* src, F2 (&r)[H]) {
#pragma unroll
    for (int i = 0; i < V; i += 4) {
      const float4 u = *reinterpret_cast<const float4*>(src + i);
      r[i / 2] = pk(u.x, u.y);
      r[i / 2 + 1] = pk(u.z, u.w);
    }
  };
  // gamma log2e and beta' log2e of this thread's columns (shared memory or registers)
  auto col_vecs = [&](F2 (&g)[H], F2 (&e)[H]) {
    if (GLSM) {
      lds_pairs(sgl, g);
      lds_pairs(sbl, e);
    } else {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        g[i] = glr[GLSM ? 0 : i];
        e[i] = blr[GLSM ? 0 : i];
      }
    }
  };
  auto store_row = [&](float* dst, const F2 (&r)[H]) {
    if (vec) {
#pragma unroll
      for (int i = 0; i < V; i += 4) {
        float u0, u1, u2, u3;
        upk(r[i / 2], u0, u1);
        upk(r[i / 2 + 1], u2, u3);
        __stcs(reinterpret_cast<float4*>(dst + c0 + i), make_float4(u0, u1, u2, u3));
      }
    } else if (any) {
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        float u0, u1;
        upk(r[i / 2], u0, u1);
        if (c0 + i < C) dst[c0 + i] = u0;
        if (c0 + i + 1 < C) dst[c0 + i + 1] = u1;
      }
    }
  };

  prefetch(blockIdx.x, 0);
  int stage = 0;
  for (int64_t row = blockIdx.x; row < P.rows; row += G, stage ^= 1) {
    prefetch(row + G, stage ^ 1);
    cp_async_wait<1>();
    const float* xs = sm + ((size_t)stage * 2 * T + threadIdx.x) * V;
    const float* cs = xs + (size_t)T * V;
    F2 sg[H], w[H];
    // ---- forward: p = x a + b ; s = sigma(2u) ; w = g = p s
    F2 s2 = sp(0.f), q2 = sp(0.f);
    {
      F2 x[H];
      lds_pairs(xs, x);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 u = mul2(p, fma2(mul2(p, p), sp(CS1), sp(CS0)));
        float u0, u1, d0, d1;
        upk(u, u0, u1);
        upk(add2(pk(ex2_approx(u0), ex2_approx(u1)), sp(1.f)), d0, d1);
        sg[i] = pk(rcp_approx(d0), rcp_approx(d1));
        w[i] = mul2(p, sg[i]);
        s2 = add2(s2, w[i]);
        q2 = fma2(w[i], w[i], q2);
      }
    }
    float sa, sb, qa, qb;
    upk(s2, sa, sb);
    upk(q2, qa, qb);
    const float2 SQ = block_pair_sum<NW>(sa + sb, qa + qb, red[0], lane, wid);
    const float mean = SQ.x * invC;
    const float rstd = rsqrtf(fmaxf(SQ.y * invC - mean * mean, 0.f) + P.eps);
    const F2 rs = sp(rstd), nmr = sp(-mean * rstd);
    // ---- z = (g_hat gamma + beta - shift) log2e ; e = 2^z ; sum e, sum c e, max e
    {
      F2 gl[H], bl[H];
      col_vecs(gl, bl);
#pragma unroll
      for (int i = 0; i < H; ++i) w[i] = fma2(fma2(w[i], rs, nmr), gl[i], bl[i]);
    }
    if (!use_shift) {  // per-row max of z
      float mz = -INFINITY;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[i], u0, u1);
        mz = fmaxf(mz, fmaxf(u0, u1));
      }
      const F2 nz = sp(-ord_value(block_max_key<NW>(ord_key(mz), red[1], lane, wid)));
#pragma unroll
      for (int i = 0; i < H; ++i) w[i] = add2(w[i], nz);
    }
    F2 se2 = sp(0.f), sce2 = sp(0.f);
    float me = 0.f;
    {
      F2 c[H];
      lds_pairs(cs, c);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[i], u0, u1);
        u0 = ex2_approx(u0);
        u1 = ex2_approx(u1);
        me = fmaxf(me, fmaxf(u0, u1));
        w[i] = pk(u0, u1);
        se2 = add2(se2, w[i]);
        sce2 = fma2(c[i], w[i], sce2);
      }
    }
    upk(se2, sa, sb);
    upk(sce2, qa, qb);
    uint32_t emax = __float_as_uint(me);  // e >= 0: the bit pattern orders like the value
    const float2 E = block_pair_sum_max<NW>(sa + sb, qa + qb, emax, red[2], lane, wid);
    const float inv = rcp_approx(E.x);  // sum e >= 2^-115 (the shift bound) is a normal number
    const float cy = E.y * inv;
    if (P.am) {  // argmax(y): the first column whose y equals the row's largest y
      const float ymax = __uint_as_float(emax) * inv;
      if (me * inv == ymax) {
        int first = 0x7fffffff;
#pragma unroll
        for (int i = H - 1; i >= 0; --i) {
          float u0, u1;
          upk(mul2(w[i], sp(inv)), u0, u1);
          if (u1 == ymax) first = c0 + 2 * i + 1;
          if (u0 == ymax) first = c0 + 2 * i;
        }
        atomicMin(&s_am, first);
      }
    }
    // ---- y = e / sum e ; dn = y (c - cy) ; w = dn gamma log2e ; S1 = sum w, S2 = sum w g_hat
    F2 s12 = sp(0.f), s22 = sp(0.f);
    {
      F2 c[H], x[H], y[H], gl[H], bl[H];
      lds_pairs(cs, c);
      lds_pairs(xs, x);
      col_vecs(gl, bl);
      const F2 iv = sp(inv), ncy = sp(-cy);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        y[i] = mul2(w[i], iv);
        const F2 dn = mul2(y[i], add2(c[i], ncy));
        const F2 gh = fma2(mul2(fma2(x[i], a[i], b[i]), sg[i]), rs, nmr);
        if (GB) {
          acc_dg[GB ? i : 0] = fma2(dn, gh, acc_dg[GB ? i : 0]);
          acc_dbe[GB ? i : 0] = add2(acc_dbe[GB ? i : 0], dn);
        }
        w[i] = mul2(dn, gl[i]);
        s12 = add2(s12, w[i]);
        s22 = fma2(w[i], gh, s22);
      }
      store_row(P.y + row * C, y);
    }
    float s1a, s1b, s2a, s2b;
    upk(s12, s1a, s1b);
    upk(s22, s2a, s2b);
    const float2 S = block_pair_sum<NW>(s1a + s1b, s2a + s2b, red[3], lane, wid);
    if (P.am && threadIdx.x == 0) {
      const int j = s_am;
      P.am[row] = j == 0x7fffffff ? 0 : j;  // no candidate: y is NaN throughout, argmax 0
      s_am = 0x7fffffff;
    }
    // ---- dg = rstd/C (C dn gamma - S1 - g_hat S2), with g_hat = g rstd - mean rstd folded in:
    //      dg = g A + (w kC + B) ; dp = dg gelu'(p) ; dx = dp a ; da += dp x ; db += dp
    {
      const float kC = rstd * (1.f / LOG2E);
      const float kS2 = -kC * invC * S.y;
      const F2 fkC = sp(kC), fA = sp(rstd * kS2), fB = sp(fmaf(-mean * rstd, kS2, -kC * invC * S.x));
      F2 x[H], dx[H];
      lds_pairs(xs, x);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 dg = fma2(mul2(p, sg[i]), fA, fma2(w[i], fkC, fB));
        // gelu'(p) = s + r (1 - s) with r = p (D0 + D1 p^2) s
        const F2 r = mul2(mul2(p, fma2(mul2(p, p), sp(D1), sp(D0))), sg[i]);
        const F2 gd = sub2(add2(sg[i], r), mul2(r, sg[i]));
        const F2 dp = mul2(dg, gd);
        dx[i] = mul2(dp, a[i]);
        acc_da[i] = fma2(dp, x[i], acc_da[i]);
        acc_db[i] = add2(acc_db[i], dp);
      }
      store_row(P.dx + row * C, dx);
    }
  }
  cp_async_wait<0>();
  // per-CTA column partials (each thread writes the columns it owns)
#pragma unroll
  for (int i = 0; i < H; ++i) {
    const int col = c0 + 2 * i;
    float u0, u1;
    F2 vals[4] = {acc_da[i], acc_db[i], GB ? acc_dg[GB ? i : 0] : sp(0.f), GB ? acc_dbe[GB ? i : 0] : sp(0.f)};
#pragma unroll
    for (int k = 0; k < (GB ? 4 : 2); ++k) {
      upk(vals[k], u0, u1);
      if (col < C) P.part[((int64_t)k * G + blockIdx.x) * C + col] = u0;
      if (col + 1 < C) P.part[((int64_t)k * G + blockIdx.x) * C + col + 1] = u1;
    }
  }
}

// out[k][col] = sum_g part[k][g][col] in a fixed order (deterministic): warp w of a block
// sums g = w, w + 8, w + 16, ... in increasing g for 32 adjacent columns, then the 8 warp
// sums are added in warp order. 8 independent chains per column keep enough loads in flight.
constexpr int CS_WARPS = 8;
__global__ void __launch_bounds__(32 * CS_WARPS) colsum_kernel(const float* __restrict__ part, float* __restrict__ o0,
                                                               float* __restrict__ o1, float* __restrict__ o2,
                                                               float* __restrict__ o3, int64_t G, int64_t C, int nk) {
  __shared__ float sh[CS_WARPS][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t col = (int64_t)blockIdx.x * 32 + lane;
  const int k = blockIdx.y;
  float* out = k == 0 ? o0 : k == 1 ? o1 : k == 2 ? o2 : o3;
  const bool live = col < C && k < nk && out != nullptr;
  float s = 0.f;
  if (live) {
    const float* p = part + (int64_t)k * G * C + col;
#pragma unroll 4
    for (int64_t g = w; g < G; g += CS_WARPS) s += __ldg(p + g * C);
  }
  sh[w][lane] = s;
  __syncthreads();
  if (w == 0 && live) {
    float t = sh[0][lane];
#pragma unroll
    for (int i = 1; i < CS_WARPS; ++i) t += sh[i][lane];
    out[col] = t;
  }
}

// ---- two rows per CTA in lockstep (4 columns per thread, no dgamma / dbeta) ----------
// The same computation as rowfused_kernel for rows r and r + G together: every block
// reduction carries both rows' values through one shuffle tree and one barrier, halving the
// barriers per row and amortising the per-row bookkeeping over twice the work.

// lanes 8k .. 8k+7 return the warp sum of v[k] (k = 0..3): one transposed shuffle tree
__device__ __forceinline__ float warp_quad_sum(float v0, float v1, float v2, float v3, int lane) {
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
  float k0 = h16 ? v2 : v0, k1 = h16 ? v3 : v1;
  const float s0 = h16 ? v0 : v2, s1 = h16 ? v1 : v3;
  k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
  k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
  float k = h8 ? k1 : k0;
  const float s = h8 ? k0 : k1;
  k += __shfl_xor_sync(0xffffffffu, s, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  return k;
}
// second level over NW warps: red[32 k + w] is warp w's sum of value k
template <int NW>
__device__ __forceinline__ float4 block_quad_finish(const float* red, int lane) {
  float t;
  if (NW == 32) {
    const float4 q = *reinterpret_cast<const float4*>(red + 4 * lane);  // value lane/8, warps 4 (lane%8) ..
    t = (q.x + q.y) + (q.z + q.w);
  } else if (NW == 16) {
    const float2 q = *reinterpret_cast<const float2*>(red + (lane >> 3) * 32 + 2 * (lane & 7));
    t = q.x + q.y;
  } else {
    t = (lane & 7) < NW ? red[(lane >> 3) * 32 + (lane & 7)] : 0.f;
  }
  t += __shfl_xor_sync(0xffffffffu, t, 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return make_float4(__shfl_sync(0xffffffffu, t, 0), __shfl_sync(0xffffffffu, t, 8), __shfl_sync(0xffffffffu, t, 16),
                     __shfl_sync(0xffffffffu, t, 24));
}
template <int NW>
__device__ __forceinline__ float4 block_quad_sum(float v0, float v1, float v2, float v3, float* red, int lane, int w) {
  const float v = warp_quad_sum(v0, v1, v2, v3, lane);
  if ((lane & 7) == 0) red[(lane >> 3) * 32 + w] = v;
  __syncthreads();
  return block_quad_finish<NW>(red, lane);
}
// the same plus the maxima of two unsigned keys (kred[0 .. NW), kred[32 .. 32 + NW))
template <int NW>
__device__ __forceinline__ float4 block_quad_sum_max2(float v0, float v1, float v2, float v3, uint32_t& m0, uint32_t& m1,
                                                      float* red, uint32_t* kred, int lane, int w) {
  const float v = warp_quad_sum(v0, v1, v2, v3, lane);
  const uint32_t w0 = __reduce_max_sync(0xffffffffu, m0), w1 = __reduce_max_sync(0xffffffffu, m1);
  if ((lane & 7) == 0) red[(lane >> 3) * 32 + w] = v;
  if (lane == 0) {
    kred[w] = w0;
    kred[32 + w] = w1;
  }
  __syncthreads();
  m0 = __reduce_max_sync(0xffffffffu, lane < NW ? kred[lane] : 0u);
  m1 = __reduce_max_sync(0xffffffffu, lane < NW ? kred[32 + lane] : 0u);
  return block_quad_finish<NW>(red, lane);
}
template <int NW>
__device__ __forceinline__ void block_max2_key(uint32_t& m0, uint32_t& m1, uint32_t* kred, int lane, int w) {
  const uint32_t w0 = __reduce_max_sync(0xffffffffu, m0), w1 = __reduce_max_sync(0xffffffffu, m1);
  if (lane == 0) {
    kred[w] = w0;
    kred[32 + w] = w1;
  }
  __syncthreads();
  m0 = __reduce_max_sync(0xffffffffu, lane < NW ? kred[lane] : 0u);
  m1 = __reduce_max_sync(0xffffffffu, lane < NW ? kred[32 + lane] : 0u);
}

// shared memory: [2 stages][x0, c0, x1, c1][T][4] (row r, row r + G), then
// [gamma log2e, beta' log2e, da accumulator, db accumulator, sigma row r, sigma row r + G][T][4]
// (224 KB at T = 1024, the static reduction sites included: just under the 227 KB limit)
constexpr size_t rowfused2_smem(int T) { return (size_t)(2 * 4 + 6) * T * 4 * sizeof(float); }

template <int T, bool RAGGED>
__global__ void __launch_bounds__(T, 1024 / T) rowfused2_kernel(const __grid_constant__ Params P) {
  constexpr int NW = T / 32, V = 4, H = 2;
  __shared__ __align__(16) float red[4][128];  // per-row reduction sites (site 0 also the set-up scratch)
  __shared__ __align__(16) uint32_t kred[2][64];  // key maxima of sites 1 and 2
  __shared__ int s_am[2];
  extern __shared__ __align__(16) float sm[];
  const int64_t C = P.cols;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c0 = threadIdx.x * V;
  const bool full = c0 + V <= C;
  const bool vec = full && ((C & 3) == 0) && P.aligned16;
  const bool any = c0 < C;
  const float invC = 1.f / (float)C;
  const int64_t G = gridDim.x;
  float* const sgl = sm + ((size_t)8 * T + threadIdx.x) * V;
  float* const sbl = sgl + (size_t)T * V;
  float* const sda = sbl + (size_t)T * V;  // this thread's column accumulators of da
  float* const sdb = sda + (size_t)T * V;  // and db
  float* const ssg = sdb + (size_t)T * V;  // sigma(2u) of this thread's columns, row r
  float* const ssg1 = ssg + (size_t)T * V;  // and row r + G

  F2 a[H], b[H];
  if (threadIdx.x < 2) s_am[threadIdx.x] = 0x7fffffff;
  bool use_shift;
  {
    float av[V], bv[V], glv[V], blv[V];
    use_shift = load_columns<NW, V, RAGGED>(P, c0, vec, av, bv, glv, blv, reinterpret_cast<float(*)[32]>(red[0]), lane, wid);
    a[0] = pk(av[0], av[1]); a[1] = pk(av[2], av[3]);
    b[0] = pk(bv[0], bv[1]); b[1] = pk(bv[2], bv[3]);
    *reinterpret_cast<float4*>(sgl) = make_float4(glv[0], glv[1], glv[2], glv[3]);
    *reinterpret_cast<float4*>(sbl) = make_float4(blv[0], blv[1], blv[2], blv[3]);
    __syncthreads();  // the set-up scratch is reduction site 0: every warp has read it
  }
  constexpr float CS0 = -2.f * LOG2E * K_GELU;
  constexpr float CS1 = -2.f * LOG2E * K_GELU * C_GELU;
  constexpr float D0 = 2.f * K_GELU, D1 = 6.f * K_GELU * C_GELU;

  *reinterpret_cast<float4*>(sda) = make_float4(0.f, 0.f, 0.f, 0.f);
  *reinterpret_cast<float4*>(sdb) = make_float4(0.f, 0.f, 0.f, 0.f);

  // slot of array k (0: x, 1: c of row r; 2: x, 3: c of row r + G) in a stage
  auto slot = [&](int stage, int k) { return sm + ((size_t)(stage * 4 + k) * T + threadIdx.x) * V; };
  auto prefetch = [&](int64_t row0, int stage) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int64_t row = row0 + r * G;
      if (row < P.rows) {
        float* dx_ = slot(stage, 2 * r);
        float* dc_ = slot(stage, 2 * r + 1);
        const float* xr = P.x + row * C + c0;
        const float* cr = P.c + row * C + c0;
        if (vec) {
          cp_async16(dx_, xr);
          cp_async16(dc_, cr);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const bool ok = c0 + i < C;
            cp_async4(dx_ + i, ok ? xr + i : P.x, ok);
            cp_async4(dc_ + i, ok ? cr + i : P.c, ok);
          }
        }
      }
    }
    cp_async_commit();
  };
  auto lds2 = [&](const float* src, F2 (&r)[H]) {
    const float4 u = *reinterpret_cast<const float4*>(src);
    r[0] = pk(u.x, u.y);
    r[1] = pk(u.z, u.w);
  };
  auto store_row = [&](float* dst, const F2 (&r)[H]) {
    if (vec) {
      float u0, u1, u2, u3;
      upk(r[0], u0, u1);
      upk(r[1], u2, u3);
      __stcs(reinterpret_cast<float4*>(dst + c0), make_float4(u0, u1, u2, u3));
    } else if (any) {
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        float u0, u1;
        upk(r[i / 2], u0, u1);
        if (c0 + i < C) dst[c0 + i] = u0;
        if (c0 + i + 1 < C) dst[c0 + i + 1] = u1;
      }
    }
  };

  const int64_t step = 2 * G;
  prefetch(blockIdx.x, 0);
  int stage = 0;
  for (int64_t row0 = blockIdx.x; row0 < P.rows; row0 += step, stage ^= 1) {
    const bool live1 = row0 + G < P.rows;  // the second row exists (uniform over the CTA)
    prefetch(row0 + step, stage ^ 1);
    cp_async_wait<1>();
    F2 w[2][H];
    // ---- forward: p = x a + b ; s = sigma(2u) ; w = g = p s
    float sv[2], qv[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      F2 x[H];
      lds2(slot(stage, 2 * r), x);
      F2 s2 = sp(0.f), q2 = sp(0.f);
      float sgv[4];
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 u = mul2(p, fma2(mul2(p, p), sp(CS1), sp(CS0)));
        float u0, u1, d0, d1;
        upk(u, u0, u1);
        upk(add2(pk(ex2_approx(u0), ex2_approx(u1)), sp(1.f)), d0, d1);
        sgv[2 * i] = rcp_approx(d0);
        sgv[2 * i + 1] = rcp_approx(d1);
        w[r][i] = mul2(p, pk(sgv[2 * i], sgv[2 * i + 1]));
        s2 = add2(s2, w[r][i]);
        q2 = fma2(w[r][i], w[r][i], q2);
      }
      *reinterpret_cast<float4*>(r ? ssg1 : ssg) = make_float4(sgv[0], sgv[1], sgv[2], sgv[3]);
      float sa, sb, qa, qb;
      upk(s2, sa, sb);
      upk(q2, qa, qb);
      sv[r] = sa + sb;
      qv[r] = qa + qb;
    }
    const float4 SQ = block_quad_sum<NW>(sv[0], qv[0], sv[1], qv[1], red[0], lane, wid);
    float mean[2], rstd[2];
    mean[0] = SQ.x * invC;
    mean[1] = SQ.z * invC;
    rstd[0] = rsqrtf(fmaxf(SQ.y * invC - mean[0] * mean[0], 0.f) + P.eps);
    rstd[1] = rsqrtf(fmaxf(SQ.w * invC - mean[1] * mean[1], 0.f) + P.eps);
    // ---- z = (g_hat gamma + beta - shift) log2e ; e = 2^z ; sum e, sum c e, max e
    {
      F2 gl[H], bl[H];
      lds2(sgl, gl);
      lds2(sbl, bl);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const F2 rs = sp(rstd[r]), nmr = sp(-mean[r] * rstd[r]);
#pragma unroll
        for (int i = 0; i < H; ++i) w[r][i] = fma2(fma2(w[r][i], rs, nmr), gl[i], bl[i]);
      }
    }
    if (!use_shift) {  // per-row max of z
      uint32_t mk[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float u0, u1, u2, u3;
        upk(w[r][0], u0, u1);
        upk(w[r][1], u2, u3);
        mk[r] = ord_key(fmaxf(fmaxf(u0, u1), fmaxf(u2, u3)));
      }
      block_max2_key<NW>(mk[0], mk[1], kred[0], lane, wid);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const F2 nz = sp(-ord_value(mk[r]));
#pragma unroll
        for (int i = 0; i < H; ++i) w[r][i] = add2(w[r][i], nz);
      }
    }
    float se[2], sce[2], me[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      F2 c[H];
      lds2(slot(stage, 2 * r + 1), c);
      F2 se2 = sp(0.f), sce2 = sp(0.f);
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[r][i], u0, u1);
        u0 = ex2_approx(u0);
        u1 = ex2_approx(u1);
        m = fmaxf(m, fmaxf(u0, u1));
        w[r][i] = pk(u0, u1);
        se2 = add2(se2, w[r][i]);
        sce2 = fma2(c[i], w[r][i], sce2);
      }
      float sa, sb, qa, qb;
      upk(se2, sa, sb);
      upk(sce2, qa, qb);
      se[r] = sa + sb;
      sce[r] = qa + qb;
      me[r] = m;
    }
    uint32_t emax0 = __float_as_uint(me[0]), emax1 = __float_as_uint(me[1]);  // e >= 0: bits order like values
    const float4 E = block_quad_sum_max2<NW>(se[0], sce[0], se[1], sce[1], emax0, emax1, red[2], kred[1], lane, wid);
    float inv[2], cy[2];
    inv[0] = rcp_approx(E.x);  // sum e >= 2^-115 (the shift bound) is a normal number
    inv[1] = rcp_approx(E.z);
    cy[0] = E.y * inv[0];
    cy[1] = E.w * inv[1];
    if (P.am) {  // argmax(y): the first column whose y equals the row's largest y
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float ymax = __uint_as_float(r ? emax1 : emax0) * inv[r];
        if ((r == 0 || live1) && me[r] * inv[r] == ymax) {
          int first = 0x7fffffff;
#pragma unroll
          for (int i = H - 1; i >= 0; --i) {
            float u0, u1;
            upk(mul2(w[r][i], sp(inv[r])), u0, u1);
            if (u1 == ymax) first = c0 + 2 * i + 1;
            if (u0 == ymax) first = c0 + 2 * i;
          }
          atomicMin(&s_am[r], first);
        }
      }
    }
    // ---- y = e / sum e ; dn = y (c - cy) ; w = dn gamma log2e ; S1 = sum w, S2 = sum w g_hat
    float s1v[2], s2v[2];
    {
      F2 gl[H];
      lds2(sgl, gl);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        F2 c[H], x[H], y[H], sg[H];
        lds2(slot(stage, 2 * r + 1), c);
        lds2(slot(stage, 2 * r), x);
        lds2(r ? ssg1 : ssg, sg);
        const F2 iv = sp(inv[r]), ncy = sp(-cy[r]);
        const F2 rs = sp(rstd[r]), nmr = sp(-mean[r] * rstd[r]);
        F2 s12 = sp(0.f), s22 = sp(0.f);
#pragma unroll
        for (int i = 0; i < H; ++i) {
          y[i] = mul2(w[r][i], iv);
          const F2 dn = mul2(y[i], add2(c[i], ncy));
          const F2 gh = fma2(mul2(fma2(x[i], a[i], b[i]), sg[i]), rs, nmr);
          w[r][i] = mul2(dn, gl[i]);
          s12 = add2(s12, w[r][i]);
          s22 = fma2(w[r][i], gh, s22);
        }
        if (r == 0 || live1) store_row(P.y + (row0 + r * G) * C, y);
        float a0, a1, b0, b1;
        upk(s12, a0, a1);
        upk(s22, b0, b1);
        s1v[r] = a0 + a1;
        s2v[r] = b0 + b1;
      }
    }
    const float4 S = block_quad_sum<NW>(s1v[0], s2v[0], s1v[1], s2v[1], red[3], lane, wid);
    if (P.am && threadIdx.x == 0) {
      const int j0 = s_am[0];
      P.am[row0] = j0 == 0x7fffffff ? 0 : j0;  // no candidate: y is NaN throughout, argmax 0
      s_am[0] = 0x7fffffff;
      if (live1) {
        const int j1 = s_am[1];
        P.am[row0 + G] = j1 == 0x7fffffff ? 0 : j1;
      }
      s_am[1] = 0x7fffffff;
    }
    // ---- dg = g A + (w kC + B) ; dp = dg gelu'(p) ; dx = dp a ; da += dp x ; db += dp
    F2 acc_da[H], acc_db[H];
    lds2(sda, acc_da);
    lds2(sdb, acc_db);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r == 1 && !live1) break;
      const float kC = rstd[r] * (1.f / LOG2E);
      const float S1 = r ? S.z : S.x, S2 = r ? S.w : S.y;
      const float kS2 = -kC * invC * S2;
      const F2 fkC = sp(kC), fA = sp(rstd[r] * kS2), fB = sp(fmaf(-mean[r] * rstd[r], kS2, -kC * invC * S1));
      F2 x[H], dx[H], sg[H];
      lds2(slot(stage, 2 * r), x);
      lds2(r ? ssg1 : ssg, sg);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 dg = fma2(mul2(p, sg[i]), fA, fma2(w[r][i], fkC, fB));
        const F2 rr = mul2(mul2(p, fma2(mul2(p, p), sp(D1), sp(D0))), sg[i]);
        const F2 gd = sub2(add2(sg[i], rr), mul2(rr, sg[i]));
        const F2 dp = mul2(dg, gd);
        dx[i] = mul2(dp, a[i]);
        acc_da[i] = fma2(dp, x[i], acc_da[i]);
        acc_db[i] = add2(acc_db[i], dp);
      }
      store_row(P.dx + (row0 + r * G) * C, dx);
    }
    {
      float u0, u1, u2, u3;
      upk(acc_da[0], u0, u1);
      upk(acc_da[1], u2, u3);
      *reinterpret_cast<float4*>(sda) = make_float4(u0, u1, u2, u3);
      upk(acc_db[0], u0, u1);
      upk(acc_db[1], u2, u3);
      *reinterpret_cast<float4*>(sdb) = make_float4(u0, u1, u2, u3);
    }
  }
  cp_async_wait<0>();
  // per-CTA column partials (each thread writes the columns it owns)
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int col = c0 + i;
    if (col < C) {
      P.part[(int64_t)blockIdx.x * C + col] = sda[i];
      P.part[((int64_t)G + blockIdx.x) * C + col] = sdb[i];
    }
  }
}

template <int T>
int launch2(const Params& P, int64_t grid, cudaStream_t s) {
  const size_t smem = rowfused2_smem(T);
  const bool ragged = P.cols != (int64_t)T * 4;
  if (ragged) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(rowfused2_kernel<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rowfused2_kernel<T, true><<<(unsigned)grid, T, smem, s>>>(P);
  } else {
    if (smem > 48 * 1024) cudaFuncSetAttribute(rowfused2_kernel<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rowfused2_kernel<T, false><<<(unsigned)grid, T, smem, s>>>(P);
  }
  return check_launch("rowfused2");
}

template <int T, int V>
int launch(const Params& P, int64_t grid, cudaStream_t s) {
  const size_t smem = (size_t)(2 * 2 + (gl_in_smem(V) ? 2 : 0)) * T * V * sizeof(float);
  const bool ragged = P.cols != (int64_t)T * V;
#define B200_RF_LAUNCH(GB_, RG_)                                                                                        \
  do {                                                                                                                   \
    if (smem > 48 * 1024)                                                                                                \
      cudaFuncSetAttribute(rowfused_kernel<T, V, GB_, RG_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);     \
    rowfused_kernel<T, V, GB_, RG_><<<(unsigned)grid, T, smem, s>>>(P);                                                  \
  } while (0)
  if (P.want_gb) {
    if (ragged) B200_RF_LAUNCH(true, true);
    else B200_RF_LAUNCH(true, false);
  } else {
    if (ragged) B200_RF_LAUNCH(false, true);
    else B200_RF_LAUNCH(false, false);
  }
#undef B200_RF_LAUNCH
  return check_launch("rowfused");
}

// threads per CTA for a row length: 4 columns per thread up to 4096 columns (32 warps
// per SM hide the reduction and transcendental latencies), 8 up to 8192, then 16
#ifndef B200_RF_V4_MAX_COLS
#define B200_RF_V4_MAX_COLS 4096
#endif
inline bool use_two_row_kernel() {
#ifdef B200_RF_ONE_ROW
  return false;
#else
  return true;
#endif
}
inline void shape_for(int64_t cols, int& T, int& V) {
  V = cols <= B200_RF_V4_MAX_COLS ? 4 : (cols <= 8192 ? 8 : 16);
  const int64_t t = (cols + V - 1) / V;
  T = 32;
  while (T < t) T *= 2;
}

// 1024 resident threads per SM for V = 4 (64 registers each), 512 otherwise
inline int64_t grid_for(int64_t rows, int64_t cols) {
  int T, V;
  shape_for(cols, T, V);
  const int64_t per_sm = V == 4 ? std::max(1, 1024 / T) : std::max(1, 512 / T);
  return std::max<int64_t>(1, std::min<int64_t>(rows, (int64_t)num_sms() * per_sm));
}

template <int T, int V>
int launch(const Params& P, int64_t grid, cudaStream_t s);

}  // namespace rf
}  // namespace b200

using namespace b200;
using namespace b200::rf;

extern "C" size_t b200_rowfused_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return (size_t)4 * (size_t)grid_for(rows, cols) * (size_t)cols * sizeof(float);
}

extern "C" int b200_rowfused_fwd_bwd(const float* x, const float* a, const float* b, const float* gamma, const float* beta,
                                     const float* cot, float* y, int64_t* am, float* dx, float* da, float* db, float* dgamma,
                                     float* dbeta, int64_t rows, int64_t cols, float eps, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  B200_REQUIRE(x && a && b && cot && y && dx && da && db, "rowfused: null required pointer");
  B200_REQUIRE(rows >= 0 && cols >= 1, "rowfused: bad sizes");
  B200_REQUIRE(cols <= 16384, "rowfused: cols %lld > 16384", (long long)cols);
  B200_REQUIRE(eps >= 0.f, "rowfused: negative eps");
  const size_t need = b200_rowfused_workspace_bytes(rows, cols);
  B200_REQUIRE(rows == 0 || (workspace && workspace_bytes >= need), "rowfused: workspace %zu bytes < %zu", workspace_bytes, need);
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    cudaMemsetAsync(da, 0, cols * 4, s);
    cudaMemsetAsync(db, 0, cols * 4, s);
    if (dgamma) cudaMemsetAsync(dgamma, 0, cols * 4, s);
    if (dbeta) cudaMemsetAsync(dbeta, 0, cols * 4, s);
    return check_launch("rowfused(empty)");
  }
  Params P;
  P.x = x; P.a = a; P.b = b; P.gamma = gamma; P.beta = beta; P.c = cot;
  P.y = y; P.dx = dx; P.am = am;
  P.part = reinterpret_cast<float*>(workspace);
  P.rows = rows; P.cols = cols; P.eps = eps;
  P.want_gb = (dgamma || dbeta) ? 1 : 0;
  auto al = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  P.aligned16 = al(x) && al(a) && al(b) && al(gamma) && al(beta) && al(cot) && al(y) && al(dx) ? 1 : 0;
  int T, V;
  shape_for(cols, T, V);
  const int64_t grid = grid_for(rows, cols);
  int rc;
  if (V == 4 && !P.want_gb && use_two_row_kernel()) {
    // rows r and r + G per CTA: half as many CTAs over the same rows
    const int64_t grid2 = std::max<int64_t>(1, std::min<int64_t>(grid, (rows + 1) / 2));
    switch (T) {
      case 32: rc = launch2<32>(P, grid2, s); break;
      case 64: rc = launch2<64>(P, grid2, s); break;
      case 128: rc = launch2<128>(P, grid2, s); break;
      case 256: rc = launch2<256>(P, grid2, s); break;
      case 512: rc = launch2<512>(P, grid2, s); break;
      default: rc = launch2<1024>(P, grid2, s); break;
    }
    if (rc) return rc;
    dim3 g2((unsigned)ceil_div(cols, 32), 2);
    colsum_kernel<<<g2, 32 * CS_WARPS, 0, s>>>(P.part, da, db, nullptr, nullptr, grid2, cols, 2);
    return check_launch("rowfused(colsum)");
  }
  if (V == 4) {
    switch (T) {
      case 32: rc = launch<32, 4>(P, grid, s); break;
      case 64: rc = launch<64, 4>(P, grid, s); break;
      case 128: rc = launch<128, 4>(P, grid, s); break;
      case 256: rc = launch<256, 4>(P, grid, s); break;
      case 512: rc = launch<512, 4>(P, grid, s); break;
      default: rc = launch<1024, 4>(P, grid, s); break;
    }
  } else if (V == 8) {
    rc = launch<1024, 8>(P, grid, s);
  } else {
    rc = launch<1024, 16>(P, grid, s);
  }
  if (rc) return rc;
  dim3 g2((unsigned)ceil_div(cols, 32), P.want_gb ? 4 : 2);
  colsum_kernel<<<g2, 32 * CS_WARPS, 0, s>>>(P.part, da, db, dgamma, dbeta, grid, cols, P.want_gb ? 4 : 2);
  return check_launch("rowfused(colsum)");
}

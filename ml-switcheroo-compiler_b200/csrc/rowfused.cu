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

// tanh(u) = 1 - 2 / (exp(2u) + 1), exp through ex2.approx, reciprocal through rcp.approx:
// absolute error ~1e-7, saturates to +-1 for large |u|.
__device__ __forceinline__ float fast_tanh(float u) {
  const float e = exp2f(2.f * LOG2E * u);
  return fmaf(-2.f, __frcp_rn(e + 1.f), 1.f);
}

struct Red2 {
  float a, b;
};

template <int NW>
__device__ __forceinline__ float bsum(float v, float* sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float t = lane < NW ? sh[lane] : 0.f;
  return warp_sum(t);
}
template <int NW>
__device__ __forceinline__ Red2 bsum2(float a, float b, float* sh) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    sh[w] = a;
    sh[32 + w] = b;
  }
  __syncthreads();
  float ta = lane < NW ? sh[lane] : 0.f, tb = lane < NW ? sh[32 + lane] : 0.f;
  return {warp_sum(ta), warp_sum(tb)};
}
template <int NW>
__device__ __forceinline__ float bmax(float v, float* sh) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float t = lane < NW ? sh[lane] : -INFINITY;
  return warp_max(t);
}
// block argmax (first max wins) fused with a block sum
template <int NW>
__device__ __forceinline__ void bsum_argmax(float& s, float& m, int& j, float* sh, int* shi) {
  s = warp_sum(s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    int j2 = __shfl_xor_sync(0xffffffffu, j, o);
    if (m2 > m || (m2 == m && j2 < j)) {
      m = m2;
      j = j2;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    sh[w] = s;
    sh[32 + w] = m;
    shi[w] = j;
  }
  __syncthreads();
  s = lane < NW ? sh[lane] : 0.f;
  m = lane < NW ? sh[32 + lane] : -INFINITY;
  j = lane < NW ? shi[lane] : 0x7fffffff;
  s = warp_sum(s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    int j2 = __shfl_xor_sync(0xffffffffu, j, o);
    if (m2 > m || (m2 == m && j2 < j)) {
      m = m2;
      j = j2;
    }
  }
}

struct Params {
  const float *x, *a, *b, *gamma, *beta, *c;
  float *y, *dx;
  int64_t* am;
  float* part;  // [4][grid][cols] partial column sums: da, db, dgamma, dbeta
  int64_t rows, cols;
  float eps;
  int want_gb;  // accumulate dgamma / dbeta partials
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
// tanh(u) = 1 - 2 / (exp(2u) + 1) on a pair; `u2l` is 2*log2(e)*u
__device__ __forceinline__ F2 tanh2_from_scaled(F2 u2l) {
  float a, b;
  upk(u2l, a, b);
  a = rcp_approx(ex2_approx(a) + 1.f);
  b = rcp_approx(ex2_approx(b) + 1.f);
  return fma2(pk(a, b), sp(-2.f), sp(1.f));
}

template <int V>
__device__ __forceinline__ void ldg_pairs(F2 (&r)[V / 2], const float* __restrict__ p, int c0, int64_t C, bool vec, float dflt) {
  if (p && vec) {
#pragma unroll
    for (int i = 0; i < V; i += 4) {
      float4 t = __ldg(reinterpret_cast<const float4*>(p + c0 + i));
      r[i / 2] = pk(t.x, t.y);
      r[i / 2 + 1] = pk(t.z, t.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < V; i += 2)
      r[i / 2] = pk((p && c0 + i < C) ? p[c0 + i] : dflt, (p && c0 + i + 1 < C) ? p[c0 + i + 1] : dflt);
  }
}

// T threads, V consecutive columns per thread (cols <= T*V), V/2 packed pairs.
// Registers hold x, c, one working row array w and the forward tanh t; a, b, gamma,
// beta are re-read through L1; the da/db (and dgamma/dbeta) column accumulators of
// this CTA live in shared memory, one slot per column, owned by one thread (no atomics).
template <int T, int V, bool GB, bool RAGGED>
__global__ void __launch_bounds__(T, T <= 256 ? 2 : 1) rowfused_kernel(const __grid_constant__ Params P) {
  constexpr int NW = T / 32;
  constexpr int H = V / 2;
  __shared__ float sh[64];
  __shared__ int shi[32];
  extern __shared__ float acc[];  // [2 or 4][cols]
  const int64_t C = P.cols;
  const int c0 = threadIdx.x * V;
  const bool vec = (c0 + V <= C) && ((C & 3) == 0);
  const bool any = c0 < C;
  const int nacc = GB ? 4 : 2;
  for (int64_t i = threadIdx.x; i < nacc * C; i += T) acc[i] = 0.f;
  // valid-column mask of pair i (only rows that do not tile exactly need it)
  auto msk = [&](int i) -> F2 {
    return RAGGED ? pk(c0 + 2 * i < C ? 1.f : 0.f, c0 + 2 * i + 1 < C ? 1.f : 0.f) : sp(1.f);
  };
  auto mul_mask = [&](F2 v, int i) -> F2 { return RAGGED ? mul2(v, msk(i)) : v; };
  const float invC = 1.f / (float)C;
  const float KG2L = 2.f * K_GELU * LOG2E;  // 2 k log2(e)

  for (int64_t row = blockIdx.x; row < P.rows; row += gridDim.x) {
    const float* xr = P.x + row * C;
    const float* cr = P.c + row * C;
    F2 x[H], c[H], w[H], t[H];
    if (vec) {
#pragma unroll
      for (int i = 0; i < V; i += 4) {
        float4 u = __ldcs(reinterpret_cast<const float4*>(xr + c0 + i));
        x[i / 2] = pk(u.x, u.y);
        x[i / 2 + 1] = pk(u.z, u.w);
        float4 q = __ldcs(reinterpret_cast<const float4*>(cr + c0 + i));
        c[i / 2] = pk(q.x, q.y);
        c[i / 2 + 1] = pk(q.z, q.w);
      }
    } else {
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        x[i / 2] = pk(c0 + i < C ? xr[c0 + i] : 0.f, c0 + i + 1 < C ? xr[c0 + i + 1] : 0.f);
        c[i / 2] = pk(c0 + i < C ? cr[c0 + i] : 0.f, c0 + i + 1 < C ? cr[c0 + i + 1] : 0.f);
      }
    }
    // ---- forward: p = x a + b ; t = tanh(k p (1 + c p^2)) ; w = g = 0.5 p (1 + t)
    F2 s2 = sp(0.f);
    {
      F2 a[H], b[H];
      ldg_pairs<V>(a, P.a, c0, C, vec, 0.f);
      ldg_pairs<V>(b, P.b, c0, C, vec, 0.f);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 q = fma2(mul2(p, p), sp(C_GELU), sp(1.f));
        t[i] = tanh2_from_scaled(mul2(mul2(p, q), sp(KG2L)));
        const F2 hp = mul2(p, sp(0.5f));
        w[i] = mul_mask(fma2(hp, t[i], hp), i);
        s2 = add2(s2, w[i]);
      }
    }
    float sa, sb;
    upk(s2, sa, sb);
    const float mean = bsum<NW>(sa + sb, sh) * invC;
    F2 q2 = sp(0.f);
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const F2 d = mul_mask(add2(w[i], sp(-mean)), i);
      q2 = fma2(d, d, q2);
    }
    upk(q2, sa, sb);
    const float rstd = rsqrtf(bsum<NW>(sa + sb, sh) * invC + P.eps);
    // w = n = LayerNorm(g); row max
    float m = -INFINITY;
    {
      F2 ga[H], be[H];
      ldg_pairs<V>(ga, P.gamma, c0, C, vec, 1.f);
      ldg_pairs<V>(be, P.beta, c0, C, vec, 0.f);
      const F2 nmr = sp(-mean * rstd), rs = sp(rstd);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        w[i] = fma2(fma2(w[i], rs, nmr), ga[i], be[i]);
        float u0, u1;
        upk(w[i], u0, u1);
        if (c0 + 2 * i < C) m = fmaxf(m, u0);
        if (c0 + 2 * i + 1 < C) m = fmaxf(m, u1);
      }
    }
    const float M = bmax<NW>(m, sh);
    // w = exp(n - M)
    F2 se2 = sp(0.f);
    {
      const F2 ml = sp(-M * LOG2E), l2 = sp(LOG2E);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(fma2(w[i], l2, ml), u0, u1);
        w[i] = mul_mask(pk(ex2_approx(u0), ex2_approx(u1)), i);
        se2 = add2(se2, w[i]);
      }
    }
    upk(se2, sa, sb);
    const float inv = 1.f / bsum<NW>(sa + sb, sh);
    // w = y ; sum(c*y) ; argmax(y) (first max wins)
    F2 cy2 = sp(0.f);
    float ym = -INFINITY;
    int yj = 0x7fffffff;
    {
      const F2 iv = sp(inv);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        w[i] = mul2(w[i], iv);
        cy2 = fma2(c[i], w[i], cy2);
        float u0, u1;
        upk(w[i], u0, u1);
        if (c0 + 2 * i < C && u0 > ym) {
          ym = u0;
          yj = c0 + 2 * i;
        }
        if (c0 + 2 * i + 1 < C && u1 > ym) {
          ym = u1;
          yj = c0 + 2 * i + 1;
        }
      }
    }
    upk(cy2, sa, sb);
    float cy = sa + sb;
    bsum_argmax<NW>(cy, ym, yj, sh, shi);
    if (P.am && threadIdx.x == 0) P.am[row] = yj;
    float* yr = P.y + row * C;
    if (vec) {
#pragma unroll
      for (int i = 0; i < V; i += 4) {
        float u0, u1, u2, u3;
        upk(w[i / 2], u0, u1);
        upk(w[i / 2 + 1], u2, u3);
        __stcs(reinterpret_cast<float4*>(yr + c0 + i), make_float4(u0, u1, u2, u3));
      }
    } else if (any) {
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        float u0, u1;
        upk(w[i / 2], u0, u1);
        if (c0 + i < C) yr[c0 + i] = u0;
        if (c0 + i + 1 < C) yr[c0 + i + 1] = u1;
      }
    }
    // ---- backward. c = dn = y (c - cy) (y dies here); t = tanh recomputed from x
    F2 s12 = sp(0.f), s22 = sp(0.f);
    {
      const F2 ncy = sp(-cy);
#pragma unroll
      for (int i = 0; i < H; ++i) c[i] = mul2(w[i], add2(c[i], ncy));
    }
    {
      F2 a[H], b[H];
      ldg_pairs<V>(a, P.a, c0, C, vec, 0.f);
      ldg_pairs<V>(b, P.b, c0, C, vec, 0.f);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 q = fma2(mul2(p, p), sp(C_GELU), sp(1.f));
        t[i] = tanh2_from_scaled(mul2(mul2(p, q), sp(KG2L)));
      }
    }
    {
      F2 a[H], b[H], ga[H];
      ldg_pairs<V>(a, P.a, c0, C, vec, 0.f);
      ldg_pairs<V>(b, P.b, c0, C, vec, 0.f);
      ldg_pairs<V>(ga, P.gamma, c0, C, vec, 1.f);
      const F2 nmr = sp(-mean * rstd), rs = sp(rstd);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 hp = mul2(p, sp(0.5f));
        const F2 gh = mul_mask(fma2(fma2(hp, t[i], hp), rs, nmr), i);
        const F2 dyg = mul2(c[i], ga[i]);
        s12 = add2(s12, dyg);
        s22 = fma2(dyg, gh, s22);
      }
    }
    float s1a, s1b, s2a, s2b;
    upk(s12, s1a, s1b);
    upk(s22, s2a, s2b);
    const Red2 S = bsum2<NW>(s1a + s1b, s2a + s2b, sh);
    {
      F2 a[H], b[H], ga[H];
      ldg_pairs<V>(a, P.a, c0, C, vec, 0.f);
      ldg_pairs<V>(b, P.b, c0, C, vec, 0.f);
      ldg_pairs<V>(ga, P.gamma, c0, C, vec, 1.f);
      const F2 k1 = sp(rstd * invC), fC = sp((float)C), nS1 = sp(-S.a), nS2 = sp(-S.b);
      const F2 nmr = sp(-mean * rstd), rs = sp(rstd);
      float* accda = acc;
      float* accdb = acc + C;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 hp0 = mul2(p, sp(0.5f));
        w[i] = mul_mask(fma2(fma2(hp0, t[i], hp0), rs, nmr), i);  // g_hat
        // dg = rstd/C (C dyg - S1 - g_hat S2)
        const F2 dg = mul2(k1, fma2(w[i], nS2, fma2(fC, mul2(c[i], ga[i]), nS1)));
        // gelu'(p) = 0.5 (1 + t) + 0.5 k p (1 - t^2) (1 + 3 c p^2)
        const F2 A = fma2(t[i], sp(0.5f), sp(0.5f));
        const F2 sech2 = fma2(t[i], mul2(t[i], sp(-1.f)), sp(1.f));
        const F2 Bq = fma2(mul2(p, p), sp(3.f * C_GELU), sp(1.f));
        const F2 gd = fma2(mul2(mul2(p, sp(0.5f * K_GELU)), sech2), Bq, A);
        const F2 dp = mul_mask(mul2(dg, gd), i);
        const int col = c0 + 2 * i;
        if (col < C) {
          float d0, d1, x0, x1;
          upk(dp, d0, d1);
          upk(x[i], x0, x1);
          accda[col] = fmaf(d0, x0, accda[col]);
          accdb[col] += d0;
          if (col + 1 < C) {
            accda[col + 1] = fmaf(d1, x1, accda[col + 1]);
            accdb[col + 1] += d1;
          }
          if (GB) {
            float n0, n1, g0, g1;
            upk(c[i], n0, n1);
            upk(w[i], g0, g1);
            acc[2 * C + col] = fmaf(n0, g0, acc[2 * C + col]);
            acc[3 * C + col] += n0;
            if (col + 1 < C) {
              acc[2 * C + col + 1] = fmaf(n1, g1, acc[2 * C + col + 1]);
              acc[3 * C + col + 1] += n1;
            }
          }
        }
        x[i] = mul2(dp, a[i]);  // x now holds dx
      }
    }
    float* dxr = P.dx + row * C;
    if (vec) {
#pragma unroll
      for (int i = 0; i < V; i += 4) {
        float u0, u1, u2, u3;
        upk(x[i / 2], u0, u1);
        upk(x[i / 2 + 1], u2, u3);
        __stcs(reinterpret_cast<float4*>(dxr + c0 + i), make_float4(u0, u1, u2, u3));
      }
    } else if (any) {
#pragma unroll
      for (int i = 0; i < V; i += 2) {
        float u0, u1;
        upk(x[i / 2], u0, u1);
        if (c0 + i < C) dxr[c0 + i] = u0;
        if (c0 + i + 1 < C) dxr[c0 + i + 1] = u1;
      }
    }
  }
  // per-CTA column partials (each thread flushes the columns it owns)
  __syncthreads();
  const int64_t G = gridDim.x;
  for (int64_t col = threadIdx.x; col < C; col += T) {
    for (int k = 0; k < nacc; ++k) P.part[((int64_t)k * G + blockIdx.x) * C + col] = acc[(int64_t)k * C + col];
  }
}

// out[k][col] = sum_g part[k][g][col], g in increasing order (deterministic)
__global__ void colsum_kernel(const float* __restrict__ part, float* __restrict__ o0, float* __restrict__ o1,
                              float* __restrict__ o2, float* __restrict__ o3, int64_t G, int64_t C, int nk) {
  const int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int k = blockIdx.y;
  if (col >= C || k >= nk) return;
  float* out = k == 0 ? o0 : k == 1 ? o1 : k == 2 ? o2 : o3;
  if (!out) return;
  const float* p = part + (int64_t)k * G * C + col;
  float s = 0.f;
  for (int64_t g = 0; g < G; ++g) s += p[g * C];
  out[col] = s;
}

template <int T, int V>
int launch(const Params& P, int64_t grid, cudaStream_t s) {
  const size_t smem = (size_t)(P.want_gb ? 4 : 2) * P.cols * sizeof(float);
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

// threads per CTA for a row length: 16 columns per thread (8 for short rows)
inline void shape_for(int64_t cols, int& T, int& V) {
  V = cols <= 512 ? 8 : 16;
  const int64_t t = (cols + V - 1) / V;
  T = 32;
  while (T < t) T *= 2;
}

// two CTAs per SM (up to 256 threads, <= 128 registers each), one for bigger CTAs
inline int64_t grid_for(int64_t rows, int64_t cols) {
  int T, V;
  shape_for(cols, T, V);
  const int64_t per_sm = T <= 256 ? 2 : 1;
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
  int T, V;
  shape_for(cols, T, V);
  const int64_t grid = grid_for(rows, cols);
  int rc;
  if (V == 8) {
    switch (T) {
      case 32: rc = launch<32, 8>(P, grid, s); break;
      default: rc = launch<64, 8>(P, grid, s); break;
    }
  } else {
    switch (T) {
      case 32: rc = launch<32, 16>(P, grid, s); break;
      case 64: rc = launch<64, 16>(P, grid, s); break;
      case 128: rc = launch<128, 16>(P, grid, s); break;
      case 256: rc = launch<256, 16>(P, grid, s); break;
      case 512: rc = launch<512, 16>(P, grid, s); break;
      default: rc = launch<1024, 16>(P, grid, s); break;
    }
  }
  if (rc) return rc;
  dim3 g2((unsigned)ceil_div(cols, 256), P.want_gb ? 4 : 2);
  colsum_kernel<<<g2, 256, 0, s>>>(P.part, da, db, dgamma, dbeta, grid, cols, P.want_gb ? 4 : 2);
  return check_launch("rowfused(colsum)");
}

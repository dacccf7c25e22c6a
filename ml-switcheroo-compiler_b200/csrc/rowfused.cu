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

// Block reductions: shuffle within each warp, then warp 0 combines the NW partials and
// broadcasts the result through shared memory (2 barriers; only one warp does the second
// level). Each reduction site in a row owns a separate shared-memory region, so no third
// barrier is needed to protect the result from the next reduction's partials: a region is
// written again only after later barriers every reader has passed.
template <int NW>
__device__ __forceinline__ float bsum(float v, float* sh) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < NW ? sh[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) sh[32] = t;
  }
  __syncthreads();
  return sh[32];
}
template <int NW>
__device__ __forceinline__ Red2 bsum2(float a, float b, float* sh) {
  a = warp_sum(a);
  b = warp_sum(b);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sh[w] = a;
    sh[32 + w] = b;
  }
  __syncthreads();
  if (w == 0) {
    float ta = lane < NW ? sh[lane] : 0.f, tb = lane < NW ? sh[32 + lane] : 0.f;
    ta = warp_sum(ta);
    tb = warp_sum(tb);
    if (lane == 0) {
      sh[64] = ta;
      sh[65] = tb;
    }
  }
  __syncthreads();
  const Red2 r = {sh[64], sh[65]};
  return r;
}
// max of 64-bit keys (shared by row-max + argmax): key = (order-preserving bits of the
// value) << 32 | ~index, so the largest key is the largest value at the smallest index.
__device__ __forceinline__ unsigned long long order_key(float v, int idx) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)o << 32) | (uint32_t)(~idx);
}
__device__ __forceinline__ float key_value(unsigned long long k) {
  const uint32_t o = (uint32_t)(k >> 32);
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)~(uint32_t)k; }
__device__ __forceinline__ unsigned long long warp_maxkey(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
    k = k2 > k ? k2 : k;
  }
  return k;
}
template <int NW>
__device__ __forceinline__ unsigned long long bmaxkey(unsigned long long k, float* sh) {
  unsigned long long* s64 = reinterpret_cast<unsigned long long*>(sh);
  k = warp_maxkey(k);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) s64[w] = k;
  __syncthreads();
  if (w == 0) {
    unsigned long long t = lane < NW ? s64[lane] : 0ull;
    t = warp_maxkey(t);
    if (lane == 0) s64[32] = t;
  }
  __syncthreads();
  return s64[32];
}
// sum of a float and max of a 64-bit key in one block reduction
template <int NW>
__device__ __forceinline__ void bsum_maxkey(float& v, unsigned long long& k, float* sh) {
  unsigned long long* s64 = reinterpret_cast<unsigned long long*>(sh);
  v = warp_sum(v);
  k = warp_maxkey(k);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    s64[w] = k;        // keys in sh[0 .. 2 NW)
    sh[68 + w] = v;    // sums in sh[68 .. 68 + NW)
  }
  __syncthreads();
  if (w == 0) {
    unsigned long long t = lane < NW ? s64[lane] : 0ull;
    float f = lane < NW ? sh[68 + lane] : 0.f;
    t = warp_maxkey(t);
    f = warp_sum(f);
    if (lane == 0) {
      s64[32] = t;
      sh[66] = f;
    }
  }
  __syncthreads();
  k = s64[32];
  v = sh[66];
}

template <int NW>
__device__ __forceinline__ float bmax(float v, float* sh) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = lane < NW ? sh[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) sh[32] = t;
  }
  __syncthreads();
  const float r = sh[32];
  __syncthreads();
  return r;
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

// T threads, V consecutive columns per thread (cols <= T*V), V/2 packed pairs.
// Registers hold this thread's slice of the column vectors (a, b, gamma, beta, loaded
// once per CTA), the forward tanh t, one working row array w and the column
// accumulators. x and c of the current and the next row sit in this thread's own
// shared-memory slot, prefetched with cp.async one row ahead (double-buffered).
template <int T, int V, bool GB, bool RAGGED>
__global__ void __launch_bounds__(T, (V == 4 ? 1024 : 512) / T > 0 ? (V == 4 ? 1024 : 512) / T : 1) rowfused_kernel(const __grid_constant__ Params P) {
  constexpr int NW = T / 32;
  constexpr int H = V / 2;
  __shared__ __align__(16) float sh[104];       // set-up reductions
  __shared__ __align__(16) float shr[5][104];   // per-row reduction sites
  extern __shared__ __align__(16) float sm[];  // [2 stages][x, c][T][V] (a warp's slices are contiguous)
  const int64_t C = P.cols;
  const int c0 = threadIdx.x * V;
  const bool full = c0 + V <= C;
  const bool vec = full && ((C & 3) == 0);
  const bool any = c0 < C;
  auto msk = [&](int i) -> F2 { return RAGGED ? pk(c0 + 2 * i < C ? 1.f : 0.f, c0 + 2 * i + 1 < C ? 1.f : 0.f) : sp(1.f); };
  auto mul_mask = [&](F2 v, int i) -> F2 { return RAGGED ? mul2(v, msk(i)) : v; };
  const float invC = 1.f / (float)C;
  const float KG2L = 2.f * K_GELU * LOG2E;
  const int64_t G = gridDim.x;

  F2 a[H], b[H], ga[H], be[H];
  ldg_pairs<V>(a, P.a, c0, C, vec, 0.f);
  ldg_pairs<V>(b, P.b, c0, C, vec, 0.f);
  ldg_pairs<V>(ga, P.gamma, c0, C, vec, 1.f);
  ldg_pairs<V>(be, P.beta, c0, C, vec, 0.f);
  // Softmax shift: for n = gamma * x_hat + beta with every gamma >= 0, each row max lies in
  // [min beta, max gamma * sqrt(C) + max beta] (|x_hat| <= sqrt(C), max x_hat >= 0). When
  // that interval is at most 80 wide, exp(n - S) with S its top never overflows and the
  // largest term never underflows, so the per-row max reduction is not needed.
  float shiftS = 0.f;
  bool use_shift;
  {
    float gmin = INFINITY, gmx = -INFINITY, bmn = INFINITY, bmx = -INFINITY;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      float g0, g1, b0, b1;
      upk(ga[i], g0, g1);
      upk(be[i], b0, b1);
      if (c0 + 2 * i < C) { gmin = fminf(gmin, g0); gmx = fmaxf(gmx, g0); bmn = fminf(bmn, b0); bmx = fmaxf(bmx, b0); }
      if (c0 + 2 * i + 1 < C) { gmin = fminf(gmin, g1); gmx = fmaxf(gmx, g1); bmn = fminf(bmn, b1); bmx = fmaxf(bmx, b1); }
    }
    gmin = -bmax<NW>(-gmin, sh);
    gmx = bmax<NW>(gmx, sh);
    bmn = -bmax<NW>(-bmn, sh);
    bmx = bmax<NW>(bmx, sh);
    shiftS = gmx * sqrtf((float)C) + bmx;
    use_shift = gmin >= 0.f && (shiftS - bmn) <= 80.f && isfinite(shiftS);
  }
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
    F2 w[H], t[H];
    // ---- forward: p = x a + b ; t = tanh(k p (1 + c p^2)) ; w = g = 0.5 p (1 + t)
    F2 s2 = sp(0.f), q2 = sp(0.f);
    {
      F2 x[H];
      lds_pairs(xs, x);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 q = fma2(mul2(p, p), sp(C_GELU), sp(1.f));
        t[i] = tanh2_from_scaled(mul2(mul2(p, q), sp(KG2L)));
        const F2 hp = mul2(p, sp(0.5f));
        w[i] = mul_mask(fma2(hp, t[i], hp), i);
        s2 = add2(s2, w[i]);
        q2 = fma2(w[i], w[i], q2);
      }
    }
    float sa, sb, qa, qb;
    upk(s2, sa, sb);
    upk(q2, qa, qb);
    const Red2 SG = bsum2<NW>(sa + sb, qa + qb, shr[0]);
    const float mean = SG.a * invC;
    const float rstd = rsqrtf(fmaxf(SG.b * invC - mean * mean, 0.f) + P.eps);
    const F2 nmr = sp(-mean * rstd), rs = sp(rstd);
    // w = n = LayerNorm(g); row max (skipped on the shift path) with its first index
    float M;
    int jn = 0;
#pragma unroll
    for (int i = 0; i < H; ++i) w[i] = fma2(fma2(w[i], rs, nmr), ga[i], be[i]);
    if (!use_shift) {
      unsigned long long mk = 0ull;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[i], u0, u1);
        if (!RAGGED || c0 + 2 * i < C) {
          const unsigned long long k0 = order_key(u0, c0 + 2 * i);
          mk = k0 > mk ? k0 : mk;
        }
        if (!RAGGED || c0 + 2 * i + 1 < C) {
          const unsigned long long k1 = order_key(u1, c0 + 2 * i + 1);
          mk = k1 > mk ? k1 : mk;
        }
      }
      mk = bmaxkey<NW>(mk, shr[1]);
      M = key_value(mk);
      jn = key_index(mk);  // first index of max(n)
    } else {
      M = shiftS;
    }
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
    const float inv = 1.f / bsum<NW>(sa + sb, shr[2]);
    // w = y ; sum(c*y) ; argmax(y), first max wins
    F2 cy2 = sp(0.f);
    {
      F2 c[H];
      lds_pairs(cs, c);
      const F2 iv = sp(inv);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        w[i] = mul2(w[i], iv);
        cy2 = fma2(c[i], w[i], cy2);
      }
    }
    upk(cy2, sa, sb);
    float cy;
    int yj;
    if (use_shift) {
      // exact argmax of y: its key max travels with the sum of c*y
      unsigned long long yk = 0ull;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[i], u0, u1);
        if (!RAGGED || c0 + 2 * i < C) {
          const unsigned long long k0 = order_key(u0, c0 + 2 * i);
          yk = k0 > yk ? k0 : yk;
        }
        if (!RAGGED || c0 + 2 * i + 1 < C) {
          const unsigned long long k1 = order_key(u1, c0 + 2 * i + 1);
          yk = k1 > yk ? k1 : yk;
        }
      }
      cy = sa + sb;
      bsum_maxkey<NW>(cy, yk, shr[3]);
      yj = key_index(yk);
    } else {
      // argmax(y) is argmax(n) unless rounding made some y beat y[jn]: one block-wide OR
      if (jn >= c0 && jn < c0 + V) {
#pragma unroll
        for (int i = 0; i < H; ++i) {
          float u0, u1;
          upk(w[i], u0, u1);
          if (c0 + 2 * i == jn) shr[3][70] = u0;
          if (c0 + 2 * i + 1 == jn) shr[3][70] = u1;
        }
      }
      cy = bsum<NW>(sa + sb, shr[3]);  // its barriers also publish shr[3][70] = y[jn]
      yj = jn;
      const float ymax = shr[3][70];
      int tie = 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float u0, u1;
        upk(w[i], u0, u1);
        const int j0 = c0 + 2 * i, j1 = j0 + 1;
        if ((!RAGGED || j0 < C) && (j0 < jn ? u0 >= ymax : (j0 > jn && u0 > ymax))) tie = 1;
        if ((!RAGGED || j1 < C) && (j1 < jn ? u1 >= ymax : (j1 > jn && u1 > ymax))) tie = 1;
      }
      if (__syncthreads_or(tie)) {
        unsigned long long yk = 0ull;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          float u0, u1;
          upk(w[i], u0, u1);
          if (!RAGGED || c0 + 2 * i < C) {
            const unsigned long long k0 = order_key(u0, c0 + 2 * i);
            yk = k0 > yk ? k0 : yk;
          }
          if (!RAGGED || c0 + 2 * i + 1 < C) {
            const unsigned long long k1 = order_key(u1, c0 + 2 * i + 1);
            yk = k1 > yk ? k1 : yk;
          }
        }
        yj = key_index(bmaxkey<NW>(yk, shr[1]));
      }
    }
    if (P.am && threadIdx.x == 0) P.am[row] = yj;
    store_row(P.y + row * C, w);
    // ---- backward 1: w = dn = y (c - cy) ; s1 = sum dn gamma ; s2 = sum dn gamma g_hat
    F2 s12 = sp(0.f), s22 = sp(0.f);
    {
      F2 c[H], x[H];
      lds_pairs(cs, c);
      lds_pairs(xs, x);
      const F2 ncy = sp(-cy);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        w[i] = mul2(w[i], add2(c[i], ncy));
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 hp = mul2(p, sp(0.5f));
        const F2 gh = mul_mask(fma2(fma2(hp, t[i], hp), rs, nmr), i);
        const F2 dyg = mul2(w[i], ga[i]);
        s12 = add2(s12, dyg);
        s22 = fma2(dyg, gh, s22);
      }
    }
    float s1a, s1b, s2a, s2b;
    upk(s12, s1a, s1b);
    upk(s22, s2a, s2b);
    const Red2 S = bsum2<NW>(s1a + s1b, s2a + s2b, shr[4]);
    // ---- backward 2: dg, gelu', dp ; dx = dp a ; da += dp x ; db += dp
    {
      F2 x[H], dx[H];
      lds_pairs(xs, x);
      const F2 k1 = sp(rstd * invC), fC = sp((float)C), nS1 = sp(-S.a), nS2 = sp(-S.b);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const F2 p = fma2(x[i], a[i], b[i]);
        const F2 hp = mul2(p, sp(0.5f));
        const F2 gh = mul_mask(fma2(fma2(hp, t[i], hp), rs, nmr), i);
        // dg = rstd/C (C dn gamma - S1 - g_hat S2)
        const F2 dg = mul2(k1, fma2(gh, nS2, fma2(fC, mul2(w[i], ga[i]), nS1)));
        // gelu'(p) = 0.5 (1 + t) + 0.5 k p (1 - t^2) (1 + 3 c p^2)
        const F2 A = fma2(t[i], sp(0.5f), sp(0.5f));
        const F2 sech2 = fma2(t[i], mul2(t[i], sp(-1.f)), sp(1.f));
        const F2 Bq = fma2(mul2(p, p), sp(3.f * C_GELU), sp(1.f));
        const F2 gd = fma2(mul2(mul2(p, sp(0.5f * K_GELU)), sech2), Bq, A);
        const F2 dp = mul_mask(mul2(dg, gd), i);
        dx[i] = mul2(dp, a[i]);
        acc_da[i] = fma2(dp, x[i], acc_da[i]);
        acc_db[i] = add2(acc_db[i], dp);
        if (GB) {
          acc_dg[i] = fma2(w[i], gh, acc_dg[i]);
          acc_dbe[i] = add2(acc_dbe[i], w[i]);
        }
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
  const size_t smem = (size_t)2 * 2 * T * V * sizeof(float);
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
  int T, V;
  shape_for(cols, T, V);
  const int64_t grid = grid_for(rows, cols);
  int rc;
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
  dim3 g2((unsigned)ceil_div(cols, 256), P.want_gb ? 4 : 2);
  colsum_kernel<<<g2, 256, 0, s>>>(P.part, da, db, dgamma, dbeta, grid, cols, P.want_gb ? 4 : 2);
  return check_launch("rowfused(colsum)");
}

// Conv2D forward / input gradient / weight gradient as implicit GEMMs on the tcgen05
// tensor cores: the im2col operand is never materialised in HBM. Producer warps gather
// each 128 x 64 operand tile straight from the fp32 NCHW activations (and the fp32 OIHW
// weights), round it to bf16 and write it into shared memory in the 128-byte swizzled
// K-major layout the UMMA descriptors read; one thread issues tcgen05.mma into a
// double-buffered TMEM accumulator; four epilogue warps write the fp32 result in NCHW
// with the activation / mask fused. Replaces Conv2D (numpy/eager/conv.py:462-489),
// Conv2DInputGrad (conv.py:634-697) and Conv2DWeightGrad (conv.py:699-764); padding is
// _compute_conv2d_padding_values (conv.py:590-633), passed in as (pt, pl).
//
// The three GEMMs (rows M, columns Nc, reduction K; kappa orders taps outermost):
//   fwd   rows = output pixels (n, oh, ow)   cols = o   K = (i, j, c)
//         A[m, k] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]      B[o, k] = w[o, c, i, j]
//         epilogue: y[n, o, oh, ow] = acc  (optionally relu(acc))
//   dgrad rows = input pixels (n, h, w)      cols = c   K = (i, j, o)
//         A[m, k] = dy[n, o, (h + pt - i) / sh, (w + pl - j) / sw]  (0 unless both divide
//                   exactly and land inside the output)           B[c, k] = w[o, c, i, j]
//         epilogue: dx[n, c, h, w] = acc  (optionally acc * (mask[n, c, h, w] > 0): the
//                   ReLU VJP of the layer below)
//   wgrad rows = taps (i, j, c)              cols = o   K = output pixels q = (n, oh, ow),
//         split over CTAs in chunks of 64-multiples
//         A[t, q] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]       B[o, q] = dy[n, o, oh, ow]
//         epilogue: per-split partials [split][o][tap], then a fixed-order sum into
//                   dw[o, c, i, j] (deterministic, no float atomics)
//
// Persistent kernel, one CTA per SM, 416 threads:
//   warps 0-7   producers: gather, round to bf16, st.shared.v4 into the stage ring
//               (16-byte pieces XORed by row & 7: the TMA 128-byte swizzle), then
//               fence.proxy.async and one mbarrier arrival per warp;
//   warp 8      allocates TMEM and issues four 128 x BN x 16 MMAs per 64-wide K block;
//   warps 9-12  epilogue, one TMEM lane quarter each (warp % 4), lane = GEMM row, so a
//               store of one column covers 32 consecutive pixels (coalesced in NCHW).
// Every mbarrier wait is bounded; a warp whose wait gives up stops, and the CTA winds down
// (the MMA warp drains its MMAs before TMEM is freed).
#include <algorithm>

#include "tc_common.cuh"

namespace b200 {
namespace igemm {

using namespace tc;

enum Mode { FWD = 0, DGRAD = 1, WGRAD = 2 };

constexpr int PROD_WARPS = 8, PROD_THREADS = PROD_WARPS * 32;
constexpr int MMA_WARP = PROD_WARPS;
constexpr int THREADS = (PROD_WARPS + 1 + 4) * 32;
constexpr int BM = 128, BK = 64;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr int KTAB_MAX = 2048;          // taps x channels one table holds
constexpr uint32_t SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per CTA

struct Args {
  int N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl;
  int P, HW;                  // OH * OW, H * W
  int M, Nc, K;               // GEMM rows, columns, reduction length (wgrad: N * P)
  int BN, BNT;                // column tile (multiple of 16, <= 256); its TMEM stride (multiple of 32)
  int tiles_m, tiles_n, splits, items;
  int lq;                     // wgrad: reduction elements per split (multiple of 64)
  int ktab;                   // table entries: fwd / dgrad K, wgrad M
  int stages;
  uint32_t stage_bytes;       // A_BYTES + BN * 128
  uint32_t tmem_cols;
  int relu;                   // fwd: relu epilogue
  const float* asrc;          // fwd: x    dgrad: dy   wgrad: x
  const float* bsrc;          // fwd: w    dgrad: w    wgrad: dy
  float* out;                 // fwd: y    dgrad: dx   wgrad: partials [splits][O][M]
  const float* mask;          // dgrad: dx *= (mask > 0) when not null
};

__device__ __forceinline__ uint32_t swz(int r, int j) { return (uint32_t)r * 128u + ((uint32_t)(j ^ (r & 7)) << 4); }

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int sleep_ns) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, sleep_ns);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ float ldf(const float* p) { return __ldg(p); }

// 8 fp32 values -> one 16-byte piece of bf16
__device__ __forceinline__ void put8(uint32_t addr, const float (&v)[8]) {
  st_shared_v4(addr, pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

// item -> (m tile, n tile, split)
__device__ __forceinline__ void item_of(const Args& a, int it, int& mt, int& nt, int& sp) {
  const int per = a.tiles_m * a.tiles_n;
  sp = it / per;
  const int r = it - sp * per;
  mt = r / a.tiles_n;
  nt = r - mt * a.tiles_n;
}
__device__ __forceinline__ int kblocks_of(const Args& a, int sp) {
  if (a.splits == 1 && a.lq == 0) return (a.K + BK - 1) / BK;
  const int q0 = sp * a.lq, q1 = min(a.K, q0 + a.lq);
  return (q1 - q0 + BK - 1) / BK;
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) conv_igemm_kernel(const __grid_constant__ Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sStages = smem;
  int4* tab = reinterpret_cast<int4*>(smem + (uint32_t)a.stages * a.stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(tab + a.ktab);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tap table: fwd {c*HW + i*W + j, i, j, c*KH*KW + t}, kappa = t*C + c
  //            dgrad {o*P, i, j, o*C*KH*KW + t},     kappa = t*O + o
  //            wgrad {c*HW + i*W + j, i, j, 0},      row   = t*C + c
  for (int k = threadIdx.x; k < a.ktab; k += blockDim.x) {
    const int inner = MODE == DGRAD ? a.O : a.C;
    const int t = k / inner, ch = k - t * inner;
    const int i = t / a.KW, j = t - i * a.KW;
    int4 e;
    if (MODE == DGRAD) e = make_int4(ch * a.P, i, j, ch * a.C * a.KH * a.KW + t);
    else e = make_int4(ch * a.HW + i * a.W + j, i, j, ch * a.KH * a.KW + t);
    tab[k] = e;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], PROD_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drained, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(a.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < PROD_WARPS) {
    // ------------------------------------------------------------ producers
    const int pt = threadIdx.x;
    uint32_t L = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      int mt, nt, sp;
      item_of(a, it, mt, nt, sp);
      const int m0 = mt * BM, n0 = nt * a.BN;
      const int nkb = kblocks_of(a, sp);
      if constexpr (MODE != WGRAD) {
        // A: thread = row r, pieces j = half, half + 2, half + 4, half + 6
        const int r = pt & (BM - 1), half = pt >> 7;
        const int m = m0 + r;
        const bool rv = m < a.M;
        int base = 0, hb = 0, wb = 0;
        if (rv) {
          if (MODE == FWD) {
            const int n = m / a.P, p = m - n * a.P, oh = p / a.OW, ow = p - oh * a.OW;
            hb = oh * a.sh - a.pt;
            wb = ow * a.sw - a.pl;
            base = n * a.C * a.HW + hb * a.W + wb;
          } else {
            const int n = m / a.HW, hw = m - n * a.HW, h = hw / a.W, w = hw - h * a.W;
            hb = h + a.pt;
            wb = w + a.pl;
            base = n * a.O * a.P;
          }
        }
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          const int s = (int)(L % (uint32_t)a.stages);
          if (!warp_wait(&empty[s], ((L / (uint32_t)a.stages) & 1) ^ 1, 0)) {
            ok = false;
            break;
          }
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
          const uint32_t sB = sA + A_BYTES;
          float v[32];
#pragma unroll
          for (int ue = 0; ue < 32; ++ue) {
            const int k = kb * BK + (half + 2 * (ue >> 3)) * 8 + (ue & 7);
            float x = 0.f;
            if (rv && k < a.K) {
              const int4 t = tab[k];
              if (MODE == FWD) {
                const int h = hb + t.y, w = wb + t.z;
                if ((unsigned)h < (unsigned)a.H && (unsigned)w < (unsigned)a.W) x = ldf(a.asrc + (base + t.x));
              } else {
                int th = hb - t.y, tw = wb - t.z;
                bool in = th >= 0 && tw >= 0;
                if (a.sh == 2) {
                  in = in && !(th & 1);
                  th >>= 1;
                } else if (a.sh != 1) {
                  const int qq = th / a.sh;
                  in = in && qq * a.sh == th;
                  th = qq;
                }
                if (a.sw == 2) {
                  in = in && !(tw & 1);
                  tw >>= 1;
                } else if (a.sw != 1) {
                  const int qq = tw / a.sw;
                  in = in && qq * a.sw == tw;
                  tw = qq;
                }
                in = in && th < a.OH && tw < a.OW;
                if (in) x = ldf(a.asrc + (base + t.x + th * a.OW + tw));
              }
            }
            v[ue] = x;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            st_shared_v4(sA + swz(r, half + 2 * u), pack_bf16(v[8 * u], v[8 * u + 1]), pack_bf16(v[8 * u + 2], v[8 * u + 3]),
                         pack_bf16(v[8 * u + 4], v[8 * u + 5]), pack_bf16(v[8 * u + 6], v[8 * u + 7]));
          // B: weights, rows = GEMM columns n0 .. n0 + BN
          for (int cid = pt; cid < a.BN * 8; cid += PROD_THREADS) {
            const int rr = cid >> 3, j = cid & 7;
            const int col = n0 + rr;
            float wv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int k = kb * BK + j * 8 + e;
              float x = 0.f;
              if (col < a.Nc && k < a.K) {
                const int4 t = tab[k];
                x = ldf(a.bsrc + (MODE == FWD ? col * a.K + t.w : t.w + col * a.KH * a.KW));
              }
              wv[e] = x;
            }
            put8(sB + swz(rr, j), wv);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      } else {
        // wgrad: piece j = lane & 7 (8 consecutive output pixels q), rows lane >> 3 + 4 * warp + 32 u
        const int j = lane & 7, rsub = (lane >> 3) + 4 * warp;
        const int qs = sp * a.lq, qe = min(a.K, qs + a.lq);
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          const int s = (int)(L % (uint32_t)a.stages);
          if (!warp_wait(&empty[s], ((L / (uint32_t)a.stages) & 1) ^ 1, 0)) {
            ok = false;
            break;
          }
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
          const uint32_t sB = sA + A_BYTES;
          // decode the 8 pixels q0 .. q0 + 7 once
          const int q0 = qs + kb * BK + j * 8;
          int xo[8], hq[8], wq[8], dq[8];
          uint32_t qv = 0;
          {
            int n = q0 / a.P, p = q0 - n * a.P;
            int oh = p / a.OW, ow = p - oh * a.OW;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if (q0 + e < qe) qv |= 1u << e;
              hq[e] = oh * a.sh - a.pt;
              wq[e] = ow * a.sw - a.pl;
              xo[e] = n * a.C * a.HW + hq[e] * a.W + wq[e];
              dq[e] = n * a.O * a.P + p;
              ++p;
              if (++ow == a.OW) {
                ow = 0;
                if (++oh == a.OH) {
                  oh = 0;
                  p = 0;
                  ++n;
                }
              }
            }
          }
          float v[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int row = m0 + rsub + 32 * u;
            const bool rv = row < a.M;
            int4 t = make_int4(0, 0, 0, 0);
            if (rv) t = tab[row];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float x = 0.f;
              if (rv && ((qv >> e) & 1)) {
                const int h = hq[e] + t.y, w = wq[e] + t.z;
                if ((unsigned)h < (unsigned)a.H && (unsigned)w < (unsigned)a.W) x = ldf(a.asrc + (xo[e] + t.x));
              }
              v[u][e] = x;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) put8(sA + swz(rsub + 32 * u, j), v[u]);
          for (int rr = rsub; rr < a.BN; rr += 32) {
            const int o = n0 + rr;
            float dv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) dv[e] = (o < a.Nc && ((qv >> e) & 1)) ? ldf(a.bsrc + (dq[e] + o * a.P)) : 0.f;
            put8(sB + swz(rr, j), dv);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(a.BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      uint32_t L = 0, T = 0;
      bool ok = true, issued = false;
      for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x, ++T) {
        int mt, nt, sp;
        item_of(a, it, mt, nt, sp);
        const int nkb = kblocks_of(a, sp);
        const uint32_t b = T & 1;
        if (!mbar_wait(&acc_empty[b], ((T >> 1) & 1) ^ 1, 32)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + b * (uint32_t)a.BNT;
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          const int s = (int)(L % (uint32_t)a.stages);
          if (!mbar_wait(&full[s], (L / (uint32_t)a.stages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc(sA + k * 32, 16, 1024);
            const uint64_t bd = smem_desc(sA + A_BYTES + k * 32, 16, 1024);
            mma_bf16(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
      // every MMA this thread issued has completed before TMEM can be freed
      if (issued) {
        mma_commit(drained);
        mbar_wait(drained, 0, 32);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    uint32_t T = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x, ++T) {
      int mt, nt, sp;
      item_of(a, it, mt, nt, sp);
      const uint32_t b = T & 1;
      ok = warp_wait(&acc_full[b], (T >> 1) & 1, 64);
      if (!ok) break;
      tc_fence_after();
      const int m = mt * BM + q * 32 + lane;  // this lane's GEMM row
      const bool rv = m < a.M;
      int64_t obase = 0, ostride = 0;
      if (rv) {
        if (MODE == FWD) {
          const int n = m / a.P, p = m - n * a.P;
          obase = (int64_t)n * a.O * a.P + p;
          ostride = a.P;
        } else if (MODE == DGRAD) {
          const int n = m / a.HW, hw = m - n * a.HW;
          obase = (int64_t)n * a.C * a.HW + hw;
          ostride = a.HW;
        } else {
          obase = (int64_t)sp * a.O * a.M + m;
          ostride = a.M;
        }
      }
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + b * (uint32_t)a.BNT;
      const int n0 = nt * a.BN;
      const int ncols = min(a.BN, a.Nc - n0);
      for (int c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t v[32];
        tmem_ld32_issue(tb + (uint32_t)c0, v);
        tmem_wait(v);
        if (c0 + 32 >= ncols) {  // last TMEM read of this item: hand the accumulator back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!rv) continue;
        float* dst = a.out + obase + (int64_t)(n0 + c0) * ostride;
        const int nn = min(32, ncols - c0);
        if (MODE == DGRAD && a.mask != nullptr) {
          const float* mk = a.mask + obase + (int64_t)(n0 + c0) * ostride;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nn) dst[(int64_t)i * ostride] = __uint_as_float(v[i]) * (__ldg(mk + (int64_t)i * ostride) > 0.f ? 1.f : 0.f);
        } else if (MODE == FWD && a.relu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = __uint_as_float(v[i]);
            if (i < nn) dst[(int64_t)i * ostride] = x > 0.f ? x : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nn) dst[(int64_t)i * ostride] = __uint_as_float(v[i]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(a.tmem_cols));
  }
}

// partials [S][O][M] (row = t*C + c) -> dw [O, C, KH, KW], summed over S in order
__global__ void wgrad_reduce_kernel(const float* __restrict__ part, float* __restrict__ dw, int S, int O, int M, int C, int KHW) {
  const int64_t total = (int64_t)O * M;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int o = (int)(e / M), row = (int)(e - (int64_t)o * M);
    float acc = 0.f;
    for (int s = 0; s < S; ++s) acc += part[((int64_t)s * O + o) * M + row];
    const int t = row / C, c = row - t * C;
    dw[((int64_t)o * C + c) * KHW + t] = acc;
  }
}

struct Plan {
  Args a;
  size_t smem;
  bool ok;
  const char* why;
};

// Shapes the kernel handles: 32-bit element offsets (tensors up to 2^30 elements), at most KTAB_MAX
// taps x channels, at most 256 x 255 column tiles.
static Plan plan(int mode, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                 int64_t sh, int64_t sw, int64_t pt, int64_t pl) {
  Plan p{};
  p.ok = false;
  const int64_t lim = (int64_t)1 << 30;
  if (N * C * H * W > lim || N * O * OH * OW > lim || O * C * KH * KW > lim) {
    p.why = "tensor above 2^30 elements";
    return p;
  }
  Args& a = p.a;
  a.N = (int)N, a.C = (int)C, a.H = (int)H, a.W = (int)W, a.O = (int)O, a.KH = (int)KH, a.KW = (int)KW, a.OH = (int)OH,
  a.OW = (int)OW, a.sh = (int)sh, a.sw = (int)sw, a.pt = (int)pt, a.pl = (int)pl;
  a.P = (int)(OH * OW);
  a.HW = (int)(H * W);
  const int64_t taps = KH * KW;
  int64_t M, Nc, K;
  if (mode == FWD) M = N * OH * OW, Nc = O, K = C * taps;
  else if (mode == DGRAD) M = N * H * W, Nc = C, K = O * taps;
  else M = C * taps, Nc = O, K = N * OH * OW;
  const int64_t ktab = mode == WGRAD ? M : K;
  if (ktab > KTAB_MAX) {
    p.why = "more than 2048 taps x channels";
    return p;
  }
  a.M = (int)M, a.Nc = (int)Nc, a.K = (int)K, a.ktab = (int)ktab;
  a.BN = (int)std::min<int64_t>(256, (Nc + 15) / 16 * 16);
  a.BNT = (a.BN + 31) / 32 * 32;
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * a.BNT)) cols <<= 1;
  a.tmem_cols = cols;
  a.tiles_m = (int)ceil_div(M, BM);
  a.tiles_n = (int)ceil_div(Nc, a.BN);
  if (a.tiles_n > 255) {
    p.why = "too many column tiles";
    return p;
  }
  const int sms = num_sms();
  if (mode == WGRAD) {
    // split the pixel reduction so that about two items per SM exist
    const int64_t kblocks = ceil_div(K, BK);
    const int64_t per = (int64_t)a.tiles_m * a.tiles_n;
    int64_t S = std::max<int64_t>(1, std::min<int64_t>(kblocks, ceil_div(2 * (int64_t)sms, per)));
    const int64_t kb_per = ceil_div(kblocks, S);
    a.lq = (int)(kb_per * BK);
    S = ceil_div(K, (int64_t)a.lq);
    a.splits = (int)S;
  } else {
    a.splits = 1;
    a.lq = 0;
  }
  const int64_t items = (int64_t)a.tiles_m * a.tiles_n * a.splits;
  if (items > lim) {
    p.why = "too many tiles";
    return p;
  }
  a.items = (int)items;
  a.stage_bytes = A_BYTES + (uint32_t)a.BN * 128u;
  const size_t fixed = 1024 + (size_t)a.ktab * 16 + 64 * 8 + 16;
  int st = (int)std::min<size_t>(8, (SMEM_LIMIT - fixed) / a.stage_bytes);
  if (st < 2) {
    p.why = "shared memory";
    return p;
  }
  a.stages = st;
  p.smem = fixed + (size_t)st * a.stage_bytes;
  p.ok = true;
  return p;
}

template <int MODE>
static int launch(Args a, size_t smem, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(conv_igemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const unsigned grid = (unsigned)std::max(1, std::min(a.items, num_sms()));
  conv_igemm_kernel<MODE><<<grid, THREADS, smem, s>>>(a);
  return check_launch("conv2d(implicit GEMM)");
}

static int check_dims(int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                      int64_t sh, int64_t sw, int64_t pt, int64_t pl) {
  B200_REQUIRE(N >= 0 && C >= 1 && H >= 1 && W >= 1 && O >= 1 && KH >= 1 && KW >= 1 && OH >= 1 && OW >= 1,
               "conv2d(implicit GEMM): bad sizes");
  B200_REQUIRE(sh >= 1 && sw >= 1 && pt >= 0 && pl >= 0, "conv2d(implicit GEMM): bad stride/padding");
  return B200_OK;
}

}  // namespace igemm
}  // namespace b200

using namespace b200;
using namespace b200::igemm;

extern "C" int b200_conv2d_igemm_supported(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW,
                                           int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl) {
  if (op < 0 || op > 2 || N < 1) return 0;
  if (check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl) != B200_OK) return 0;
  return plan(op, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl).ok ? 1 : 0;
}

extern "C" size_t b200_conv2d_wgrad_igemm_workspace_bytes(int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH,
                                                          int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                                                          int64_t pl) {
  if (N < 1) return 0;
  Plan p = plan(WGRAD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) return 0;
  return (size_t)p.a.splits * (size_t)O * (size_t)p.a.M * 4;
}

extern "C" int b200_conv2d_fwd_igemm(const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                                     int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                     int64_t pt, int64_t pl, int relu, void* stream) {
  int rc = check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(x && w && y, "conv2d_fwd_igemm: null pointer");
  Plan p = plan(FWD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) {
    set_error("conv2d_fwd_igemm: unsupported shape (%s)", p.why);
    return B200_ERR_UNSUPPORTED;
  }
  p.a.relu = relu ? 1 : 0;
  p.a.asrc = x, p.a.bsrc = w, p.a.out = y, p.a.mask = nullptr;
  return launch<FWD>(p.a, p.smem, as_stream(stream));
}

extern "C" int b200_conv2d_dgrad_igemm(const float* dy, const float* w, const float* mask, float* dx, int64_t N, int64_t C,
                                       int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                                       int64_t sh, int64_t sw, int64_t pt, int64_t pl, void* stream) {
  int rc = check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(dy && w && dx, "conv2d_dgrad_igemm: null pointer");
  Plan p = plan(DGRAD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) {
    set_error("conv2d_dgrad_igemm: unsupported shape (%s)", p.why);
    return B200_ERR_UNSUPPORTED;
  }
  p.a.relu = 0;
  p.a.asrc = dy, p.a.bsrc = w, p.a.out = dx, p.a.mask = mask;
  return launch<DGRAD>(p.a, p.smem, as_stream(stream));
}

extern "C" int b200_conv2d_wgrad_igemm(const float* x, const float* dy, float* dw, int64_t N, int64_t C, int64_t H, int64_t W,
                                       int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                       int64_t pt, int64_t pl, void* ws, size_t ws_bytes, void* stream) {
  int rc = check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (rc) return rc;
  B200_REQUIRE(x && dy && dw, "conv2d_wgrad_igemm: null pointer");
  cudaStream_t s = as_stream(stream);
  if (N == 0) {
    cudaMemsetAsync(dw, 0, (size_t)O * C * KH * KW * 4, s);
    return check_launch("conv2d_wgrad_igemm(empty)");
  }
  Plan p = plan(WGRAD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) {
    set_error("conv2d_wgrad_igemm: unsupported shape (%s)", p.why);
    return B200_ERR_UNSUPPORTED;
  }
  const size_t need = (size_t)p.a.splits * (size_t)O * (size_t)p.a.M * 4;
  B200_REQUIRE(ws && ws_bytes >= need, "conv2d_wgrad_igemm: workspace %zu < %zu", ws_bytes, need);
  p.a.relu = 0;
  p.a.asrc = x, p.a.bsrc = dy, p.a.out = reinterpret_cast<float*>(ws), p.a.mask = nullptr;
  rc = launch<WGRAD>(p.a, p.smem, s);
  if (rc) return rc;
  const int64_t total = O * (int64_t)p.a.M;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)num_sms() * 8));
  wgrad_reduce_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float*>(ws), dw, p.a.splits, (int)O, p.a.M, (int)C,
                                           (int)(KH * KW));
  return check_launch("conv2d_wgrad_igemm(sum)");
}

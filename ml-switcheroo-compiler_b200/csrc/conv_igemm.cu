// Conv2D forward / input gradient / weight gradient as implicit GEMMs on the tcgen05
// tensor cores: the im2col operand is never materialised in HBM. Producer warps gather
// each 128 x 64 operand tile straight from the fp32 NCHW activations, round it to bf16
// and write it into shared memory in the 128-byte swizzled K-major layout the UMMA
// descriptors read; one thread issues tcgen05.mma into a double-buffered TMEM
// accumulator; four epilogue warps write the fp32 result in NCHW with the activation /
// mask fused. Replaces Conv2D (numpy/eager/conv.py:462-489), Conv2DInputGrad
// (conv.py:634-697) and Conv2DWeightGrad (conv.py:699-764); padding is
// _compute_conv2d_padding_values (conv.py:590-633), passed in as (pt, pl).
//
// The three GEMMs (rows M, columns Nc, reduction K; the reduction index runs over taps
// outermost):
//   fwd   rows = output pixels (n, oh, ow)   cols = o   K = (i, j, c)
//         A[m, k] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]      B[o, k] = w[o, c, i, j]
//         epilogue: y = acc, or relu(acc)
//   dgrad rows = input pixels (n, h, w) of one stride-parity class (h % sh, w % sw): only
//         the taps with i = (h + pt) mod sh and j = (w + pl) mod sw reach such a pixel, so
//         each class is a dense GEMM over its own taps (at stride 2 a quarter of the taps)
//         cols = c   K = (class taps, o)
//         A[m, k] = dy[n, o, (h + pt - i) / sh, (w + pl - j) / sw]   B[c, k] = w[o, c, i, j]
//         epilogue: dx = acc, or acc * (mask > 0) (the ReLU VJP of the layer below)
//   wgrad rows = taps (i, j, c)              cols = o   K = output pixels q = (n, oh, ow),
//         split over CTAs in multiples of 64
//         A[t, q] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]       B[o, q] = dy[n, o, oh, ow]
//         epilogue: per-split partials [split][o][tap], then a fixed-order sum into
//         dw[o, c, i, j] (deterministic, no float atomics)
//
// Persistent kernel, one CTA per SM, 416 threads:
//   warps 0-7   producers. fwd / dgrad: two groups of four warps take alternate 64-wide
//               K blocks (two blocks in flight per SM); a thread owns one tile row and
//               gathers its 64 values with clamped, unconditional loads (a masked-off
//               element reads the tensor's first element and is replaced by zero), so all
//               64 loads are in flight together. The weights (B) are gathered once per CTA
//               into shared memory and stay resident. wgrad: one group of eight warps
//               gathers A and B of each block. Pieces of 16 bytes are XORed by row & 7 (the
//               TMA 128-byte swizzle); then fence.proxy.async and one mbarrier arrival per
//               warp;
//   warp 8      allocates TMEM and issues four 128 x BN x 16 MMAs per K block;
//   warps 9-12  epilogue, one TMEM lane quarter each (warp % 4), lane = GEMM row, so a
//               store of one column covers 32 consecutive pixels.
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
constexpr int MAX_CLS = 16;             // stride-parity classes of the input gradient (sh * sw)
constexpr uint32_t SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per CTA

struct Args {
  int N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl;
  int P, HW;                  // OH * OW, H * W
  int M, Nc, K;               // fwd / wgrad: GEMM rows, columns, reduction length (wgrad: N * P)
  int BN, BNT;                // column tile (multiple of 16, <= 256); its TMEM stride (multiple of 32)
  int tiles_n, splits, items;
  int lq;                     // wgrad: reduction elements per split (multiple of 64)
  int ktab;                   // table entries
  int stages;
  uint32_t stage_bytes;       // fwd / dgrad: A_BYTES; wgrad: A_BYTES + BN * 128
  uint32_t resb_off;          // fwd / dgrad: byte offset of the resident B operand
  int kb_total;               // fwd / dgrad: K blocks over all classes
  uint32_t tmem_cols;
  int relu;                   // fwd: relu epilogue
  // classes: fwd / wgrad one (the whole GEMM); dgrad sh * sw parity classes
  int ncls, max_tiles;        // item = (tile * ncls + class) * tiles_n + column tile
  int cls_ph[MAX_CLS], cls_pw[MAX_CLS];
  int cls_hc[MAX_CLS], cls_wc[MAX_CLS];  // dgrad: rows and columns of the class per image
  int cls_m[MAX_CLS];         // GEMM rows of the class
  int cls_k[MAX_CLS];         // reduction length of the class
  int cls_ktab[MAX_CLS];      // first table entry
  int cls_kb[MAX_CLS];        // first K block in the resident B operand
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

__device__ __forceinline__ void put8(uint32_t addr, const float* v) {
  st_shared_v4(addr, pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

// item -> class, row tile, column tile, split; false for an empty slot (a class with fewer
// tiles than the largest). Every role walks the same items and skips the same slots.
struct Item {
  int cls, mt, nt, sp;
};
__device__ __forceinline__ bool item_of(const Args& a, int it, Item& r) {
  const int per = a.max_tiles * a.ncls * a.tiles_n;
  r.sp = it / per;
  int x = it - r.sp * per;
  r.nt = x % a.tiles_n;
  x /= a.tiles_n;
  r.cls = x % a.ncls;
  r.mt = x / a.ncls;
  return r.mt * BM < a.cls_m[r.cls];
}
__device__ __forceinline__ int kblocks_of(const Args& a, const Item& r) {
  if (a.lq == 0) return (a.cls_k[r.cls] + BK - 1) / BK;
  const int q0 = r.sp * a.lq, q1 = min(a.K, q0 + a.lq);
  return (q1 - q0 + BK - 1) / BK;
}

// fwd / dgrad: the A element of a row (base offset, position hb / wb) and reduction
// index k of its class (table entry {offset, dh, dw, B offset}), bounds-checked against
// the source image (x for fwd, dy for dgrad); a masked-off element loads asrc[0]
template <int MODE>
__device__ __forceinline__ float gather_a(const Args& a, const int4* tab, bool rv, int base, int hb, int wb, int k, int kend) {
  const int4 t = tab[min(k, kend - 1)];
  const int h = hb + t.y, w = wb + t.z;
  const int HH = MODE == FWD ? a.H : a.OH, WW = MODE == FWD ? a.W : a.OW;
  const bool ok = rv && k < kend && (unsigned)h < (unsigned)HH && (unsigned)w < (unsigned)WW;
  const float x = __ldg(a.asrc + (ok ? base + t.x : 0));
  return ok ? x : 0.f;
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) conv_igemm_kernel(const __grid_constant__ Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sStages = smem;
  uint8_t* sResB = smem + a.resb_off;
  int4* tab = reinterpret_cast<int4*>(smem + a.resb_off + (MODE == WGRAD ? 0u : (uint32_t)a.kb_total * a.tiles_n * a.BN * 128u));
  uint64_t* full = reinterpret_cast<uint64_t*>(tab + a.ktab);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int GROUPS = MODE == WGRAD ? 1 : 2;  // producer groups taking alternate K blocks
  constexpr int GROUP_WARPS = PROD_WARPS / GROUPS;

  // Tables (entry per reduction index k of each class):
  //   fwd   k = t*C + c:               {c*HW + i*W + j, i, j, c*KH*KW + t}
  //   dgrad class (ph, pw), k = u*O + o over the class taps u = (i, j):
  //                                    {o*P + dh*OW + dw, dh, dw, o*C*KH*KW + i*KW + j}
  //                                    dh = (ph + pt - i) / sh (exact), dw likewise
  //   wgrad row = t*C + c:             {c*HW + i*W + j, i, j, 0}
  if (MODE == DGRAD) {
    for (int c = 0; c < a.ncls; ++c) {
      const int ph = a.cls_ph[c], pw = a.cls_pw[c];
      const int i0 = (ph + a.pt) % a.sh, j0 = (pw + a.pl) % a.sw;
      const int nj = (a.KW - j0 + a.sw - 1) / a.sw;
      for (int k = threadIdx.x; k < a.cls_k[c]; k += blockDim.x) {
        const int u = k / a.O, o = k - u * a.O;
        const int ui = u / nj, uj = u - ui * nj;
        const int i = i0 + ui * a.sh, j = j0 + uj * a.sw;
        const int dh = (ph + a.pt - i) / a.sh, dw = (pw + a.pl - j) / a.sw;
        tab[a.cls_ktab[c] + k] = make_int4(o * a.P + dh * a.OW + dw, dh, dw, o * a.C * a.KH * a.KW + i * a.KW + j);
      }
    }
  } else {
    for (int k = threadIdx.x; k < a.ktab; k += blockDim.x) {
      const int t = k / a.C, ch = k - t * a.C;
      const int i = t / a.KW, j = t - i * a.KW;
      tab[k] = make_int4(ch * a.HW + i * a.W + j, i, j, ch * a.KH * a.KW + t);
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], GROUP_WARPS);
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

  if constexpr (MODE != WGRAD) {
    // resident B: [K blocks of all classes][column tiles][BN rows x 64] bf16, gathered once.
    // A pass keeps 8 pieces per thread in flight (64 loads), then stores them.
    if (warp < PROD_WARPS) {
      const int pieces_per_kb = a.tiles_n * a.BN * 8;
      const int total = a.kb_total * pieces_per_kb;
      const int KHW = a.KH * a.KW;
      for (int p0 = threadIdx.x; p0 < total; p0 += 8 * PROD_THREADS) {
        float v[64];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int p = min(p0 + u * PROD_THREADS, total - 1);
          const int kbg = p / pieces_per_kb, rem = p - kbg * pieces_per_kb;
          const int col = rem >> 3, j = rem & 7;  // column over all column tiles
          int c = 0;
          while (c + 1 < a.ncls && a.cls_kb[c + 1] <= kbg) ++c;
          const int kk0 = (kbg - a.cls_kb[c]) * BK + j * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int k = kk0 + e;
            const int4 t = tab[a.cls_ktab[c] + min(k, a.cls_k[c] - 1)];
            const bool ok = col < a.Nc && k < a.cls_k[c];
            const float x = __ldg(a.bsrc + (ok ? (MODE == FWD ? col * a.K + t.w : t.w + col * KHW) : 0));
            v[u * 8 + e] = ok ? x : 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int p = p0 + u * PROD_THREADS;
          if (p < total) {
            const int kbg = p / pieces_per_kb, rem = p - kbg * pieces_per_kb;
            const int col = rem >> 3, j = rem & 7;
            const int nt = col / a.BN, rr = col - nt * a.BN;
            put8(smem_u32(sResB) + (uint32_t)((kbg * a.tiles_n + nt) * a.BN) * 128u + swz(rr, j), &v[u * 8]);
          }
        }
      }
      fence_proxy_async_smem();
    }
    __syncthreads();
  }

  if (warp < PROD_WARPS) {
    // ------------------------------------------------------------ producers
    const int grp = warp / GROUP_WARPS, gw = warp % GROUP_WARPS;
    uint32_t L = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      Item r;
      if (!item_of(a, it, r)) continue;
      const int m0 = r.mt * BM, n0 = r.nt * a.BN;
      const int nkb = kblocks_of(a, r);
      if constexpr (MODE != WGRAD) {
        // A: thread = tile row, all 8 pieces of it
        const int row = threadIdx.x & (BM - 1);
        const int m = m0 + row;
        const bool rv = m < a.cls_m[r.cls];
        const int mm = rv ? m : 0;
        int base, hb, wb;
        if (MODE == FWD) {
          const int n = mm / a.P, p = mm - n * a.P, oh = p / a.OW, ow = p - oh * a.OW;
          hb = oh * a.sh - a.pt;
          wb = ow * a.sw - a.pl;
          base = n * a.C * a.HW + hb * a.W + wb;
        } else {
          const int hc = a.cls_hc[r.cls], wc = a.cls_wc[r.cls];
          const int n = mm / (hc * wc), rem = mm - n * (hc * wc), hh = rem / wc, ww = rem - hh * wc;
          hb = hh;
          wb = ww;
          base = n * a.O * a.P + hh * a.OW + ww;
        }
        const int4* ctab = tab + a.cls_ktab[r.cls];
        const int kend = a.cls_k[r.cls];
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          if ((int)(L % GROUPS) != grp) continue;
          const int s = (int)(L % (uint32_t)a.stages);
          if (!warp_wait(&empty[s], ((L / (uint32_t)a.stages) & 1) ^ 1, 0)) {
            ok = false;
            break;
          }
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
          float v[64];
#pragma unroll
          for (int e = 0; e < 64; ++e) v[e] = gather_a<MODE>(a, ctab, rv, base, hb, wb, kb * BK + e, kend);
#pragma unroll
          for (int j = 0; j < 8; ++j) put8(sA + swz(row, j), &v[8 * j]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      } else {
        // wgrad: piece j = lane & 7 (8 consecutive output pixels q), rows (lane >> 3) + 4 warp + 32 u
        const int j = lane & 7, rsub = (lane >> 3) + 4 * gw;
        const int qs = r.sp * a.lq, qe = min(a.K, qs + a.lq);
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
          float v[32], dv[32];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int row = m0 + rsub + 32 * u;
            const bool rv = row < a.M;
            const int4 t = tab[min(row, a.M - 1)];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int h = hq[e] + t.y, w = wq[e] + t.z;
              const bool okk = rv && ((qv >> e) & 1) && (unsigned)h < (unsigned)a.H && (unsigned)w < (unsigned)a.W;
              const float x = __ldg(a.asrc + (okk ? xo[e] + t.x : 0));
              v[u * 8 + e] = okk ? x : 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int o = n0 + rsub + 32 * u;
            const bool ov = rsub + 32 * u < a.BN && o < a.Nc;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const bool okk = ov && ((qv >> e) & 1);
              const float x = __ldg(a.bsrc + (okk ? dq[e] + o * a.P : 0));
              dv[u * 8 + e] = okk ? x : 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) put8(sA + swz(rsub + 32 * u, j), &v[8 * u]);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (rsub + 32 * u < a.BN) put8(sB + swz(rsub + 32 * u, j), &dv[8 * u]);
          // B rows beyond 128 (BN > 128): a second pass
          for (int rr = rsub + 128; rr < a.BN; rr += 32) {
            const int o = n0 + rr;
            float ev[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const bool okk = o < a.Nc && ((qv >> e) & 1);
              const float x = __ldg(a.bsrc + (okk ? dq[e] + o * a.P : 0));
              ev[e] = okk ? x : 0.f;
            }
            put8(sB + swz(rr, j), ev);
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
      for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
        Item r;
        if (!item_of(a, it, r)) continue;
        const int nkb = kblocks_of(a, r);
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
          const uint32_t sB = MODE == WGRAD ? sA + A_BYTES
                                            : smem_u32(sResB) + (uint32_t)(((a.cls_kb[r.cls] + kb) * a.tiles_n + r.nt) * a.BN) * 128u;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = smem_desc(sA + k * 32, 16, 1024);
            const uint64_t bd = smem_desc(sB + k * 32, 16, 1024);
            mma_bf16(d, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
        ++T;
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
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      Item r;
      if (!item_of(a, it, r)) continue;
      const uint32_t b = T & 1;
      ok = warp_wait(&acc_full[b], (T >> 1) & 1, 64);
      ++T;
      if (!ok) break;
      tc_fence_after();
      const int m = r.mt * BM + q * 32 + lane;  // this lane's GEMM row
      const bool rv = m < a.cls_m[r.cls];
      int64_t obase, ostride;
      {
        const int mm = rv ? m : 0;
        if (MODE == FWD) {
          const int n = mm / a.P, p = mm - n * a.P;
          obase = (int64_t)n * a.O * a.P + p;
          ostride = a.P;
        } else if (MODE == DGRAD) {
          const int hc = a.cls_hc[r.cls], wc = a.cls_wc[r.cls];
          const int n = mm / (hc * wc), rem = mm - n * (hc * wc), hh = rem / wc, ww = rem - hh * wc;
          const int h = a.cls_ph[r.cls] + a.sh * hh, w = a.cls_pw[r.cls] + a.sw * ww;
          obase = (int64_t)n * a.C * a.HW + h * a.W + w;
          ostride = a.HW;
        } else {
          obase = (int64_t)r.sp * a.O * a.M + mm;
          ostride = a.M;
        }
      }
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + b * (uint32_t)a.BNT;
      const int n0 = r.nt * a.BN;
      const int ncols = min(a.BN, a.Nc - n0);
      for (int c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t v[32];
        tmem_ld32_issue(tb + (uint32_t)c0, v);
        const int nn = min(32, ncols - c0);
        float* __restrict__ dst = a.out + obase + (int64_t)(n0 + c0) * ostride;
        float mv[32];
        if (MODE == DGRAD && a.mask != nullptr) {
          // the chunk's 32 mask values are all loaded before its first store
          const float* __restrict__ mk = a.mask + obase + (int64_t)(n0 + c0) * ostride;
#pragma unroll
          for (int i = 0; i < 32; ++i) mv[i] = __ldg(mk + (rv && i < nn ? (int64_t)i * ostride : 0));
        }
        tmem_wait(v);
        if (c0 + 32 >= ncols) {  // last TMEM read of this item: hand the accumulator back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!rv) continue;
        if (MODE == DGRAD && a.mask != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nn) dst[(int64_t)i * ostride] = __uint_as_float(v[i]) * (mv[i] > 0.f ? 1.f : 0.f);
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

// Shapes the kernel handles: 32-bit element offsets (tensors up to 2^30 elements), at most
// KTAB_MAX taps x channels, at most 16 stride-parity classes, and (fwd / dgrad) the whole
// bf16 weight operand resident in shared memory beside two A stages.
static Plan plan(int mode, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                 int64_t sh, int64_t sw, int64_t pt, int64_t pl) {
  Plan p{};
  p.ok = false;
  const int64_t lim = (int64_t)1 << 30;
  if (N * C * H * W > lim || N * O * OH * OW > lim || O * C * KH * KW > lim) {
    p.why = "tensor above 2^30 elements";
    return p;
  }
  if (mode == DGRAD && sh * sw > MAX_CLS) {
    p.why = "stride above the parity-class limit";
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
  a.tiles_n = (int)ceil_div(Nc, a.BN);
  int64_t max_tiles = 0;
  if (mode == DGRAD) {
    a.ncls = (int)(sh * sw);
    int koff = 0, kboff = 0;
    for (int c = 0; c < a.ncls; ++c) {
      const int ph = (int)(c / sw), pw = (int)(c % sw);
      const int hc = ph < H ? (int)ceil_div(H - ph, sh) : 0, wc = pw < W ? (int)ceil_div(W - pw, sw) : 0;
      const int i0 = (int)((ph + pt) % sh), j0 = (int)((pw + pl) % sw);
      const int ni = i0 < KH ? (int)ceil_div(KH - i0, sh) : 0, nj = j0 < KW ? (int)ceil_div(KW - j0, sw) : 0;
      a.cls_ph[c] = ph, a.cls_pw[c] = pw, a.cls_hc[c] = hc, a.cls_wc[c] = wc;
      a.cls_k[c] = (int)(O * ni * nj);
      a.cls_m[c] = a.cls_k[c] > 0 ? (int)(N * hc * wc) : 0;  // pixels no tap reaches are zero-filled by the caller
      a.cls_ktab[c] = koff;
      a.cls_kb[c] = kboff;
      koff += a.cls_k[c];
      kboff += (int)ceil_div(a.cls_k[c], BK);
      max_tiles = std::max<int64_t>(max_tiles, ceil_div(a.cls_m[c], BM));
    }
    a.kb_total = kboff;
  } else {
    a.ncls = 1;
    a.cls_ph[0] = a.cls_pw[0] = 0;
    a.cls_hc[0] = a.cls_wc[0] = 1;
    a.cls_m[0] = (int)M;
    a.cls_k[0] = (int)(mode == WGRAD ? 0 : K);
    a.cls_ktab[0] = 0;
    a.cls_kb[0] = 0;
    a.kb_total = mode == WGRAD ? 0 : (int)ceil_div(K, BK);
    max_tiles = ceil_div(M, BM);
  }
  a.max_tiles = (int)max_tiles;
  if (a.tiles_n > 255 || max_tiles < 1) {
    p.why = "tile count";
    return p;
  }
  const int sms = num_sms();
  if (mode == WGRAD) {
    // split the pixel reduction so that about two items per SM exist
    const int64_t kblocks = ceil_div(K, BK);
    const int64_t per = max_tiles * a.tiles_n;
    int64_t S = std::max<int64_t>(1, std::min<int64_t>(kblocks, ceil_div(2 * (int64_t)sms, per)));
    const int64_t kb_per = ceil_div(kblocks, S);
    a.lq = (int)(kb_per * BK);
    S = ceil_div(K, (int64_t)a.lq);
    a.splits = (int)S;
  } else {
    a.splits = 1;
    a.lq = 0;
  }
  const int64_t items = max_tiles * a.ncls * a.tiles_n * a.splits;
  if (items > lim) {
    p.why = "too many tiles";
    return p;
  }
  a.items = (int)items;
  size_t resb = 0;
  if (mode == WGRAD) {
    a.stage_bytes = A_BYTES + (uint32_t)a.BN * 128u;
  } else {
    a.stage_bytes = A_BYTES;
    resb = (size_t)a.kb_total * a.tiles_n * a.BN * 128;
  }
  const size_t fixed = 1024 + resb + (size_t)a.ktab * 16 + 64 * 8 + 16;
  if (fixed + 2 * (size_t)a.stage_bytes > SMEM_LIMIT) {
    p.why = "shared memory (weights too large to stay resident)";
    return p;
  }
  const int st = (int)std::min<size_t>(8, (SMEM_LIMIT - fixed) / a.stage_bytes);
  a.stages = st;
  a.resb_off = (uint32_t)st * a.stage_bytes;
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
  cudaStream_t s = as_stream(stream);
  // pixels that no tap reaches (a class without taps: stride above the kernel size) are zero
  for (int c = 0; c < p.a.ncls; ++c)
    if (p.a.cls_k[c] == 0) {
      cudaMemsetAsync(dx, 0, (size_t)N * C * H * W * 4, s);
      if ((rc = check_launch("conv2d_dgrad_igemm(zero)"))) return rc;
      break;
    }
  p.a.relu = 0;
  p.a.asrc = dy, p.a.bsrc = w, p.a.out = dx, p.a.mask = mask;
  return launch<DGRAD>(p.a, p.smem, s);
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

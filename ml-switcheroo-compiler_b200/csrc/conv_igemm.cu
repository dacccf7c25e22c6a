// Conv2D forward / input gradient / weight gradient as implicit GEMMs on the tcgen05
// tensor cores: the im2col operand is never materialised in HBM. Operand tiles are built
// in shared memory in the 128-byte swizzled K-major layout the UMMA descriptors read; one
// thread issues tcgen05.mma into up to four TMEM accumulators; eight epilogue warps
// write the fp32 result in NCHW with the activation / mask fused. Replaces Conv2D
// (numpy/eager/conv.py:462-489), Conv2DInputGrad (conv.py:634-697) and Conv2DWeightGrad
// (conv.py:699-764); padding is _compute_conv2d_padding_values (conv.py:590-633), passed
// in as (pt, pl).
//
// The three GEMMs (rows M, columns Nc, reduction K):
//   fwd   rows = output pixels (n, oh, ow)   cols = o   K = (i, j, c), c padded to Cp = 8k
//         A[m, k] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]      B[o, k] = w[o, c, i, j]
//         epilogue: y = acc, or relu(acc)
//   dgrad rows = input pixels (n, h, w) of one stride-parity class (h % sh, w % sw): only
//         the taps with i = (h + pt) mod sh and j = (w + pl) mod sw reach such a pixel, so
//         each class is a dense GEMM over its own taps (at stride 2 a quarter of the taps)
//         cols = c   K = (class taps, o), o padded to Op = 8k
//         A[m, k] = dy[n, o, (h + pt - i) / sh, (w + pl - j) / sw]   B[c, k] = w[o, c, i, j]
//         epilogue: dx = acc, or acc * (mask > 0) (the ReLU VJP of the layer below)
//   wgrad rows = taps (i, j, c), c padded to Cp  cols = o   K = output pixels q = (n, oh, ow),
//         split over CTAs in multiples of 64
//         A[t, q] = x[n, c, oh*sh - pt + i, ow*sw - pl + j]       B[o, q] = dy[n, o, oh, ow]
//         epilogue: per-split partials [split][o][tap], then a fixed-order sum into
//         dw[o, c, i, j] (deterministic, no float atomics)
//
// fwd / dgrad: a repack kernel first writes the source (x, or dy) as bf16 NHWC with the
// channels padded to a multiple of 8 into the caller's workspace, so 8 consecutive
// reduction indices of one tap are 16 contiguous bytes. Each producer warp then builds a
// whole 128 x 64 A tile with 16-byte cp.async copies (zero-filled where a tap falls
// outside the image), waits for its own copies, and arrives on the stage's barrier; each
// producer warp owns one stage and the warps take K blocks round-robin, so up to seven
// tiles are in flight per SM. The weights (B) are gathered once per CTA into shared memory
// and stay resident.
// wgrad: x and dy both get channels-last bf16 copies (dy's channels padded to 64); the
// pixel index is the GEMM's K, so both operands are MN-major tiles: for each of the 64
// pixels of a K block, 128-byte rows of 64 GEMM rows (taps x channels) of A and of 64
// output channels of B, copied by the same one-warp-per-stage cp.async producers.
//
// Persistent kernel, one CTA per SM, 512 threads: warps 0-6 producers, warp 7 allocates
// TMEM and issues four 128 x BN x 16 MMAs per K block into accumulator T % 4 (T % 2 for
// tiles over 128 columns), warps 8-15 epilogue in two groups of four on alternate tiles
// (warp % 4 = TMEM lane quarter, all column chunks of it; lane = GEMM row, so a store of one
// column covers 32 consecutive pixels): two tiles drain at once while the MMA runs ahead. Pieces of 16 bytes are XORed by row & 7 (the TMA 128-byte
// swizzle). Every mbarrier wait is bounded; a warp whose wait gives up stops, and the CTA
// winds down (the MMA warp drains its MMAs before TMEM is freed).
#include <algorithm>

#include "tc_common.cuh"

namespace b200 {
namespace igemm {

using namespace tc;

enum Mode { FWD = 0, DGRAD = 1, WGRAD = 2 };

// seven producer warps, the MMA warp and eight epilogue warps: 16 warps, four per SM
// sub-partition, so each thread may hold 128 registers
constexpr int PROD_WARPS = 7, PROD_THREADS = PROD_WARPS * 32;
constexpr int MMA_WARP = PROD_WARPS;
constexpr int EPI_WARPS = 8;  // two groups of four (one per TMEM lane quarter), on alternate tiles
constexpr int THREADS = (PROD_WARPS + 1 + EPI_WARPS) * 32;
constexpr int BM = 128, BK = 64;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr int KTAB_MAX = 2048;          // reduction indices (fwd / dgrad) or taps x channels (wgrad) one table holds
constexpr int MAX_CLS = 16;             // stride-parity classes of the input gradient (sh * sw)
constexpr uint32_t SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per CTA

struct Args {
  int N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl;
  int P, HW;                  // OH * OW, H * W
  int M, Nc, K;               // GEMM rows, columns, reduction length (wgrad: N * P; fwd: taps * Cp)
  int CP;                     // fwd / wgrad: Cp, dgrad: Op (channels of the NHWC x or dy copy, a multiple of 8)
  int OPW;                    // wgrad: channels of the NHWC dy copy (O padded to a multiple of 64)
  int BN, BNT;                // column tile (multiple of 16, <= 256); its TMEM stride (multiple of 32)
  int tiles_n, splits, items;
  int lq;                     // wgrad: reduction elements per split (multiple of 64)
  int ktab;                   // table entries (fwd / dgrad: 8-element chunks; wgrad: tap rows)
  int stages;
  uint32_t stage_bytes;       // fwd / dgrad: A_BYTES; wgrad: A_BYTES + BN * 128
  uint32_t resb_off;          // fwd / dgrad: byte offset of the resident B operand
  int kb_total;               // fwd / dgrad: K blocks over all classes
  uint32_t tmem_cols;
  int nacc;                   // TMEM accumulators (4, or 2 when a tile is wider than 128 columns)
  int relu;                   // fwd: relu epilogue
  // classes: fwd / wgrad one (the whole GEMM); dgrad sh * sw parity classes
  int ncls, max_tiles;        // item = ((split * max_tiles + tile) * ncls + class) * tiles_n + column tile
  int cls_ph[MAX_CLS], cls_pw[MAX_CLS];
  int cls_hc[MAX_CLS], cls_wc[MAX_CLS];  // dgrad: rows and columns of the class per image
  int cls_nj[MAX_CLS];        // dgrad: class taps along w
  int cls_m[MAX_CLS];         // GEMM rows of the class
  int cls_k[MAX_CLS];         // reduction length of the class (a multiple of 8)
  int cls_ktab[MAX_CLS];      // first table entry
  int cls_kb[MAX_CLS];        // first K block in the resident B operand
  const __nv_bfloat16* an;    // fwd / wgrad: x, dgrad: dy, as bf16 NHWC [n][h][w][CP]
  const __nv_bfloat16* bn;    // wgrad: dy as bf16 NHWC [n][oh][ow][OPW]
  const float* bsrc;          // fwd / dgrad: w (fp32 OIHW)
  const uint8_t* bimg;        // fwd / dgrad: the resident B operand, bf16 and swizzled as in shared memory
  float* out;                 // fwd: y    dgrad: dx   wgrad: partials [splits][O][M]; fwd / dgrad: null
                              // when only the channels-last copy is wanted
  const float* mask;          // dgrad: dx *= (mask > 0) when not null
  const __nv_bfloat16* mask_cl;  // dgrad, instead: dx *= (mask_cl != 0), the ReLU output's channels-last copy
  int mask_cp;                // its channels
  __nv_bfloat16* out_cl;      // fwd / dgrad, optional: the result's bf16 channels-last copy [pixels][out_cp]
  int out_cp;                 // its channels (Nc rounded up to 8; channels >= Nc are written as zero)
  // fwd / dgrad with 64-channel K blocks: one TMA box per K block instead of cp.async.
  // A tile is tn images x th rows x tw columns of output pixels (fwd) or class pixels
  // (dgrad); tile = image block * tiles_h + row block
  int tma, tw, th, tn, tiles_h;
  uint32_t box_bytes;         // tw * th * tn * 128
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

// 16-byte copy global -> shared through L2 (the little L1 left beside the shared memory
// would not hold the taps' reuse anyway); src_bytes = 0 writes zeros (nothing is read)
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
  if (a.tma) {  // row block inside the image (fwd: OH rows, dgrad: the class's rows)
    return a.cls_k[r.cls] > 0 && (r.mt % a.tiles_h) * a.th < a.cls_hc[r.cls];
  }
  return r.mt * BM < a.cls_m[r.cls];
}

// TMA tiles: tile row r -> (image, row, column); false past the tile's pixels
__device__ __forceinline__ bool tile_pixel(const Args& a, const Item& it, int r, int& n, int& hh, int& ww) {
  const int wi = r % a.tw, q = r / a.tw, hi = q % a.th, ni = q / a.th;
  n = (it.mt / a.tiles_h) * a.tn + ni;
  hh = (it.mt % a.tiles_h) * a.th + hi;
  ww = wi;
  return ni < a.tn && n < a.N && hh < a.cls_hc[it.cls] && ww < a.cls_wc[it.cls];
}
__device__ __forceinline__ int kblocks_of(const Args& a, const Item& r) {
  if (a.lq == 0) return (a.cls_k[r.cls] + BK - 1) / BK;
  const int q0 = r.sp * a.lq, q1 = min(a.K, q0 + a.lq);
  return (q1 - q0 + BK - 1) / BK;
}

// fp32 NCHW [N, C, HW] -> bf16 NHWC [N, HW, Cp] (channels >= C zero): a thread writes 8
// channels of one pixel (one 16-byte store); consecutive threads take consecutive pixels,
// so every fp32 read of a warp is one contiguous run
__global__ void __launch_bounds__(256) nchw_to_nhwc_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                                                int64_t N, int C, int64_t HW, int Cp) {
  const int cg = Cp / 8;
  const int64_t total = N * HW * cg;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int g = (int)(e / (N * HW));  // channel group outermost: a warp reads 32 consecutive pixels
    const int64_t pix = e - (int64_t)g * (N * HW);
    const int64_t n = pix / HW, hw = pix - n * HW;
    const float* s = src + (n * C) * HW + hw;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = g * 8 + k;
      v[k] = c < C ? __ldg(s + (int64_t)c * HW) : 0.f;
    }
    *reinterpret_cast<uint4*>(dst + pix * Cp + g * 8) =
        make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  }
}

// The fwd / dgrad weight operand as the kernel keeps it in shared memory: [K blocks of all
// classes][column tiles][BN rows x 64] bf16 in the 128-byte swizzle, built once per call
// from the fp32 OIHW weights (one 16-byte piece per thread), so each CTA only copies it.
//   fwd:   B[o, k = t*Cp + c]            = w[o, c, i, j]   (0 for c >= C)
//   dgrad: B[c, k = u*Op + o] of a class = w[o, c, i, j]   (0 for o >= O)
template <int MODE>
__global__ void __launch_bounds__(256) pack_b_kernel(const __grid_constant__ Args a, uint8_t* __restrict__ img) {
  const int pieces_per_kb = a.tiles_n * a.BN * 8;
  const int total = a.kb_total * pieces_per_kb;
  const int KHW = a.KH * a.KW;
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < total; p += gridDim.x * blockDim.x) {
    const int kbg = p / pieces_per_kb, rem = p - kbg * pieces_per_kb;
    const int col = rem >> 3, j8 = rem & 7;  // column over all column tiles
    int c = 0;
    while (c + 1 < a.ncls && a.cls_kb[c + 1] <= kbg) ++c;
    const int k0 = (kbg - a.cls_kb[c]) * BK + j8 * 8;  // chunk start within the class
    int tap = 0, ch0 = 0;
    if (MODE == FWD) {
      tap = k0 / a.CP;
      ch0 = k0 - tap * a.CP;
    } else {
      const int uu = k0 / a.CP, nj = a.cls_nj[c];
      const int ui = uu / nj, uj = uu - ui * nj;
      const int i = (a.cls_ph[c] + a.pt) % a.sh + ui * a.sh, j = (a.cls_pw[c] + a.pl) % a.sw + uj * a.sw;
      tap = i * a.KW + j;
      ch0 = k0 - uu * a.CP;
    }
    const bool kin = k0 < a.cls_k[c] && col < a.Nc;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int ch = ch0 + e;  // fwd: input channel c; dgrad: output channel o
      const bool ok = kin && ch < (MODE == FWD ? a.C : a.O);
      const int off = MODE == FWD ? (col * a.C + ch) * KHW + tap : (ch * a.C + col) * KHW + tap;
      v[e] = ok ? __ldg(a.bsrc + off) : 0.f;
    }
    const int nt = col / a.BN, rr = col - nt * a.BN;
    *reinterpret_cast<uint4*>(img + (size_t)((kbg * a.tiles_n + nt) * a.BN) * 128u + swz(rr, j8)) =
        make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) conv_igemm_kernel(const __grid_constant__ Args a,
                                                                const __grid_constant__ CUtensorMap amap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sStages = smem;
  uint8_t* sResB = smem + a.resb_off;
  int4* tab = reinterpret_cast<int4*>(smem + a.resb_off + (MODE == WGRAD ? 0u : (uint32_t)a.kb_total * a.tiles_n * a.BN * 128u));
  uint64_t* full = reinterpret_cast<uint64_t*>(tab + a.ktab);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;  // [4]
  uint64_t* acc_empty = acc_full + 4;     // [4]
  uint64_t* drained = acc_empty + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Tables:
  //   fwd   per 8-element chunk k0 = t*Cp + c0 of the reduction:  {(i*W + j)*Cp + c0, i, j, 0}
  //   wgrad the same per 8-row chunk t*Cp + c0 of the GEMM rows
  //   dgrad per chunk of class (ph, pw), k0 = u*Op + o0 over the class taps u = (i, j):
  //                              {(dh*OW + dw)*Op + o0, dh, dw, 0},  dh = (ph + pt - i) / sh (exact)
  if (MODE == DGRAD) {
    for (int c = 0; c < a.ncls; ++c) {
      const int ph = a.cls_ph[c], pw = a.cls_pw[c];
      const int i0 = (ph + a.pt) % a.sh, j0 = (pw + a.pl) % a.sw;
      const int nj = a.cls_nj[c];
      for (int kc = threadIdx.x; kc < a.cls_k[c] / 8; kc += blockDim.x) {
        const int k0 = kc * 8;
        const int u = k0 / a.CP, o0 = k0 - u * a.CP;
        const int ui = u / nj, uj = u - ui * nj;
        const int i = i0 + ui * a.sh, j = j0 + uj * a.sw;
        const int dh = (ph + a.pt - i) / a.sh, dw = (pw + a.pl - j) / a.sw;
        tab[a.cls_ktab[c] + kc] = make_int4((dh * a.OW + dw) * a.CP + o0, dh, dw, 0);
      }
    }
  } else {
    for (int kc = threadIdx.x; kc < a.ktab; kc += blockDim.x) {
      const int k0 = kc * 8;
      const int t = k0 / a.CP, c0 = k0 - t * a.CP;
      const int i = t / a.KW, j = t - i * a.KW;
      tab[kc] = make_int4((i * a.W + j) * a.CP + c0, i, j, 0);
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);  // one producer warp per stage
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS / 2);  // the four warps of the group that drains it
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
    // resident B: the packed image (pack_b_kernel) copied in with 16-byte cp.async, every
    // piece of a thread in flight at once (a load-then-store loop would pay one L2 round
    // trip per piece: about 40 in a row for a 147 KB image)
    if (warp < PROD_WARPS) {
      const int n16 = (int)((uint32_t)a.kb_total * a.tiles_n * a.BN * 8u);
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.bimg);
      const uint32_t dst = smem_u32(sResB);
      for (int i = threadIdx.x; i < n16; i += PROD_THREADS) cp16(dst + (uint32_t)i * 16u, src + (size_t)i * 16u, 16u);
      cp_wait_all();
      fence_proxy_async_smem();
    }
    __syncthreads();
  }

  if (warp < PROD_WARPS) {
    // ------------------------------------------------------------ producers
    uint32_t L = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      Item r;
      if (!item_of(a, it, r)) continue;
      const int m0 = r.mt * BM, n0 = r.nt * a.BN;
      const int nkb = kblocks_of(a, r);
      if (MODE != WGRAD && a.tma) {
        // one thread loads each K block as one TMA box: 64 channels of one tap for every
        // pixel of the tile (fwd: the box walks the input with the convolution's stride;
        // dgrad: dy at the class tap's offset); taps falling outside the image read zeros
        if (nkb <= 0) continue;
        const uint32_t first = L;
        L += (uint32_t)nkb;
        if (warp != 0 || lane != 0) continue;
        const int cbs = a.CP / 64;  // 64-channel blocks per tap
        const int nb = r.mt / a.tiles_h, hb0 = (r.mt % a.tiles_h) * a.th;
        for (int kb = 0; kb < nkb; ++kb) {
          const uint32_t Lk = first + (uint32_t)kb;
          const int s = (int)(Lk % (uint32_t)a.stages);
          if (!mbar_wait(&empty[s], ((Lk / (uint32_t)a.stages) & 1) ^ 1)) {
            ok = false;
            break;
          }
          const int u = kb / cbs, cb = kb - u * cbs;
          int c1, c2;
          if (MODE == FWD) {
            const int i = u / a.KW, j = u - i * a.KW;
            c1 = j - a.pl;                       // input column of output column 0
            c2 = hb0 * a.sh - a.pt + i;          // input row of the tile's first output row
          } else {
            const int nj = a.cls_nj[r.cls];
            const int ui = u / nj, uj = u - ui * nj;
            const int i = (a.cls_ph[r.cls] + a.pt) % a.sh + ui * a.sh, j = (a.cls_pw[r.cls] + a.pl) % a.sw + uj * a.sw;
            c1 = (a.cls_pw[r.cls] + a.pl - j) / a.sw;        // dw
            c2 = hb0 + (a.cls_ph[r.cls] + a.pt - i) / a.sh;  // first class row + dh
          }
          mbar_expect_tx(&full[s], a.box_bytes);
          tma_load_4d(sStages + (uint32_t)s * a.stage_bytes, &amap, &full[s], cb * 64, c1, c2, nb * a.tn);
        }
        continue;
      }
      if constexpr (MODE != WGRAD) {
        // K block L goes to warp L % stages into stage L % stages: every stage has one
        // producer warp that refills it in order, so a parity wait can never pass a phase
        // that is two uses ahead. Lane = rows lane + 32 q, all 8 chunks of each.
        if (nkb <= 0) continue;
        const uint32_t np = (uint32_t)a.stages;
        const uint32_t first = L;
        L += (uint32_t)nkb;
        if ((uint32_t)warp >= np) continue;
        uint32_t mine = first + ((uint32_t)warp + np - first % np) % np;
        if (mine >= L) continue;
        int base[4], hb[4], wb[4];
        bool rv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int m = m0 + lane + 32 * q;
          rv[q] = m < a.cls_m[r.cls];
          const int mm = rv[q] ? m : 0;
          if (MODE == FWD) {
            const int n = mm / a.P, p = mm - n * a.P, oh = p / a.OW, ow = p - oh * a.OW;
            hb[q] = oh * a.sh - a.pt;
            wb[q] = ow * a.sw - a.pl;
            base[q] = ((n * a.H + hb[q]) * a.W + wb[q]) * a.CP;
          } else {
            const int hc = a.cls_hc[r.cls], wc = a.cls_wc[r.cls];
            const int n = mm / (hc * wc), rem = mm - n * (hc * wc), hh = rem / wc, ww = rem - hh * wc;
            hb[q] = hh;
            wb[q] = ww;
            base[q] = ((n * a.OH + hh) * a.OW + ww) * a.CP;
          }
        }
        const int4* ctab = tab + a.cls_ktab[r.cls];
        const int nchunks = a.cls_k[r.cls] / 8;
        const int HH = MODE == FWD ? a.H : a.OH, WW = MODE == FWD ? a.W : a.OW;
        for (; mine < L; mine += np) {
          const int kb = (int)(mine - first);
          const int s = (int)(mine % (uint32_t)a.stages);
          if (!warp_wait(&empty[s], ((mine / (uint32_t)a.stages) & 1) ^ 1, 0)) {
            ok = false;
            break;
          }
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
#pragma unroll
          for (int j8 = 0; j8 < 8; ++j8) {
            const int kc = kb * 8 + j8;
            const int4 t = ctab[min(kc, nchunks - 1)];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int h = hb[q] + t.y, w = wb[q] + t.z;
              const bool okk = rv[q] && kc < nchunks && (unsigned)h < (unsigned)HH && (unsigned)w < (unsigned)WW;
              cp16(sA + swz(lane + 32 * q, j8), a.an + (okk ? base[q] + t.x : 0), okk ? 16u : 0u);
            }
          }
          cp_wait_all();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      } else {
        // wgrad: K block L (64 output pixels q) goes to warp L % stages into stage L % stages,
        // as for fwd / dgrad. Both operands are MN-major (the pixel index q is K): for each
        // q a 128-byte row holds 64 consecutive GEMM rows (taps x channels) of A, or 64
        // output channels of B, copied from the channels-last copies of x and dy. Lane = q
        // rows lane and lane + 32.
        if (nkb <= 0) continue;
        const uint32_t np = (uint32_t)a.stages;
        const uint32_t first = L;
        L += (uint32_t)nkb;
        if ((uint32_t)warp >= np) continue;
        uint32_t mine = first + ((uint32_t)warp + np - first % np) % np;
        const int qs = r.sp * a.lq, qe = min(a.K, qs + a.lq);
        const int mchunks = a.M / 8;  // M = taps * Cp
        const int nb = a.BN / 64;     // 64-column blocks of B
        for (; mine < L; mine += np) {
          const int kb = (int)(mine - first);
          const int s = (int)(mine % (uint32_t)a.stages);
          if (!warp_wait(&empty[s], ((mine / (uint32_t)a.stages) & 1) ^ 1, 0)) {
            ok = false;
            break;
          }
          const uint32_t sA = smem_u32(sStages + (uint32_t)s * a.stage_bytes);
          const uint32_t sB = sA + A_BYTES;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int qr = lane + 32 * h2;  // K row of the tile
            const int q = qs + kb * BK + qr;
            const bool qv = q < qe;
            const int qq = qv ? q : 0;
            const int n = qq / a.P, p = qq - n * a.P, oh = p / a.OW, ow = p - oh * a.OW;
            const int hq = oh * a.sh - a.pt, wq = ow * a.sw - a.pl;
            const int xbase = ((n * a.H + hq) * a.W + wq) * a.CP;
            const int dbase = ((n * a.OH + oh) * a.OW + ow) * a.OPW;
            const uint32_t rowoff = (uint32_t)qr * 128u;
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
              for (int j8 = 0; j8 < 8; ++j8) {
                const int mc = (m0 + 64 * b) / 8 + j8;
                const int4 t = tab[min(mc, mchunks - 1)];
                const int hh = hq + t.y, ww = wq + t.z;
                const bool okk = qv && mc < mchunks && (unsigned)hh < (unsigned)a.H && (unsigned)ww < (unsigned)a.W;
                cp16(sA + (uint32_t)b * 8192u + rowoff + ((uint32_t)(j8 ^ (qr & 7)) << 4), a.an + (okk ? xbase + t.x : 0),
                     okk ? 16u : 0u);
              }
            for (int b = 0; b < nb; ++b)
#pragma unroll
              for (int j8 = 0; j8 < 8; ++j8) {
                const int o0 = n0 + 64 * b + 8 * j8;
                const bool okk = qv && o0 < a.OPW;
                cp16(sB + (uint32_t)b * 8192u + rowoff + ((uint32_t)(j8 ^ (qr & 7)) << 4), a.bn + (okk ? dbase + o0 : 0),
                     okk ? 16u : 0u);
              }
          }
          cp_wait_all();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // wgrad: A and B MN-major (bits 15, 16)
      const uint32_t mn = MODE == WGRAD ? (1u << 15) | (1u << 16) : 0u;
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | mn | ((uint32_t)(a.BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
      uint32_t L = 0, T = 0;
      bool ok = true, issued = false;
      for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
        Item r;
        if (!item_of(a, it, r)) continue;
        const int nkb = kblocks_of(a, r);
        if (nkb <= 0) continue;
        const uint32_t b = T % (uint32_t)a.nacc;
        if (!mbar_wait(&acc_empty[b], ((T / (uint32_t)a.nacc) & 1) ^ 1, 32)) break;
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
            // K-major: +32 B per 16-wide K step inside the swizzled rows; MN-major: +2048 B
            // (16 K rows of 128 B), 64-element blocks 8192 B apart
            const uint64_t ad = MODE == WGRAD ? smem_desc(sA + k * 2048, 8192, 1024) : smem_desc(sA + k * 32, 16, 1024);
            const uint64_t bd = MODE == WGRAD ? smem_desc(sB + k * 2048, 8192, 1024) : smem_desc(sB + k * 32, 16, 1024);
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
    // warps 8-11 drain the even accumulator tiles, warps 12-15 the odd ones: one warp per
    // TMEM lane quarter, every 32-column chunk of its quarter, so two tiles drain at once
    const int q = warp & 3, grp = (warp - MMA_WARP - 1) >> 2;
    uint32_t T = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < a.items && ok; it += gridDim.x) {
      Item r;
      if (!item_of(a, it, r)) continue;
      if (kblocks_of(a, r) <= 0) continue;
      const uint32_t tt = T++;
      if ((int)(tt & 1u) != grp) continue;
      const uint32_t b = tt % (uint32_t)a.nacc;
      ok = warp_wait(&acc_full[b], (tt / (uint32_t)a.nacc) & 1, 64);
      if (!ok) break;
      tc_fence_after();
      const int m = r.mt * BM + q * 32 + lane;  // this lane's GEMM row
      bool rv = m < a.cls_m[r.cls];
      int64_t obase, ostride, pix = 0;  // pix: the row's pixel in the channels-last copy
      if (MODE != WGRAD && a.tma) {
        int n, hh, ww;
        rv = tile_pixel(a, r, q * 32 + lane, n, hh, ww);
        if (!rv) n = hh = ww = 0;
        if (MODE == FWD) {
          obase = (int64_t)n * a.O * a.P + hh * a.OW + ww;
          ostride = a.P;
          pix = (int64_t)n * a.P + hh * a.OW + ww;
        } else {
          const int h = a.cls_ph[r.cls] + a.sh * hh, w = a.cls_pw[r.cls] + a.sw * ww;
          obase = (int64_t)n * a.C * a.HW + h * a.W + w;
          ostride = a.HW;
          pix = (int64_t)n * a.HW + h * a.W + w;
        }
      } else {
        const int mm = rv ? m : 0;
        if (MODE == FWD) {
          const int n = mm / a.P, p = mm - n * a.P;
          obase = (int64_t)n * a.O * a.P + p;
          ostride = a.P;
          pix = mm;
        } else if (MODE == DGRAD) {
          const int hc = a.cls_hc[r.cls], wc = a.cls_wc[r.cls];
          const int n = mm / (hc * wc), rem = mm - n * (hc * wc), hh = rem / wc, ww = rem - hh * wc;
          const int h = a.cls_ph[r.cls] + a.sh * hh, w = a.cls_pw[r.cls] + a.sw * ww;
          obase = (int64_t)n * a.C * a.HW + h * a.W + w;
          ostride = a.HW;
          pix = (int64_t)n * a.HW + h * a.W + w;
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
        float mv[32];
        if (MODE == DGRAD && a.mask != nullptr) {
          // the chunk's 32 mask values are all loaded before its first store
          const float* __restrict__ mk = a.mask + obase + (int64_t)(n0 + c0) * ostride;
#pragma unroll
          for (int i = 0; i < 32; ++i) mv[i] = __ldg(mk + (rv && i < nn ? (int64_t)i * ostride : 0));
        } else if (MODE == DGRAD && a.mask_cl != nullptr) {
          // the mask from the ReLU output's bf16 channels-last copy (nonzero exactly where
          // the output is positive): this row's 32 channels in four 16-byte loads
          const uint4* mk = reinterpret_cast<const uint4*>(a.mask_cl + (rv ? pix : 0) * a.mask_cp + n0 + c0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 u = 8 * k < nn ? __ldg(mk + k) : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              mv[8 * k + 2 * h] = (wv[h] & 0xFFFFu) ? 1.f : 0.f;
              mv[8 * k + 2 * h + 1] = (wv[h] >> 16) ? 1.f : 0.f;
            }
          }
        }
        tmem_wait(v);
        if (c0 + 32 >= ncols) {  // this warp's last TMEM read of the item: hand the accumulator back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!rv) continue;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = __uint_as_float(v[i]);
          if (MODE == DGRAD && (a.mask != nullptr || a.mask_cl != nullptr)) o[i] = x * (mv[i] > 0.f ? 1.f : 0.f);
          else if (MODE == FWD && a.relu) o[i] = x > 0.f ? x : 0.f;
          else o[i] = x;
        }
        if (a.out != nullptr) {
          float* __restrict__ dst = a.out + obase + (int64_t)(n0 + c0) * ostride;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nn) dst[(int64_t)i * ostride] = o[i];
        }
        if (MODE != WGRAD && a.out_cl != nullptr) {
          // the row's channels n0 + c0 .. + 31 of the channels-last bf16 copy, 16 bytes at a
          // time; channels past Nc (up to out_cp) are zero
          __nv_bfloat16* cl = a.out_cl + pix * a.out_cp + n0 + c0;
          const int room = a.out_cp - (n0 + c0);
          // a ReLU output's copy keeps every positive value nonzero (below 2^-133, where
          // round-to-nearest would give +0, the smallest bf16 subnormal instead), so the
          // copy is also the exact Greater(pre, 0) mask of the ReLU VJP
          const bool keep = MODE == FWD && a.relu;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (8 * k < room) {
              uint32_t wv[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const int i0 = 8 * k + 2 * h;
                const float lo = i0 < nn ? o[i0] : 0.f, hi = i0 + 1 < nn ? o[i0 + 1] : 0.f;
                uint32_t pw = pack_bf16(lo, hi);
                if (keep) {
                  if (lo > 0.f && (pw & 0xFFFFu) == 0u) pw |= 1u;
                  if (hi > 0.f && (pw >> 16) == 0u) pw |= 1u << 16;
                }
                wv[h] = pw;
              }
              *reinterpret_cast<uint4*>(cl + 8 * k) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
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

// partials [S][O][M] (row = t*Cp + c, channels padded to Cp) -> dw [O, C, KH, KW]. A block
// takes 32 consecutive (o, row) outputs; warp k sums splits k, k + 8, k + 16, ... of them in
// order (each split's 32 values are one 128-byte read), then lane l adds the 8 warp sums
// in warp order, so the result is the same on every run
__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float* __restrict__ part, float* __restrict__ dw, int S, int O,
                                                           int M, int C, int Cp, int KHW) {
  __shared__ float sh[8][33];
  const int lane = threadIdx.x & 31, k = threadIdx.x >> 5;
  const int64_t total = (int64_t)O * M;
  const int64_t e = (int64_t)blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (e < total) {
    const float* p = part + e;
#pragma unroll 4
    for (int sp = k; sp < S; sp += 8) acc += __ldg(p + (int64_t)sp * total);
  }
  sh[k][lane] = acc;
  __syncthreads();
  if (k == 0 && e < total) {
    float t = sh[0][lane];
#pragma unroll
    for (int i = 1; i < 8; ++i) t += sh[i][lane];
    const int o = (int)(e / M), row = (int)(e - (int64_t)o * M);
    const int tap = row / Cp, c = row - tap * Cp;
    if (c < C) dw[((int64_t)o * C + c) * KHW + tap] = t;
  }
}

struct Plan {
  Args a;
  size_t smem;
  size_t ws;  // workspace: fwd / dgrad the NHWC bf16 source, wgrad the split partials
  bool ok;
  const char* why;
};

inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

// Shapes the kernel handles: 32-bit element offsets (tensors up to 2^30 elements), at most
// KTAB_MAX reduction indices (fwd / dgrad, channels padded to 8) or taps x channels
// (wgrad), at most 16 stride-parity classes, and (fwd / dgrad) the whole bf16 weight
// operand resident in shared memory beside two A stages.
static Plan plan(int mode, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                 int64_t sh, int64_t sw, int64_t pt, int64_t pl) {
  Plan p{};
  p.ok = false;
  const int64_t lim = (int64_t)1 << 30;
  const int64_t Cp = (C + 7) / 8 * 8, Op = (O + 7) / 8 * 8;
  if (N * Cp * H * W > lim || N * Op * OH * OW > lim || O * C * KH * KW > lim) {
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
  const int64_t Opw = (O + 63) / 64 * 64;
  if (mode == WGRAD && N * Opw * OH * OW > lim) {
    p.why = "tensor above 2^30 elements";
    return p;
  }
  a.OPW = (int)Opw;
  if (mode == FWD) M = N * OH * OW, Nc = O, K = Cp * taps, a.CP = (int)Cp;
  else if (mode == DGRAD) M = N * H * W, Nc = C, K = Op * taps, a.CP = (int)Op;
  else M = Cp * taps, Nc = O, K = N * OH * OW, a.CP = (int)Cp;
  if ((mode == WGRAD ? M : K) > KTAB_MAX) {
    p.why = "more than 2048 reduction indices (or taps x channels)";
    return p;
  }
  a.M = (int)M, a.Nc = (int)Nc, a.K = (int)K;
  // wgrad: B is MN-major in 64-column blocks
  a.BN = mode == WGRAD ? (int)std::min<int64_t>(256, Opw) : (int)std::min<int64_t>(256, (Nc + 15) / 16 * 16);
  a.BNT = (a.BN + 31) / 32 * 32;
  a.nacc = 4 * a.BNT <= 512 ? 4 : 2;
  uint32_t cols = 32;
  while (cols < (uint32_t)(a.nacc * a.BNT)) cols <<= 1;
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
      a.cls_ph[c] = ph, a.cls_pw[c] = pw, a.cls_hc[c] = hc, a.cls_wc[c] = wc, a.cls_nj[c] = nj;
      a.cls_k[c] = (int)(Op * ni * nj);
      a.cls_m[c] = a.cls_k[c] > 0 ? (int)(N * hc * wc) : 0;  // pixels no tap reaches are zero-filled by the caller
      a.cls_ktab[c] = koff;
      a.cls_kb[c] = kboff;
      koff += a.cls_k[c] / 8;
      kboff += (int)ceil_div(a.cls_k[c], BK);
      max_tiles = std::max<int64_t>(max_tiles, ceil_div(a.cls_m[c], BM));
    }
    a.kb_total = kboff;
    a.ktab = koff;
  } else {
    a.ncls = 1;
    a.cls_ph[0] = a.cls_pw[0] = 0;
    a.cls_hc[0] = a.cls_wc[0] = a.cls_nj[0] = 1;
    a.cls_m[0] = (int)M;
    a.cls_k[0] = (int)(mode == WGRAD ? 0 : K);
    a.cls_ktab[0] = 0;
    a.cls_kb[0] = 0;
    a.kb_total = mode == WGRAD ? 0 : (int)ceil_div(K, BK);
    a.ktab = (int)(mode == WGRAD ? M / 8 : K / 8);
    max_tiles = ceil_div(M, BM);
  }
  // fwd / dgrad with whole 64-channel K blocks: TMA boxes over tiles of whole pixel rows
  a.tma = 0;
  if (mode != WGRAD && a.CP % 64 == 0) {
    int rows = 0, cols = 0;  // output rows / columns (fwd), largest class rows / columns (dgrad)
    for (int c = 0; c < a.ncls; ++c) {
      rows = std::max(rows, mode == FWD ? (int)OH : a.cls_hc[c]);
      cols = std::max(cols, mode == FWD ? (int)OW : a.cls_wc[c]);
    }
    const int64_t wbox = mode == FWD ? (int64_t)cols * sw : cols;  // elements the box traverses along w
    if (cols >= 1 && cols <= BM && wbox <= 256) {
      int th, tn, tiles_h;
      if ((int64_t)cols * rows <= BM) {
        th = rows, tiles_h = 1, tn = (int)std::min<int64_t>(BM / (cols * rows), N);
      } else {
        tn = 1;
        tiles_h = (int)ceil_div(rows, BM / cols);
        th = (int)ceil_div(rows, tiles_h);
      }
      if ((mode == FWD ? (int64_t)th * sh : th) <= 256 && tn <= 256) {
        a.tma = 1, a.tw = cols, a.th = th, a.tn = tn, a.tiles_h = tiles_h;
        a.box_bytes = (uint32_t)(cols * th * tn) * 128u;
        if (mode == FWD) a.cls_hc[0] = (int)OH, a.cls_wc[0] = (int)OW;
        max_tiles = ceil_div(N, (int64_t)tn) * tiles_h;
      }
    }
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
    // channels-last x, channels-last dy, then the split partials
    p.ws = al256((size_t)N * H * W * Cp * 2) + al256((size_t)N * OH * OW * Opw * 2) + (size_t)a.splits * (size_t)O * (size_t)M * 4;
  } else {
    a.stage_bytes = A_BYTES;
    resb = (size_t)a.kb_total * a.tiles_n * a.BN * 128;
    // the packed weight image, then (when the caller passes none) the channels-last copy
    p.ws = al256(resb) + (mode == FWD ? (size_t)N * H * W * Cp * 2 : (size_t)N * OH * OW * Op * 2);
  }
  const size_t fixed = 1024 + resb + (size_t)a.ktab * 16 + 64 * 8 + 16;
  if (fixed + 2 * (size_t)a.stage_bytes > SMEM_LIMIT) {
    p.why = "shared memory (weights too large to stay resident)";
    return p;
  }
  // fwd / dgrad: one producer warp per stage, so at most PROD_WARPS stages
  const int st = (int)std::min<size_t>(PROD_WARPS, (SMEM_LIMIT - fixed) / a.stage_bytes);
  a.stages = st;
  a.resb_off = (uint32_t)st * a.stage_bytes;
  p.smem = fixed + (size_t)st * a.stage_bytes;
  p.ok = true;
  return p;
}

// tensor map of a TMA-mode source: the channels-last copy [N, rows, cols, CP] (fwd: x, dgrad:
// dy), box = 64 channels x the tile's pixels; the fwd box steps through the input with the
// convolution's stride (element strides sw, sh)
static int make_source_map(int mode, const Args& a, CUtensorMap* map) {
  auto enc = get_encode();
  if (!enc) {
    set_error("conv2d(implicit GEMM): cuTensorMapEncodeTiled unavailable");
    return B200_ERR_CUDA;
  }
  const uint64_t W = mode == FWD ? a.W : a.OW, H = mode == FWD ? a.H : a.OH;
  cuuint64_t dims[4] = {(cuuint64_t)a.CP, W, H, (cuuint64_t)a.N};
  cuuint64_t strides[3] = {(cuuint64_t)a.CP * 2, W * a.CP * 2, H * W * a.CP * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)(mode == FWD ? a.tw * a.sw : a.tw), (cuuint32_t)(mode == FWD ? a.th * a.sh : a.th),
                       (cuuint32_t)a.tn};
  cuuint32_t estr[4] = {1, (cuuint32_t)(mode == FWD ? a.sw : 1), (cuuint32_t)(mode == FWD ? a.sh : 1), 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(a.an), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("conv2d(implicit GEMM): cuTensorMapEncodeTiled failed (%d)", (int)r);
    return B200_ERR_ARG;
  }
  return B200_OK;
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
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  if (MODE != WGRAD && a.tma) {
    const int rc = make_source_map(MODE, a, &map);
    if (rc) return rc;
  }
  const unsigned grid = (unsigned)std::max(1, std::min(a.items, num_sms()));
  conv_igemm_kernel<MODE><<<grid, THREADS, smem, s>>>(a, map);
  return check_launch("conv2d(implicit GEMM)");
}

static int repack(const float* src, __nv_bfloat16* dst, int64_t N, int64_t C, int64_t HW, int64_t Cp, cudaStream_t s) {
  const int64_t total = N * HW * (Cp / 8);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)num_sms() * 16));
  nchw_to_nhwc_bf16_kernel<<<grid, 256, 0, s>>>(src, dst, N, (int)C, HW, (int)Cp);
  return check_launch("conv2d(implicit GEMM, NHWC repack)");
}

template <int MODE>
static int pack_b(Args a, const float* w, uint8_t* img, cudaStream_t s) {
  a.bsrc = w;
  const int64_t total = (int64_t)a.kb_total * a.tiles_n * a.BN * 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)num_sms() * 8));
  pack_b_kernel<MODE><<<grid, 256, 0, s>>>(a, img);
  return check_launch("conv2d(implicit GEMM, weight image)");
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

extern "C" size_t b200_conv2d_igemm_workspace_bytes(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH,
                                                    int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                                                    int64_t pl) {
  if (op < 0 || op > 2 || N < 1) return 0;
  Plan p = plan(op, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  return p.ok ? p.ws : 0;
}

extern "C" int b200_conv2d_channels_last(const float* src, void* dst, int64_t N, int64_t C, int64_t HW, int64_t Cp,
                                         void* stream) {
  B200_REQUIRE(src && dst && (reinterpret_cast<uintptr_t>(dst) & 15) == 0, "conv2d_channels_last: null or unaligned pointer");
  B200_REQUIRE(N >= 0 && C >= 1 && HW >= 1 && Cp >= C && Cp % 8 == 0, "conv2d_channels_last: bad sizes");
  if (N == 0) return B200_OK;
  return repack(src, reinterpret_cast<__nv_bfloat16*>(dst), N, C, HW, Cp, as_stream(stream));
}

extern "C" int b200_conv2d_fwd_igemm(const float* x, const void* x_cl, const float* w, float* y, void* y_cl, int64_t N,
                                     int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH,
                                     int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl, int relu, void* ws,
                                     size_t ws_bytes, void* stream) {
  int rc = check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(x && w && (y || y_cl), "conv2d_fwd_igemm: null pointer");
  Plan p = plan(FWD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) {
    set_error("conv2d_fwd_igemm: unsupported shape (%s)", p.why);
    return B200_ERR_UNSUPPORTED;
  }
  cudaStream_t s = as_stream(stream);
  B200_REQUIRE(ws && ws_bytes >= p.ws && (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
               "conv2d_fwd_igemm: workspace %zu < %zu (256-byte aligned)", ws_bytes, p.ws);
  uint8_t* img = reinterpret_cast<uint8_t*>(ws);
  const __nv_bfloat16* xn = reinterpret_cast<const __nv_bfloat16*>(x_cl);
  if (xn) {
    B200_REQUIRE((reinterpret_cast<uintptr_t>(xn) & 15) == 0, "conv2d_fwd_igemm: x_cl not 16-byte aligned");
  } else {
    auto* cp = reinterpret_cast<__nv_bfloat16*>(img + al256((size_t)p.a.kb_total * p.a.tiles_n * p.a.BN * 128));
    if ((rc = repack(x, cp, N, C, H * W, p.a.CP, s))) return rc;
    xn = cp;
  }
  if ((rc = pack_b<FWD>(p.a, w, img, s))) return rc;
  p.a.relu = relu ? 1 : 0;
  B200_REQUIRE((reinterpret_cast<uintptr_t>(y_cl) & 15) == 0, "conv2d_fwd_igemm: y_cl not 16-byte aligned");
  p.a.an = xn, p.a.bn = nullptr, p.a.bsrc = w, p.a.bimg = img, p.a.out = y, p.a.mask = nullptr;
  p.a.mask_cl = nullptr, p.a.mask_cp = 0;
  p.a.out_cl = reinterpret_cast<__nv_bfloat16*>(y_cl), p.a.out_cp = (int)((O + 7) / 8 * 8);
  return launch<FWD>(p.a, p.smem, s);
}

extern "C" int b200_conv2d_dgrad_igemm(const float* dy, const void* dy_cl, const float* w, const float* mask,
                                       const void* mask_cl, int64_t mask_cp, float* dx, void* dx_cl, int64_t N, int64_t C,
                                       int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                                       int64_t sh, int64_t sw, int64_t pt, int64_t pl, void* ws, size_t ws_bytes,
                                       void* stream) {
  int rc = check_dims(N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(dy && w && (dx || dx_cl), "conv2d_dgrad_igemm: null pointer");
  B200_REQUIRE(!(mask && mask_cl), "conv2d_dgrad_igemm: mask and mask_cl both given");
  B200_REQUIRE(!mask_cl || (mask_cp >= (C + 7) / 8 * 8 && mask_cp % 8 == 0 && (reinterpret_cast<uintptr_t>(mask_cl) & 15) == 0),
               "conv2d_dgrad_igemm: mask_cl needs >= %lld channels (a multiple of 8) and 16-byte alignment",
               (long long)((C + 7) / 8 * 8));
  Plan p = plan(DGRAD, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl);
  if (!p.ok) {
    set_error("conv2d_dgrad_igemm: unsupported shape (%s)", p.why);
    return B200_ERR_UNSUPPORTED;
  }
  cudaStream_t s = as_stream(stream);
  B200_REQUIRE(ws && ws_bytes >= p.ws && (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
               "conv2d_dgrad_igemm: workspace %zu < %zu (256-byte aligned)", ws_bytes, p.ws);
  B200_REQUIRE((reinterpret_cast<uintptr_t>(dy_cl) & 15) == 0, "conv2d_dgrad_igemm: dy_cl not 16-byte aligned");
  uint8_t* img = reinterpret_cast<uint8_t*>(ws);
  // pixels that no tap reaches (a class without taps: stride above the kernel size) are zero
  for (int c = 0; c < p.a.ncls; ++c)
    if (p.a.cls_k[c] == 0) {
      if (dx) cudaMemsetAsync(dx, 0, (size_t)N * C * H * W * 4, s);
      if (dx_cl) cudaMemsetAsync(dx_cl, 0, (size_t)N * H * W * ((C + 7) / 8 * 8) * 2, s);
      if ((rc = check_launch("conv2d_dgrad_igemm(zero)"))) return rc;
      break;
    }
  const __nv_bfloat16* dyn = reinterpret_cast<const __nv_bfloat16*>(dy_cl);
  if (!dyn) {
    auto* cp = reinterpret_cast<__nv_bfloat16*>(img + al256((size_t)p.a.kb_total * p.a.tiles_n * p.a.BN * 128));
    if ((rc = repack(dy, cp, N, O, OH * OW, p.a.CP, s))) return rc;
    dyn = cp;
  }
  if ((rc = pack_b<DGRAD>(p.a, w, img, s))) return rc;
  p.a.relu = 0;
  B200_REQUIRE((reinterpret_cast<uintptr_t>(dx_cl) & 15) == 0, "conv2d_dgrad_igemm: dx_cl not 16-byte aligned");
  p.a.an = dyn, p.a.bn = nullptr, p.a.bsrc = w, p.a.bimg = img, p.a.out = dx, p.a.mask = mask;
  p.a.mask_cl = reinterpret_cast<const __nv_bfloat16*>(mask_cl), p.a.mask_cp = (int)mask_cp;
  p.a.out_cl = reinterpret_cast<__nv_bfloat16*>(dx_cl), p.a.out_cp = (int)((C + 7) / 8 * 8);
  return launch<DGRAD>(p.a, p.smem, s);
}

extern "C" int b200_conv2d_wgrad_igemm(const float* x, const void* x_cl, const float* dy, const void* dy_cl, float* dw,
                                       int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW,
                                       int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl, void* ws,
                                       size_t ws_bytes, void* stream) {
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
  B200_REQUIRE(ws && ws_bytes >= p.ws && (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
               "conv2d_wgrad_igemm: workspace %zu < %zu (256-byte aligned)", ws_bytes, p.ws);
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  auto* xn = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)N * H * W * p.a.CP * 2);
  auto* dyn = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)N * OH * OW * p.a.OPW * 2);
  float* part = reinterpret_cast<float*>(base);
  B200_REQUIRE((reinterpret_cast<uintptr_t>(x_cl) & 15) == 0 && (reinterpret_cast<uintptr_t>(dy_cl) & 15) == 0,
               "conv2d_wgrad_igemm: channels-last copies not 16-byte aligned");
  if (x_cl) xn = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(x_cl));
  else if ((rc = repack(x, xn, N, C, H * W, p.a.CP, s))) return rc;
  if (dy_cl) dyn = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(dy_cl));
  else if ((rc = repack(dy, dyn, N, O, OH * OW, p.a.OPW, s))) return rc;
  p.a.relu = 0;
  p.a.an = xn, p.a.bn = dyn, p.a.bsrc = nullptr, p.a.out = part, p.a.mask = nullptr, p.a.mask_cl = nullptr;
  rc = launch<WGRAD>(p.a, p.smem, s);
  if (rc) return rc;
  const int64_t total = O * (int64_t)p.a.M;
  wgrad_reduce_kernel<<<(unsigned)ceil_div(total, 32), 256, 0, s>>>(part, dw, p.a.splits, (int)O, p.a.M, (int)C, p.a.CP,
                                                                          (int)(KH * KW));
  return check_launch("conv2d_wgrad_igemm(sum)");
}

// Attention score rows on the tensor cores, with the row softmax (or its VJP) fused into
// the GEMM epilogue, so the [.., M, N] fp32 scores never go to HBM:
//
//   forward : y  = softmax(scale * A.B)                      (rows of N <= 512)
//   backward: dx = scale * y * (G - rowsum(G * y)),  G = A.B  (y read from HBM)
//
// The graph ops replaced: Matmul (eager/core_math_ops/math_matrix.py:21-64) of the
// attention scores Q.K^T (forward) or of dO.V^T (backward), Multiply by the scale and
// Softmax (numpy/eager/math_advanced/math_signal.py:450-467), and the Softmax VJP chain
// the AD pass emits (Multiply / ReduceSum / Subtract, numpy/eager/math_binary.py:9-51,
// eager/core_math_ops/math_reduction.py:37) times the scale.
//
// Persistent kernel, one CTA per SM (the 128 x 512 fp32 accumulator fills the SM's TMEM).
// A tile is 128 rows x all N <= 512 columns of one matrix of the batch:
//   warp 0      TMA producer of the operands: A [128, 64] and B [N, 64] per 64-wide K block
//               (K <= 128), one shared-memory stage; the next tile's loads go out as soon as
//               the MMAs have read the stage, so they land while the epilogue still runs;
//   warp 1      owns TMEM and issues N / 256 x K / 16 tcgen05.mma per tile;
//   warps 2-9   epilogue: two warps per TMEM lane quarter, each owning 256 of a row's columns;
//   warp 10     (backward) TMA producer of y: 128-row x 32-column slabs into a ring per
//               column half, read twice per tile (the second pass mostly from L2).
// Forward epilogue: one TMEM pass keeps a running row maximum and sum of exp2 (log2
// domain: w = x * scale * log2 e), the two warps of a quarter merge theirs through shared
// memory, a second pass writes y = exp2(w - max) / sum. Backward: one pass t = rowsum(G * y),
// merge, a second pass dx = scale * y * (G - t). Outputs leave as 32 x 32 chunks staged in
// swizzled shared memory (two buffers per warp) by TMA bulk-tensor stores, which clip the
// ragged edges; the warp releases the accumulator after its last TMEM read, so the next
// tile's MMAs overlap the end of the epilogue. Every mbarrier wait is bounded; after a
// failed wait a warp stops waiting and the CTA winds down (TMEM freed, stores drained).
#include <algorithm>

#include "tc_common.cuh"

namespace b200 {
namespace attn {

using namespace tc;

constexpr int BMR = 128, NMAX = 512, KMAX = 128, EPI_WARPS = 8;
constexpr uint32_t A_BYTES = BMR * 64 * 2;             // one 64-wide K block of A
constexpr uint32_t B_BYTES = 256 * 64 * 2;             // one 256-row half of B per K block
constexpr uint32_t OPS_BYTES = A_BYTES + 2 * B_BYTES;  // the operand stage
constexpr uint32_t SMEM_LIMIT = 232448;                // opt-in dynamic shared memory per CTA
constexpr float LOG2E = 1.4426950408889634f;

template <bool BWD>
struct Cfg {
  static constexpr int THREADS = BWD ? 352 : 320;
};

struct RowArgs {
  int64_t M, N, K;
  int tiles_m, tiles;                        // 128-row tiles per matrix, tiles in all
  int b_in;                                  // z = z_out * b_in + z_in
  int a_bc_out, a_bc_in, b_bc_out, b_bc_in;  // operand shared along a batch level
  const float* scale;                        // device scalar (nullptr: 1)
  int out_f32, out_bf16;                     // outputs written (y, or dx for the backward)
  int yin_bf16;                              // backward: y is bf16 (else fp32)
  uint32_t stage_bytes;                      // per warp and buffer: fp32 part (4 KB), bf16 part (2 KB)
  int nbuf;                                  // staging buffers per warp (1 or 2)
  int ys;                                    // backward: y ring slots per column half
  uint32_t y_chunk;                          // backward: bytes of one 128 x 32 y slab
};

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// bounded wait whose outcome is the same on every lane of the warp
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int sleep_ns) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, sleep_ns);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

template <bool BWD>
__global__ void __launch_bounds__(Cfg<BWD>::THREADS, 1)
    rows_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                const __grid_constant__ CUtensorMap mapO32, const __grid_constant__ CUtensorMap mapO16,
                const __grid_constant__ CUtensorMap mapY, const __grid_constant__ RowArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ys = BWD ? args.ys : 0;
  uint8_t* sOps = smem;
  uint8_t* sStage = smem + OPS_BYTES;  // [8 warps][nbuf][stage_bytes], 1024-aligned pieces
  uint8_t* sY = sStage + (uint32_t)EPI_WARPS * (uint32_t)args.nbuf * args.stage_bytes;  // [2 halves][ys][y_chunk]
  float* red = reinterpret_cast<float*>(sY + (uint32_t)(2 * ys) * args.y_chunk);        // [2 values][2 halves][128 rows]
  uint64_t* op_full = reinterpret_cast<uint64_t*>(red + 4 * BMR);
  uint64_t* op_empty = op_full + 1;
  uint64_t* acc_full = op_full + 2;
  uint64_t* acc_empty = op_full + 3;
  uint64_t* y_full = op_full + 4;       // [2][ys]
  uint64_t* y_empty = y_full + 2 * ys;  // [2][ys]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(y_empty + 2 * ys);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (int)((args.K + 63) / 64);  // 1 or 2
  const int nh = args.N > 256 ? 2 : 1;        // 256-column halves
  auto half_cols = [&](int h) { return (int)max((int64_t)0, min((int64_t)256, args.N - (int64_t)h * 256)); };

  if (threadIdx.x == 0) {
    mbar_init(op_full, 1);
    mbar_init(op_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_WARPS);
    for (int i = 0; i < 2 * ys; ++i) {
      mbar_init(&y_full[i], 1);
      mbar_init(&y_empty[i], 4);  // the four quarter warps of that column half
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(NMAX));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- operand producer ----------------
      uint32_t L = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x) {
        const int z = tile / args.tiles_m, m0 = (tile % args.tiles_m) * BMR;
        const int zo = z / args.b_in, zi = z % args.b_in;
        const int ai = args.a_bc_in ? 0 : zi, ao = args.a_bc_out ? 0 : zo;
        const int bi = args.b_bc_in ? 0 : zi, bo = args.b_bc_out ? 0 : zo;
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          if (!mbar_wait(op_empty, (L & 1) ^ 1, 32)) {
            ok = false;
            break;
          }
          mbar_expect_tx(op_full, A_BYTES + (uint32_t)nh * B_BYTES);
          tma_load_4d(sOps, &mapA, op_full, kb * 64, m0, ai, ao);
          for (int h = 0; h < nh; ++h) tma_load_4d(sOps + A_BYTES + h * B_BYTES, &mapB, op_full, kb * 64, h * 256, bi, bo);
        }
      }
      // the last load has landed before the CTA may exit
      if (L > 0) mbar_wait(op_full, (L - 1) & 1, 32);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(BMR >> 4) << 24);
      uint32_t L = 0, T = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x, ++T) {
        if (!mbar_wait(acc_empty, (T & 1) ^ 1, 32)) break;  // the epilogue has read the previous tile
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++L) {
          if (!mbar_wait(op_full, L & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (kb * 64 + k * 16 >= args.K) break;
            const uint64_t ad = smem_desc(smem_u32(sOps) + k * 32, 16, 1024);
            for (int h = 0; h < nh; ++h) {
              const uint64_t bd = smem_desc(smem_u32(sOps + A_BYTES + h * B_BYTES) + k * 32, 16, 1024);
              mma_bf16(tmem_base + (uint32_t)(h * 256), ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(op_empty);  // the stage is free once these MMAs have read it
        }
        if (ok) mma_commit(acc_full);
      }
    }
  } else if (warp >= 2 && warp < 2 + EPI_WARPS) {
    // ---------------- epilogue: quarter q = warp % 4, column half `half` ----------------
    // Every warp walks every tile of the CTA and meets its partner warp (same quarter) at
    // the same named barriers, also after a failed wait (it then skips the TMEM and the
    // shared-memory work): tcgen05.ld is warp-collective and only warp-uniform values
    // steer the loops around it.
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int r = q * 32 + lane;  // row within the tile (= TMEM lane)
    const int ncols = half_cols(half);
    const float s = args.scale ? __ldg(args.scale) : 1.f;
    const float sl = s * LOG2E;
    const uint32_t stage0 = smem_u32(sStage) + (uint32_t)((warp - 2) * args.nbuf) * args.stage_bytes;
    const uint32_t off16 = args.out_f32 ? 4096u : 0u;
    uint32_t T = 0, sc = 0, yn = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++T) {
      const int z = tile / args.tiles_m, m0 = (tile % args.tiles_m) * BMR;
      const int zo = z / args.b_in, zi = z % args.b_in;
      const int row0 = m0 + q * 32;  // this warp's first row
      if (ok) ok = warp_wait(acc_full, T & 1, 64);
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * 256);
      const int last_c = ((ncols + 31) / 32 - 1) * 32;  // the last chunk holding columns (-32: none)
      bool released = false;
      auto release = [&]() {  // after this warp's last TMEM read of the tile
        if (released) return;
        released = true;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
      };
      // one 32 x 32 output chunk (rows row0.., this half's columns col..) through the staging buffers
      auto put = [&](const float (&val)[32], int col) {
        if (row0 >= args.M) return;  // warp-uniform: none of this warp's rows exist
        const uint32_t buf = stage0 + (sc % (uint32_t)args.nbuf) * args.stage_bytes;
        if (sc >= (uint32_t)args.nbuf && lane == 0) {
          if (args.nbuf == 2) bulk_wait_read1();  // the store that used this buffer has read it
          else bulk_wait_read0();
        }
        __syncwarp();
        if (args.out_f32) {
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(val[i]);
          stage_chunk<4>(buf, lane, w);
        }
        if (args.out_bf16) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack_bf16(val[2 * i], val[2 * i + 1]);
          stage_chunk<2>(buf + off16, lane, w);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int x = half * 256 + col;
          if (args.out_f32) tma_store_4d(&mapO32, buf, x, row0, zi, zo);
          if (args.out_bf16) tma_store_4d(&mapO16, buf + off16, x, row0, zi, zo);
          bulk_commit();
        }
        ++sc;
      };
      uint32_t v[32];
      if constexpr (!BWD) {
        // pass 1: running maximum and sum of exp2 over this warp's columns
        float m = -INFINITY, l = 0.f;
        for (int c = 0; c < ncols && ok; c += 32) {
          tmem_ld32_issue(tb + (uint32_t)c, v);
          tmem_wait(v);
          float w[32], cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            w[i] = c + i < ncols ? __uint_as_float(v[i]) * sl : -INFINITY;
            cm = fmaxf(cm, w[i]);
          }
          const float mn = fmaxf(m, cm);
          if (mn == -INFINITY) continue;
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) acc += exp2f(w[i] - mn);
          l = l * exp2f(m - mn) + acc;
          m = mn;
        }
        red[half * BMR + r] = m;
        red[2 * BMR + half * BMR + r] = l;
        named_sync(1 + q, 64);
        const float ma = red[r], mb = red[BMR + r], la = red[2 * BMR + r], lb = red[3 * BMR + r];
        named_sync(1 + q, 64);
        const float mx = fmaxf(ma, mb);
        const float sum = (ma == -INFINITY ? 0.f : la * exp2f(ma - mx)) + (mb == -INFINITY ? 0.f : lb * exp2f(mb - mx));
        const float inv = 1.f / sum;
        // pass 2: y = exp2(w - max) / sum
        for (int c = 0; c < ncols && ok; c += 32) {
          tmem_ld32_issue(tb + (uint32_t)c, v);
          tmem_wait(v);
          if (c == last_c) release();
          float y[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = exp2f(fmaf(__uint_as_float(v[i]), sl, -mx)) * inv;
          put(y, c);
        }
      } else {
        // the y slab of this half's next chunk: wait for it, read this lane's row, release it
        auto take_y = [&](float (&yv)[32]) {
          const uint32_t slot = yn % (uint32_t)ys;
          if (ok) ok = warp_wait(&y_full[half * ys + slot], (yn / (uint32_t)ys) & 1, 0);
          if (ok) {
            const uint32_t base = smem_u32(sY + (uint32_t)(half * ys + slot) * args.y_chunk);
            if (!args.yin_bf16) {
              const uint32_t rb = base + (uint32_t)r * 128u, sw = (uint32_t)(r & 7);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint4 u = ld_shared_v4(rb + (((uint32_t)j ^ sw) << 4));
                yv[4 * j] = __uint_as_float(u.x);
                yv[4 * j + 1] = __uint_as_float(u.y);
                yv[4 * j + 2] = __uint_as_float(u.z);
                yv[4 * j + 3] = __uint_as_float(u.w);
              }
            } else {
              const uint32_t rb = base + (uint32_t)r * 64u, sw = (uint32_t)((r >> 1) & 3);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint4 u = ld_shared_v4(rb + (((uint32_t)j ^ sw) << 4));
                const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  yv[8 * j + 2 * k] = __uint_as_float(wd[k] << 16);
                  yv[8 * j + 2 * k + 1] = __uint_as_float(wd[k] & 0xFFFF0000u);
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&y_empty[half * ys + slot]);
          }
          ++yn;
        };
        // pass 1: t = rowsum(G * y)
        float t = 0.f;
        for (int c = 0; c < ncols && ok; c += 32) {
          tmem_ld32_issue(tb + (uint32_t)c, v);
          tmem_wait(v);
          float yv[32];
          take_y(yv);
          if (!ok) break;
#pragma unroll
          for (int i = 0; i < 32; ++i) t += __uint_as_float(v[i]) * yv[i];
        }
        red[half * BMR + r] = t;
        named_sync(1 + q, 64);
        t = red[r] + red[BMR + r];
        named_sync(1 + q, 64);
        // pass 2: dx = scale * y * (G - t)
        for (int c = 0; c < ncols && ok; c += 32) {
          tmem_ld32_issue(tb + (uint32_t)c, v);
          tmem_wait(v);
          if (c == last_c) release();
          float yv[32];
          take_y(yv);
          if (!ok) break;
          float d[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) d[i] = s * (yv[i] * (__uint_as_float(v[i]) - t));
          put(d, c);
        }
      }
      release();
    }
    if (lane == 0) bulk_wait0();  // this warp's stores have left shared memory and completed
  } else if (warp == 2 + EPI_WARPS) {
    if constexpr (BWD) {
      if (lane == 0) {
      // ---------------- y producer (backward) ----------------
      uint32_t n[2] = {0, 0};
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x) {
        const int z = tile / args.tiles_m, m0 = (tile % args.tiles_m) * BMR;
        const int zo = z / args.b_in, zi = z % args.b_in;
        for (int pass = 0; pass < 2 && ok; ++pass)
          for (int c = 0; c < 256 && ok; c += 32)
            for (int h = 0; h < nh; ++h) {
              if (c >= half_cols(h)) continue;
              const uint32_t slot = n[h] % (uint32_t)ys;
              if (!mbar_wait(&y_empty[h * ys + slot], ((n[h] / (uint32_t)ys) & 1) ^ 1, 32)) {
                ok = false;
                break;
              }
              mbar_expect_tx(&y_full[h * ys + slot], args.y_chunk);
              tma_load_4d(sY + (uint32_t)(h * ys + slot) * args.y_chunk, &mapY, &y_full[h * ys + slot], h * 256 + c, m0, zi, zo);
              ++n[h];
            }
      }
      // every slab this warp issued has landed before the CTA may exit
      for (int h = 0; h < 2; ++h)
        for (uint32_t k = n[h] > (uint32_t)ys ? n[h] - (uint32_t)ys : 0u; k < n[h]; ++k)
          mbar_wait(&y_full[h * ys + k % (uint32_t)ys], (k / (uint32_t)ys) & 1, 32);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(NMAX));
  }
}

// Shared memory of one CTA (1024-byte alignment slack included).
static size_t smem_bytes(bool bwd, const RowArgs& a) {
  return 1024 + OPS_BYTES + (size_t)EPI_WARPS * a.nbuf * a.stage_bytes + (size_t)(bwd ? 2 * a.ys : 0) * a.y_chunk +
         4 * BMR * sizeof(float) + 8 * (4 + 4 * (size_t)(bwd ? a.ys : 0)) + 16;
}

template <bool BWD>
static int launch_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N, int64_t K, int64_t sA_out,
                       int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in, int64_t rsB, int64_t csB,
                       const void* o32, const void* o16, const void* yin, int64_t s_out, int64_t s_in, int64_t ld, RowArgs a,
                       cudaStream_t s) {
  B200_REQUIRE(A && B, "attn rows: null operand");
  B200_REQUIRE(M >= 0 && N >= 1 && K >= 1 && b_out >= 1 && b_in >= 1, "attn rows: bad sizes");
  if (N > NMAX || K > KMAX) {
    set_error("attn rows: N %lld > %d or K %lld > %d", (long long)N, NMAX, (long long)K, KMAX);
    return B200_ERR_UNSUPPORTED;
  }
  // both operands K-major (unit stride along K), 16-byte aligned rows and batch strides
  if (csA != 1 || rsB != 1) {
    set_error("attn rows: operands must be K-major (A cs %lld, B rs %lld)", (long long)csA, (long long)rsB);
    return B200_ERR_UNSUPPORTED;
  }
  auto bad16 = [](int64_t v) { return ((v * 2) % 16) != 0; };
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) || bad16(rsA) || bad16(csB) ||
      (b_out > 1 && (bad16(sA_out) || bad16(sB_out))) || (b_in > 1 && (bad16(sA_in) || bad16(sB_in))) || sA_out < 0 ||
      sA_in < 0 || sB_out < 0 || sB_in < 0) {
    set_error("attn rows: TMA needs 16-byte aligned operands");
    return B200_ERR_UNSUPPORTED;
  }
  B200_REQUIRE(b_out * b_in < 65536 && ceil_div(M, BMR) * b_out * b_in < INT32_MAX, "attn rows: too many tiles");
  if (M == 0) return B200_OK;
  a.M = M;
  a.N = N;
  a.K = K;
  a.b_in = (int)b_in;
  a.tiles_m = (int)ceil_div(M, BMR);
  a.tiles = (int)(a.tiles_m * b_out * b_in);
  a.a_bc_out = (b_out == 1 || sA_out == 0);
  a.a_bc_in = (b_in == 1 || sA_in == 0);
  a.b_bc_out = (b_out == 1 || sB_out == 0);
  a.b_bc_in = (b_in == 1 || sB_in == 0);
  a.out_f32 = o32 != nullptr;
  a.out_bf16 = o16 != nullptr;
  a.stage_bytes = (a.out_f32 ? 4096u : 0u) + (a.out_bf16 ? 2048u : 0u);
  a.nbuf = 2;
  a.ys = 0;
  a.y_chunk = BWD ? (uint32_t)(BMR * 32 * (a.yin_bf16 ? 2 : 4)) : 0u;
  if (BWD) {
    // the deepest y ring (up to four slabs per half) that fits with two staging buffers
    // per warp; one buffer per warp when two would leave fewer than two slabs per half
    for (int nbuf = 2; nbuf >= 1; --nbuf) {
      a.nbuf = nbuf;
      for (a.ys = 4; a.ys >= 1 && smem_bytes(true, a) > SMEM_LIMIT; --a.ys) {
      }
      if (a.ys >= 2) break;
    }
    if (a.ys < 1) {
      set_error("attn rows: shared memory does not fit");
      return B200_ERR_UNSUPPORTED;
    }
  }
  const size_t smem = smem_bytes(BWD, a);
  if (smem > SMEM_LIMIT) {
    set_error("attn rows: shared memory does not fit");
    return B200_ERR_UNSUPPORTED;
  }
  const uint64_t aIn = a.a_bc_in ? 1 : b_in, aOut = a.a_bc_out ? 1 : b_out;
  const uint64_t bIn = a.b_bc_in ? 1 : b_in, bOut = a.b_bc_out ? 1 : b_out;
  const uint64_t spanA = (uint64_t)rsA * 2 * M, spanB = (uint64_t)csB * 2 * N;
  const uint64_t sAi = a.a_bc_in ? spanA : (uint64_t)sA_in * 2, sAo = a.a_bc_out ? sAi * aIn : (uint64_t)sA_out * 2;
  const uint64_t sBi = a.b_bc_in ? spanB : (uint64_t)sB_in * 2, sBo = a.b_bc_out ? sBi * bIn : (uint64_t)sB_out * 2;
  CUtensorMap ma, mb, m32, m16, my;
  memset(&m32, 0, sizeof(m32));
  memset(&m16, 0, sizeof(m16));
  memset(&my, 0, sizeof(my));
  int rc = make_map(&ma, A, K, M, aIn, aOut, rsA * 2, sAi, sAo, 64, BMR);
  if (rc) return rc;
  rc = make_map(&mb, B, K, N, bIn, bOut, csB * 2, sBi, sBo, 64, 256);
  if (rc) return rc;
  // outputs (and y) are [b_out, b_in, M, N] with element strides (s_out, s_in, ld)
  bool ok = true;
  if (o32) ok = ok && make_store_map(&m32, o32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, b_in, b_out, ld, s_in, s_out);
  if (o16) ok = ok && make_store_map(&m16, o16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, b_in, b_out, ld, s_in, s_out);
  if (BWD)
    ok = ok && make_store_map(&my, yin, a.yin_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              a.yin_bf16 ? 2 : 4, N, M, b_in, b_out, ld, s_in, s_out, BMR);
  if (!ok) {
    set_error("attn rows: the row tensors are not addressable by TMA (16-byte aligned base and strides)");
    return B200_ERR_UNSUPPORTED;
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(rows_kernel<BWD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int grid = (int)std::min<int64_t>(a.tiles, num_sms());
  rows_kernel<BWD><<<grid, Cfg<BWD>::THREADS, smem, s>>>(ma, mb, m32, m16, my, a);
  return check_launch(BWD ? "attn softmax_bwd rows" : "attn softmax rows");
}

}  // namespace attn
}  // namespace b200

using namespace b200;

extern "C" int b200_gemm_softmax_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N, int64_t K,
                                      int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in,
                                      int64_t rsB, int64_t csB, const float* scale, float* y, void* y_bf16, int64_t sY_out,
                                      int64_t sY_in, int64_t ldy, void* stream) {
  B200_REQUIRE(y || y_bf16, "gemm_softmax_rows: no output");
  B200_REQUIRE(ldy >= N, "gemm_softmax_rows: ldy < N");
  attn::RowArgs a = {};
  a.scale = scale;
  return attn::launch_rows<false>(A, B, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, y, y_bf16,
                                  nullptr, sY_out, sY_in, ldy, a, as_stream(stream));
}

extern "C" int b200_gemm_softmax_bwd_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N,
                                          int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out,
                                          int64_t sB_in, int64_t rsB, int64_t csB, const float* scale, int y_dtype, const void* y,
                                          float* dx, void* dx_bf16, int64_t s_out, int64_t s_in, int64_t ld, void* stream) {
  B200_REQUIRE(y && (dx || dx_bf16), "gemm_softmax_bwd_rows: null y or no output");
  B200_REQUIRE(y_dtype == B200_F32 || y_dtype == B200_BF16, "gemm_softmax_bwd_rows: y dtype %d", y_dtype);
  B200_REQUIRE(ld >= N, "gemm_softmax_bwd_rows: ld < N");
  attn::RowArgs a = {};
  a.scale = scale;
  a.yin_bf16 = y_dtype == B200_BF16;
  return attn::launch_rows<true>(A, B, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, dx, dx_bf16, y,
                                 s_out, s_in, ld, a, as_stream(stream));
}

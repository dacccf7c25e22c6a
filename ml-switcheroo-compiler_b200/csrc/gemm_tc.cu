// bf16 tensor-core GEMM for sm_100a: TMA -> shared memory (128B swizzle) ->
// tcgen05.mma (one elected thread) -> fp32 accumulator in TMEM -> tcgen05.ld ->
// fused epilogue (alpha, bias, ReLU/GELU, ReLU mask) -> global.
//
// CTA = 6 warps: warp 0 issues TMA loads, warp 1 owns TMEM and issues the MMAs,
// warps 2..5 run the epilogue (each reads the 32 TMEM lanes its warp may access).
// Tile 128 x BN x 64, STAGES-deep mbarrier ring. Operands may be K-major or MN-major
// (a transposed graph operand is only a different tensor map + descriptor bit, it is
// never materialised). Batched through the third tensor-map dimension.
//
// Every mbarrier wait is bounded by a wall-clock limit: on expiry the thread records
// B200_ERR_TIMEOUT in the device error flag and the CTA winds down (TMEM is freed).
#include <cuda.h>
#include <stdlib.h>
#include <string.h>
#include <cudaTypedefs.h>

#include "tc_common.cuh"

namespace b200 {
namespace tc {

// GELU (tanh approximation) in its sigmoid form: 0.5 x (1 + tanh(u)) = x / (1 + exp(-2u)),
// u = sqrt(2/pi) (x + 0.044715 x^3): one exp2 and one fast division instead of tanhf, which
// would otherwise bound the epilogue of the FFN GEMM (134 M elements per step)
__device__ __forceinline__ float gelu_sigmoid_form(float x) {
  const float k2 = -2.f * 0.7978845608028654f * 1.4426950408889634f;  // -2 sqrt(2/pi) log2(e)
  const float u2 = k2 * x * fmaf(0.044715f * x, x, 1.f);
  return __fdividef(x, 1.f + exp2f(u2));
}

#ifndef B200_GEMM_EPI_WARPS
#define B200_GEMM_EPI_WARPS 8
#endif
// Epilogue: 8 warps, two per TMEM lane quarter, splitting the tile's columns. Store mode
// (per launch): 0 = each lane stores its own row from registers (best when the tile's
// main loop is short, K <= 128); 2 = the 32 x 32 chunk is staged in a swizzled 4 KB
// shared-memory buffer per warp and leaves through a TMA bulk-tensor store; 1 = staged
// the same way, then written back as whole row segments (when no store map fits).
constexpr int BM = 128, BK = 64, STAGES = 4, STAGES_PAIR = 6, EPI_WARPS = B200_GEMM_EPI_WARPS, THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t EPI_BUF = 4096;  // per epilogue warp
constexpr uint32_t EPI_SMEM = EPI_WARPS * EPI_BUF;  // after the operand ring
static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "4 or 8 epilogue warps (the staging buffers must fit)");
struct Args {
  void* C;
  void* C2;  // optional bf16 copy of the activation; C then receives the pre-activation
  const float* bias;
  uint8_t* aux;
  int store_mode;  // 0 direct, 1 staged + row-segment stores, 2 staged + TMA bulk stores
  int64_t M, N, K, sC, ldc;
  float alpha;
  int c_dt, epi, a_mn, b_mn, batch;  // batch = b_out * b_in tiles-of-matrices
  int b_in;                          // inner batch count (z = z_out * b_in + z_in)
  int a_bc_out, a_bc_in, b_bc_out, b_bc_in;  // operand shared along that batch level (stride 0)
  int64_t sC_in;                     // C stride of the inner batch level (sC = outer)
  const float* resid;                // optional fp32 residual in C's layout, added after the bias
};

// ---- CTA pairs (tcgen05 cta_group::2) ----
// In a cluster of two CTAs, bit 24 of a shared-memory address selects the CTA; clearing
// it names the same offset in CTA 0, the pair's leader, which owns the barriers the MMA
// waits on.
constexpr uint32_t LEADER_MASK = 0xFEFFFFFFu;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of both CTAs (not warp-aligned: lanes may arrive separately)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n barrier.cluster.wait.acquire;" ::: "memory");
}
// TMA load into this CTA's shared memory whose completed bytes count on the leader's barrier
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                                 int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar) & LEADER_MASK)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
// arrive once on the barrier at this offset in both CTAs when the issued MMAs complete
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"((uint16_t)3)
               : "memory");
}
// arrive on the leader's copy of `bar` (a no-op remap in the leader itself)
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(smem_u32(bar) & LEADER_MASK) : "memory");
}

// Persistent kernel: the CTAs (one per SM) walk the output tiles in a static
// round-robin order (n fastest, then m, then batch: concurrent CTAs share operand panels
// in L2). The TMEM accumulator is double-buffered (2 x BN columns), so the epilogue of
// tile i (TMEM -> registers -> HBM) overlaps the MMAs of tile i+1, and the TMA/MMA
// pipeline runs continuously across tile boundaries.
//
// PAIR: two CTAs of a cluster compute one 256 x BN tile with tcgen05 cta_group::2. Each
// CTA loads its 128 rows of A and half of B's BN columns into its own shared memory; the
// pair's MMA (issued by the leader, CTA 0) reads A and B from both, and writes each CTA's
// 128 x BN accumulator into that CTA's TMEM. Per SM that halves the B operand's
// shared-memory traffic (TMA writes + MMA reads), which bounds the single-CTA kernel on
// 128 x 256 tiles. Both CTAs' loads complete on the leader's stage barrier (it expects
// the bytes of both); the leader's commits arrive on both CTAs' barriers; the epilogue
// warps of both CTAs release an accumulator on the leader's barrier.
template <int BN, int EPI, bool PAIR>
__device__ __forceinline__ void gemm_body(const CUtensorMap& mapA, const CUtensorMap& mapB, const CUtensorMap& mapC,
                                          const CUtensorMap& mapC2, const CUtensorMap& mapAux, const Args& args) {
  constexpr int STG = PAIR ? STAGES_PAIR : STAGES;
  constexpr uint32_t A_BYTES = BM * BK * 2;                    // 16 KB
  constexpr uint32_t B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // this CTA's share of B
  constexpr int TM = PAIR ? 2 * BM : BM;                       // output rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STG * A_BYTES;
  uint8_t* sEpi = sB + STG * B_BYTES;  // EPI_SMEM bytes, 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sEpi + EPI_SMEM);
  uint64_t* empty_bar = full_bar + STG;
  uint64_t* acc_full = empty_bar + STG;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;        // CTA within the pair
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // tile walker
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int num_kb = (int)((args.K + BK - 1) / BK);
  const int tiles_n = (int)((args.N + BN - 1) / BN);
  const int tiles_m = (int)((args.M + TM - 1) / TM);
  const int tiles_mn = tiles_n * tiles_m;
  const int total = tiles_mn * args.batch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(&full_bar[s], 1);   // the (leader's) producer arrival + the loads' bytes
      mbar_init(&empty_bar[s], 1);  // one MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], (PAIR ? 2 : 1) * EPI_WARPS);  // one arrive per epilogue warp (of both CTAs)
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(2 * BN));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(2 * BN));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  // both CTAs' barriers are initialised before either CTA's loads or commits can reach them
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t it = 0;
      bool ok = true;
      for (int tile = unit; tile < total && ok; tile += units) {
        const int z = tile / tiles_mn, r = tile % tiles_mn;
        const int m_tile = r / tiles_n, n_tile = r % tiles_n;
        const int m0 = m_tile * TM + (int)rank * BM;                       // this CTA's A rows
        const int n0 = n_tile * BN + (PAIR ? (int)rank * (BN / 2) : 0);   // this CTA's B columns
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STG;
          const uint32_t round = it / STG;
          if (!mbar_wait(&empty_bar[s], (round & 1) ^ 1)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_expect_tx(&full_bar[s], (PAIR ? 2u : 1u) * (A_BYTES + B_BYTES));
          const int k0 = kb * BK;
          uint8_t* a_dst = sA + s * A_BYTES;
          uint8_t* b_dst = sB + s * B_BYTES;
          const int zo = z / args.b_in, zi = z % args.b_in;
          const int ai = args.a_bc_in ? 0 : zi, ao = args.a_bc_out ? 0 : zo;
          const int bi = args.b_bc_in ? 0 : zi, bo = args.b_bc_out ? 0 : zo;
          auto load = [&](void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3) {
            if constexpr (PAIR) tma_load_4d_pair(dst, map, &full_bar[s], c0, c1, c2, c3);
            else tma_load_4d(dst, map, &full_bar[s], c0, c1, c2, c3);
          };
          if (!args.a_mn) {
            load(a_dst, &mapA, k0, m0, ai, ao);
          } else {
            load(a_dst, &mapA, m0, k0, ai, ao);
            load(a_dst + 8192, &mapA, m0 + 64, k0, ai, ao);
          }
          if (!args.b_mn) {
            load(b_dst, &mapB, k0, n0, bi, bo);
          } else {
#pragma unroll
            for (int j = 0; j < (PAIR ? BN / 2 : BN) / 64; ++j) load(b_dst + j * 8192, &mapB, n0 + 64 * j, k0, bi, bo);
          }
        }
      }
      if constexpr (PAIR) {
        // producer tail: wait until the MMAs released every stage this CTA filled, so no
        // commit from the leader can arrive on this CTA's barriers after it has exited
        for (int i = 0; i < STG && ok; ++i, ++it) ok = mbar_wait(&empty_bar[it % STG], ((it / STG) & 1) ^ 1, 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (the leader, for a pair) ----------------
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)args.a_mn << 15) | ((uint32_t)args.b_mn << 16) |
                             ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int tile = unit; tile < total && ok; tile += units, ++local) {
        const int b = local & 1;
        const uint32_t use = local >> 1;
        if (!mbar_wait(&acc_empty[b], (use & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STG;
          const uint32_t round = it / STG;
          if (!mbar_wait(&full_bar[s], round & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * A_BYTES);
          const uint32_t b_base = smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: +32 B per 16-element K step inside the 128 B swizzle row.
            // MN-major: +2048 B per K step (two 8-row groups of 1024 B).
            const uint64_t ad = args.a_mn ? smem_desc(a_base + k * 2048, 8192, 1024) : smem_desc(a_base + k * 32, 16, 1024);
            const uint64_t bd = args.b_mn ? smem_desc(b_base + k * 2048, 8192, 1024) : smem_desc(b_base + k * 32, 16, 1024);
            if constexpr (PAIR) mma_bf16_pair(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else mma_bf16(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          // stage s free once these MMAs have read it (in both CTAs of a pair)
          if constexpr (PAIR) mma_commit_pair(&empty_bar[s]);
          else mma_commit(&empty_bar[s]);
        }
        // accumulator b complete (also fires when num_kb == 0)
        if (ok) {
          if constexpr (PAIR) mma_commit_pair(&acc_full[b]);
          else mma_commit(&acc_full[b]);
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2 .. 2 + EPI_WARPS) ----------------
    // A warp may only read the TMEM lanes of its quarter (warp id % 4); the two warps of a
    // quarter split the tile's columns. TMEM loads are software-pipelined: the next
    // 32-column chunk is in flight while the current one is finished and stored.
    const int q = warp & 3;
    constexpr int NHALF = EPI_WARPS / 4;
    const int half = (warp - 2) >> 2;
    constexpr int CH = BN / 32 / NHALF;  // chunks per warp per tile
    uint32_t local = 0;
    for (int tile = unit; tile < total; tile += units, ++local) {
      const int z = tile / tiles_mn, r = tile % tiles_mn;
      const int m_tile = r / tiles_n, n_tile = r % tiles_n;
      const int b = local & 1;
      const uint32_t use = local >> 1;
      if (!mbar_wait(&acc_full[b], use & 1)) break;
      tc_fence_after();
      const int64_t row = (int64_t)m_tile * TM + (int64_t)rank * BM + q * 32 + lane;
      const int64_t col0 = (int64_t)n_tile * BN + half * (BN / NHALF);
      const int zo = z / args.b_in, zi = z % args.b_in;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + half * (BN / NHALF));
#pragma unroll 1
      for (int c = 0; c < CH; ++c) {
        uint32_t cur[32];
        if (num_kb > 0) {
          tmem_ld32_issue(tbase + (uint32_t)(c * 32), cur);
          tmem_wait(cur);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) cur[i] = 0u;
        }
        const int64_t cbase = col0 + c * 32;
        if (cbase >= args.N) continue;  // warp-uniform
        // pre = alpha * acc + bias; act = epi(pre); mask bit = pre > 0. The activation is a
        // template parameter and the other choices are uniform branches outside the element
        // loops, so a chunk without them costs one multiply per element (a runtime-selected
        // activation inside the loop is if-converted: tanh would run for every element).
        float v[32], act[32];
        uint32_t mbits = 0;
        if (args.bias && cbase + 32 <= args.N) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaf(args.alpha, __uint_as_float(cur[i]), __ldg(args.bias + cbase + i));
        } else if (args.bias) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = args.alpha * __uint_as_float(cur[i]) + (cbase + i < args.N ? __ldg(args.bias + cbase + i) : 0.f);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = args.alpha * __uint_as_float(cur[i]);
        }
        if (args.resid && row < args.M) {
          // the residual Add that follows the bias Add: y = (acc + bias) + r, rounded twice
          // as the two Adds are
          const float* rp = args.resid + (int64_t)zo * args.sC + (int64_t)zi * args.sC_in + row * args.ldc + cbase;
          if (cbase + 32 <= args.N && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 t = __ldg(reinterpret_cast<const float4*>(rp + i));
              v[i] += t.x; v[i + 1] += t.y; v[i + 2] += t.z; v[i + 3] += t.w;
            }
          } else {
            for (int i = 0; i < 32; ++i)
              if (cbase + i < args.N) v[i] += __ldg(rp + i);
          }
        }
        if (args.aux) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mbits |= (v[i] > 0.f ? 1u : 0u) << i;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if constexpr (EPI == B200_EPI_RELU) act[i] = v[i] > 0.f ? v[i] : 0.f;
          else if constexpr (EPI == B200_EPI_GELU) act[i] = gelu_sigmoid_form(v[i]);
          else act[i] = v[i];
        }
        if (!args.C2) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = act[i];
        }
        const int64_t zoff = (int64_t)zo * args.sC + (int64_t)zi * args.sC_in;
        if (args.store_mode != 0) {
          const int row0 = (int)(m_tile * TM + (int)rank * BM + q * 32);
          if (row0 >= args.M) continue;  // warp-uniform: none of this warp's rows exist
          const int rows_in = (int)min((int64_t)32, args.M - row0);
          const int64_t cols_in = min((int64_t)32, args.N - cbase);
          const uint32_t buf = smem_u32(sEpi) + (uint32_t)(warp - 2) * EPI_BUF;
          const bool tma = args.store_mode == 2;
          // C (fp32 or bf16), then C2 (bf16), then the mask, through the same buffer
#pragma unroll 1
          for (int part = 0; part < 3; ++part) {
            if (part == 1 && !args.C2) continue;
            if (part == 2 && !args.aux) continue;
            const int esz = part == 0 ? (args.c_dt == B200_F32 ? 4 : 2) : (part == 1 ? 2 : 1);
            if (tma) {
              if (lane == 0) bulk_wait_read0();  // the previous bulk store has read the buffer
            }
            __syncwarp();
            if (esz == 4) {
              uint32_t w[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
              stage_chunk<4>(buf, lane, w);
            } else if (esz == 2) {
              const float* src = part == 0 ? v : act;
              uint32_t w[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) w[i] = pack_bf16(src[2 * i], src[2 * i + 1]);
              stage_chunk<2>(buf, lane, w);
            } else {
              uint32_t w[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const uint32_t nib = (mbits >> (4 * k)) & 0xFu;
                w[k] = (nib & 1u) | ((nib >> 1) & 1u) << 8 | ((nib >> 2) & 1u) << 16 | ((nib >> 3) & 1u) << 24;
              }
              stage_chunk<1>(buf, lane, w);
            }
            if (tma) {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                const CUtensorMap* m = part == 0 ? &mapC : (part == 1 ? &mapC2 : &mapAux);
                tma_store_4d(m, buf, (int)cbase, row0, zi, zo);
                bulk_commit();
              }
              continue;
            }
            __syncwarp();
            uint8_t* dst = part == 0 ? reinterpret_cast<uint8_t*>(args.C) : (part == 1 ? reinterpret_cast<uint8_t*>(args.C2) : args.aux);
            dst += (zoff + (int64_t)row0 * args.ldc + cbase) * esz;
            if (esz == 4) write_chunk<4>(buf, lane, dst, args.ldc, rows_in, cols_in);
            else if (esz == 2) write_chunk<2>(buf, lane, dst, args.ldc, rows_in, cols_in);
            else write_chunk<1>(buf, lane, dst, args.ldc, rows_in, cols_in);
          }
          continue;
        }
        if (row >= args.M) continue;
        const int64_t off = zoff + row * args.ldc + cbase;
        const bool full = cbase + 32 <= args.N;
        if (args.c_dt == B200_F32) {
          float* dst = reinterpret_cast<float*>(args.C) + off;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          } else {
            for (int i = 0; i < 32; ++i)
              if (cbase + i < args.N) dst[i] = v[i];
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.C) + off;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16(v[i], v[i + 1]), pack_bf16(v[i + 2], v[i + 3]),
                                                              pack_bf16(v[i + 4], v[i + 5]), pack_bf16(v[i + 6], v[i + 7]));
          } else {
            for (int i = 0; i < 32; ++i)
              if (cbase + i < args.N) dst[i] = __float2bfloat16_rn(v[i]);
          }
        }
        if (args.C2) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.C2) + off;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16(act[i], act[i + 1]), pack_bf16(act[i + 2], act[i + 3]),
                                                              pack_bf16(act[i + 4], act[i + 5]), pack_bf16(act[i + 6], act[i + 7]));
          } else {
            for (int i = 0; i < 32; ++i)
              if (cbase + i < args.N) dst[i] = __float2bfloat16_rn(act[i]);
          }
        }
        if (args.aux) {
          uint8_t* mdst = args.aux + off;
          for (int i = 0; i < 32; ++i)
            if (cbase + i < args.N) mdst[i] = (uint8_t)((mbits >> i) & 1u);
        }
      }
      // accumulator b may be overwritten once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_leader(&acc_empty[b]);
        else mbar_arrive(&acc_empty[b]);
      }
    }
  }
  if (args.store_mode == 2 && warp >= 2 && lane == 0) bulk_wait0();  // this warp's bulk stores are complete
  tc_fence_before();
  // a pair's TMEM is written by the leader's MMAs and read by both epilogues: free it only
  // after both CTAs are done
  if constexpr (PAIR) cluster_sync_all();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN));
    else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * BN));
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA,
                                                             const __grid_constant__ CUtensorMap mapB,
                                                             const __grid_constant__ CUtensorMap mapC,
                                                             const __grid_constant__ CUtensorMap mapC2,
                                                             const __grid_constant__ CUtensorMap mapAux,
                                                             const __grid_constant__ Args args) {
  gemm_body<BN, EPI, false>(mapA, mapB, mapC, mapC2, mapAux, args);
}

// the CTA-pair kernel: clusters of two CTAs along x (CTAs 2p and 2p + 1 form pair p)
template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                    const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapC2,
                    const __grid_constant__ CUtensorMap mapAux, const __grid_constant__ Args args) {
  gemm_body<BN, EPI, true>(mapA, mapB, mapC, mapC2, mapAux, args);
}

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------
template <int BN, int EPI, bool PAIR>
static int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mc2,
                  const CUtensorMap& maux, const Args& a, int64_t batch, cudaStream_t s) {
  constexpr int STG = PAIR ? STAGES_PAIR : STAGES;
  constexpr int BNC = PAIR ? BN / 2 : BN;  // B columns one CTA loads
  const size_t smem = (size_t)STG * (BM * BK * 2 + BNC * BK * 2) + EPI_SMEM + 1024 + 256;
  const int64_t tiles = ceil_div(a.N, BN) * ceil_div(a.M, PAIR ? 2 * BM : BM) * batch;  // batch = b_out * b_in
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    if constexpr (PAIR) cudaFuncSetAttribute(gemm_tc2_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    else cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  if constexpr (PAIR) {
    // as many CTA pairs as can be resident at once (at most one per two SMs; a pair needs
    // two SMs of one GPC), each walking its share of the tiles
    static int max_pairs[64] = {0};
    int cap = num_sms() / 2;
    if (dev >= 0 && dev < 64) {
      if (!max_pairs[dev]) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(2 * cap), 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<BN, EPI>, &cfg) != cudaSuccess || n <= 0) {
          cudaGetLastError();  // clear: fall back to one pair per two SMs
          n = cap;
        }
        max_pairs[dev] = std::min(n, cap);
      }
      cap = max_pairs[dev];
    }
    const int64_t pairs = std::max<int64_t>(1, std::min<int64_t>(tiles, cap));
    gemm_tc2_kernel<BN, EPI><<<(unsigned)(2 * pairs), THREADS, smem, s>>>(ma, mb, mc, mc2, maux, a);
    return check_launch("gemm(bf16 tcgen05, CTA pairs)");
  } else {
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(tiles, num_sms()));
    gemm_tc_kernel<BN, EPI><<<grid, THREADS, smem, s>>>(ma, mb, mc, mc2, maux, a);
    return check_launch("gemm(bf16 tcgen05)");
  }
}

// CTA pairs for large GEMMs: 256 x 256 tiles, both M and N at least one full pair tile.
// B200_GEMM_PAIR=0 in the environment selects the single-CTA kernel everywhere.
static bool use_pairs(int64_t M, int64_t N) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("B200_GEMM_PAIR");
    env = (e && e[0] == '0') ? 0 : 1;
  }
  return env == 1 && N > 128 && M >= 256;
}

}  // namespace tc

int gemm_bf16_tcgen05_b2(int c_dt, const void* A, const void* B, void* C, int64_t b_out, int64_t b_in, int64_t M, int64_t N,
                         int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in,
                         int64_t rsB, int64_t csB, int64_t sC_out, int64_t sC_in, int64_t ldc, float alpha, const float* bias,
                         int epi, void* aux, void* C2, const float* resid, cudaStream_t s) {
  using namespace tc;
  // operand majors: A K-major if csA == 1, MN-major if rsA == 1; B K-major if rsB == 1, MN-major if csB == 1
  int a_mn, b_mn;
  if (csA == 1) a_mn = 0;
  else if (rsA == 1) a_mn = 1;
  else {
    set_error("gemm(bf16): A needs a unit stride (rs %lld cs %lld)", (long long)rsA, (long long)csA);
    return B200_ERR_UNSUPPORTED;
  }
  if (rsB == 1) b_mn = 0;
  else if (csB == 1) b_mn = 1;
  else {
    set_error("gemm(bf16): B needs a unit stride (rs %lld cs %lld)", (long long)rsB, (long long)csB);
    return B200_ERR_UNSUPPORTED;
  }
  const int64_t lda = a_mn ? csA : rsA;  // elements between consecutive non-contiguous indices
  const int64_t ldb = b_mn ? rsB : csB;
  auto bad16 = [](int64_t v) { return ((v * 2) % 16) != 0; };
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) || bad16(lda) || bad16(ldb) ||
      (b_out > 1 && (bad16(sA_out) || bad16(sB_out))) || (b_in > 1 && (bad16(sA_in) || bad16(sB_in))) || sA_out < 0 ||
      sA_in < 0 || sB_out < 0 || sB_in < 0) {
    set_error("gemm(bf16): TMA needs 16-byte aligned bases and strides (lda %lld ldb %lld)", (long long)lda, (long long)ldb);
    return B200_ERR_UNSUPPORTED;
  }
  B200_REQUIRE(M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX && b_out >= 1 && b_in >= 1, "gemm(bf16): bad dims");
  const int BN = N > 128 ? 256 : 128;
  const int64_t batch = b_out * b_in;
  B200_REQUIRE(ceil_div(N, 256) * ceil_div(M, BM) * batch < INT32_MAX && batch < INT32_MAX, "gemm(bf16): too many tiles");
  // a batch level with stride 0 (or count 1) is a 1-deep tensor-map dim read at index 0
  const int a_bc_out = (b_out == 1 || sA_out == 0), a_bc_in = (b_in == 1 || sA_in == 0);
  const int b_bc_out = (b_out == 1 || sB_out == 0), b_bc_in = (b_in == 1 || sB_in == 0);
  const uint64_t rowsA = a_mn ? K : M, rowsB = b_mn ? K : N;
  const uint64_t spanA = (uint64_t)lda * 2 * rowsA, spanB = (uint64_t)ldb * 2 * rowsB;
  const uint64_t aIn = a_bc_in ? 1 : b_in, aOut = a_bc_out ? 1 : b_out;
  const uint64_t bIn = b_bc_in ? 1 : b_in, bOut = b_bc_out ? 1 : b_out;
  const uint64_t sAi = a_bc_in ? spanA : (uint64_t)sA_in * 2, sAo = a_bc_out ? sAi * aIn : (uint64_t)sA_out * 2;
  const uint64_t sBi = b_bc_in ? spanB : (uint64_t)sB_in * 2, sBo = b_bc_out ? sBi * bIn : (uint64_t)sB_out * 2;
  CUtensorMap ma, mb;
  int rc;
  if (!a_mn) rc = make_map(&ma, A, K, M, aIn, aOut, lda * 2, sAi, sAo, 64, 128);
  else rc = make_map(&ma, A, M, K, aIn, aOut, lda * 2, sAi, sAo, 64, 64);
  if (rc) return rc;
  const bool pair = BN == 256 && use_pairs(M, N);
  // K-major B: a CTA of a pair loads BN / 2 of the tile's columns
  if (!b_mn) rc = make_map(&mb, B, K, N, bIn, bOut, ldb * 2, sBi, sBo, 64, pair ? BN / 2 : BN);
  else rc = make_map(&mb, B, N, K, bIn, bOut, ldb * 2, sBi, sBo, 64, 64);
  if (rc) return rc;
  Args a;
  a.C = C;
  a.C2 = C2;
  a.bias = bias;
  a.aux = (uint8_t*)aux;
  a.M = M;
  a.N = N;
  a.K = K;
  a.sC = sC_out;
  a.sC_in = sC_in;
  a.ldc = ldc;
  a.alpha = alpha;
  a.c_dt = c_dt;
  a.epi = epi;
  a.a_mn = a_mn;
  a.b_mn = b_mn;
  a.batch = (int)batch;
  a.b_in = (int)b_in;
  a.a_bc_out = a_bc_out;
  a.a_bc_in = a_bc_in;
  a.b_bc_out = b_bc_out;
  a.b_bc_in = b_bc_in;
  a.resid = resid;
  B200_REQUIRE(ceil_div(M, BM) <= 65535, "gemm(bf16): M too large");
  CUtensorMap mc, mc2, maux;
  memset(&mc, 0, sizeof(mc));
  memset(&mc2, 0, sizeof(mc2));
  memset(&maux, 0, sizeof(maux));
  a.store_mode = K <= 128 ? 0 : 1;
  if (a.store_mode && M <= INT32_MAX && N <= INT32_MAX) {
    const bool f32 = c_dt == B200_F32;
    bool ok = make_store_map(&mc, C, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, f32 ? 4 : 2, N, M,
                             b_in, b_out, ldc, sC_in, sC_out);
    if (ok && C2) ok = make_store_map(&mc2, C2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, b_in, b_out, ldc, sC_in, sC_out);
    if (ok && aux) ok = make_store_map(&maux, aux, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, M, b_in, b_out, ldc, sC_in, sC_out);
    if (ok) a.store_mode = 2;
  }
#define B200_GEMM_LAUNCH(E)                                                          \
  return pair ? launch<256, E, true>(ma, mb, mc, mc2, maux, a, batch, s)           \
              : (BN == 256 ? launch<256, E, false>(ma, mb, mc, mc2, maux, a, batch, s) \
                           : launch<128, E, false>(ma, mb, mc, mc2, maux, a, batch, s))
  if (epi == B200_EPI_RELU) B200_GEMM_LAUNCH(B200_EPI_RELU);
  if (epi == B200_EPI_GELU) B200_GEMM_LAUNCH(B200_EPI_GELU);
  B200_GEMM_LAUNCH(B200_EPI_NONE);
#undef B200_GEMM_LAUNCH
}

int gemm_bf16_tcgen05(int c_dt, const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N, int64_t K,
                      int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB, int64_t csB, int64_t sC, int64_t ldc,
                      float alpha, const float* bias, int epi, void* aux, cudaStream_t s) {
  return gemm_bf16_tcgen05_b2(c_dt, A, B, C, batch, 1, M, N, K, sA, 0, rsA, csA, sB, 0, rsB, csB, sC, 0, ldc, alpha, bias, epi,
                              aux, nullptr, nullptr, s);
}

}  // namespace b200

using namespace b200;

extern "C" int b200_gemm_batched2(int ab_dt, int c_dt, const void* A, const void* B, void* C, int64_t b_out, int64_t b_in,
                                  int64_t M, int64_t N, int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA,
                                  int64_t sB_out, int64_t sB_in, int64_t rsB, int64_t csB, int64_t sC_out, int64_t sC_in,
                                  int64_t ldc, float alpha, const float* bias, int epi, void* aux, void* C2, void* stream) {
  B200_REQUIRE(A && B && C, "gemm_batched2: null operand");
  B200_REQUIRE(b_out >= 0 && b_in >= 0 && M >= 0 && N >= 0 && K >= 0, "gemm_batched2: negative size");
  B200_REQUIRE(ldc >= N, "gemm_batched2: ldc < N");
  B200_REQUIRE(epi == B200_EPI_NONE || epi == B200_EPI_RELU || epi == B200_EPI_GELU, "gemm_batched2: bad epilogue %d", epi);
  if (c_dt != B200_F32 && c_dt != B200_BF16) {
    set_error("gemm_batched2: output dtype %d", c_dt);
    return B200_ERR_DTYPE;
  }
  if (ab_dt != B200_BF16) {
    set_error("gemm_batched2: tensor-core operands must be bf16 (dtype %d)", ab_dt);
    return B200_ERR_DTYPE;
  }
  if (b_out == 0 || b_in == 0 || M == 0 || N == 0) return B200_OK;
  return gemm_bf16_tcgen05_b2(c_dt, A, B, C, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, sC_out,
                              sC_in, ldc, alpha, bias, epi, aux, C2, nullptr, as_stream(stream));
}

extern "C" int b200_gemm_batched2_residual(const void* A, const void* B, float* C, int64_t b_out, int64_t b_in, int64_t M,
                                           int64_t N, int64_t K, int64_t sA_out, int64_t sA_in, int64_t rsA, int64_t csA,
                                           int64_t sB_out, int64_t sB_in, int64_t rsB, int64_t csB, int64_t sC_out,
                                           int64_t sC_in, int64_t ldc, const float* bias, const float* resid, void* stream) {
  B200_REQUIRE(A && B && C && resid, "gemm_batched2_residual: null operand");
  B200_REQUIRE(b_out >= 0 && b_in >= 0 && M >= 0 && N >= 0 && K >= 0, "gemm_batched2_residual: negative size");
  B200_REQUIRE(ldc >= N, "gemm_batched2_residual: ldc < N");
  if (b_out == 0 || b_in == 0 || M == 0 || N == 0) return B200_OK;
  return gemm_bf16_tcgen05_b2(B200_F32, A, B, C, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, sC_out,
                              sC_in, ldc, 1.f, bias, B200_EPI_NONE, nullptr, nullptr, resid, as_stream(stream));
}

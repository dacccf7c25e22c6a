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
// One CTA computes 128 rows x all N <= 512 columns: A [128, K] and B [N, K] (both K-major,
// K <= 128) arrive by TMA in one shot, one elected thread issues N / 256 x K / 16
// tcgen05.mma into a 128 x 512 fp32 accumulator that fills the whole TMEM, then 8 epilogue
// warps (two per TMEM lane quarter, each owning half of a row's columns) run the row
// reduction in three (forward) or two (backward) passes over TMEM, exchanging their
// partial maxima / sums through shared memory. Rows are written row-per-lane (each lane
// owns a row) as fp32 and / or bf16. Every mbarrier wait is bounded.
#include "tc_common.cuh"

namespace b200 {
namespace attn {

using namespace tc;

constexpr int BMR = 128, NMAX = 512, KMAX = 128, THREADS = 320;  // 2 + 8 warps
constexpr uint32_t A_BYTES = BMR * 64 * 2;                       // one 64-wide K block of A
constexpr uint32_t B_BYTES = 256 * 64 * 2;                       // one 256-row half of B per K block

struct RowArgs {
  int64_t M, N, K;
  int b_in;                                  // z = z_out * b_in + z_in
  int a_bc_out, a_bc_in, b_bc_out, b_bc_in;  // operand shared along a batch level
  const float* scale;                        // device scalar (nullptr: 1)
  // forward outputs / backward input y and outputs: [b_out, b_in, M, N] with strides
  float* y;
  __nv_bfloat16* y_bf16;
  const void* yin;  // backward: y (fp32 or bf16)
  int yin_bf16;
  float* dx;
  __nv_bfloat16* dx_bf16;
  int64_t s_out, s_in, ld;  // element strides of the y / dx tensors
};

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

template <bool BWD>
__global__ void __launch_bounds__(THREADS, 1) rows_kernel(const __grid_constant__ CUtensorMap mapA,
                                                          const __grid_constant__ CUtensorMap mapB, const __grid_constant__ RowArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nkb = (int)((args.K + 63) / 64);  // 1 or 2
  const int nh = args.N > 256 ? 2 : 1;        // 256-column halves
  uint8_t* sA = smem;                         // nkb x 16 KB
  uint8_t* sB = smem + 2 * A_BYTES;           // nkb x nh x 32 KB
  float* red = reinterpret_cast<float*>(sB + 2 * 2 * B_BYTES);  // [2 halves][128 rows]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(red + 2 * BMR);
  uint64_t* mma_bar = full_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BMR;
  const int z = blockIdx.y;
  const int zo = z / args.b_in, zi = z % args.b_in;

  if (threadIdx.x == 0) {
    mbar_init(full_bar, 1);
    mbar_init(mma_bar, 1);
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
      // ---------------- loads: every K block of A and of B's column halves ----------------
      mbar_expect_tx(full_bar, (uint32_t)nkb * (A_BYTES + (uint32_t)nh * B_BYTES));
      const int ai = args.a_bc_in ? 0 : zi, ao = args.a_bc_out ? 0 : zo;
      const int bi = args.b_bc_in ? 0 : zi, bo = args.b_bc_out ? 0 : zo;
      for (int kb = 0; kb < nkb; ++kb) {
        tma_load_4d(sA + kb * A_BYTES, &mapA, full_bar, kb * 64, m0, ai, ao);
        for (int h = 0; h < nh; ++h) tma_load_4d(sB + (kb * 2 + h) * B_BYTES, &mapB, full_bar, kb * 64, h * 256, bi, bo);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA: 128 x (nh * 256) x K into TMEM columns [0, nh * 256) ----------------
      if (mbar_wait(full_bar, 0)) {
        tc_fence_after();
        const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(BMR >> 4) << 24);
        for (int kb = 0; kb < nkb; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (kb * 64 + k * 16 >= args.K) break;
            const uint64_t ad = smem_desc(smem_u32(sA + kb * A_BYTES) + k * 32, 16, 1024);
            for (int h = 0; h < nh; ++h) {
              const uint64_t bd = smem_desc(smem_u32(sB + (kb * 2 + h) * B_BYTES) + k * 32, 16, 1024);
              mma_bf16(tmem_base + (uint32_t)(h * 256), ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
        mma_commit(mma_bar);
      }
    }
  } else {
    // ---------------- epilogue: warps 2..9, quarter q = warp % 4, column half `half` ----------------
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int r = q * 32 + lane;  // row within the tile (= TMEM lane)
    const int64_t row = (int64_t)m0 + r;
    const bool live = row < args.M;
    const int c0 = half * 256;
    const int ncols = (int)max((int64_t)0, min((int64_t)256, args.N - c0));  // this warp's columns
    const float s = args.scale ? __ldg(args.scale) : 1.f;
    // tcgen05.ld is warp-collective: every loop around it runs warp-uniformly (`ok` is made
    // uniform, `live` only guards the stores)
    const bool ok = __all_sync(0xffffffffu, mbar_wait(mma_bar, 0, 64) ? 1 : 0) != 0;
    tc_fence_after();
    const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
    const int64_t yoff = (int64_t)zo * args.s_out + (int64_t)zi * args.s_in + row * args.ld + c0;
    uint32_t v[32];
    if constexpr (!BWD) {
      // pass 1: row max of scale * x
      float mx = -INFINITY;
      for (int c = 0; c < 256; c += 32) {
        if (!ok) break;
        tmem_ld32_issue(tb + (uint32_t)c, v);
        tmem_wait(v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c + i < ncols) mx = fmaxf(mx, s * __uint_as_float(v[i]));
      }
      red[half * BMR + r] = mx;
      named_sync(1 + q, 64);
      mx = fmaxf(red[r], red[BMR + r]);
      named_sync(1 + q, 64);
      // pass 2: sum of exp(scale * x - max)
      float sum = 0.f;
      for (int c = 0; c < 256; c += 32) {
        if (!ok) break;
        tmem_ld32_issue(tb + (uint32_t)c, v);
        tmem_wait(v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c + i < ncols) sum += expf(s * __uint_as_float(v[i]) - mx);
      }
      red[half * BMR + r] = sum;
      named_sync(1 + q, 64);
      sum = red[r] + red[BMR + r];
      // pass 3: y = exp(scale * x - max) / sum
      for (int c = 0; c < 256 && ok; c += 32) {
        tmem_ld32_issue(tb + (uint32_t)c, v);
        tmem_wait(v);
        if (c >= ncols || !live) continue;
        float yv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) yv[i] = expf(s * __uint_as_float(v[i]) - mx) / sum;
        const bool full = c + 32 <= ncols;
        if (args.y) {
          float* dst = args.y + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(yv[i], yv[i + 1], yv[i + 2], yv[i + 3]);
          } else {
            for (int i = 0; i < 32 && c + i < ncols; ++i) dst[i] = yv[i];
          }
        }
        if (args.y_bf16) {
          __nv_bfloat16* dst = args.y_bf16 + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16(yv[i], yv[i + 1]), pack_bf16(yv[i + 2], yv[i + 3]),
                                                              pack_bf16(yv[i + 4], yv[i + 5]), pack_bf16(yv[i + 6], yv[i + 7]));
          } else {
            for (int i = 0; i < 32 && c + i < ncols; ++i) dst[i] = __float2bfloat16_rn(yv[i]);
          }
        }
      }
    } else {
      // y of this row segment, fp32 or bf16
      auto load_y = [&](int c, float (&yv)[32]) {
        const bool full = live && c + 32 <= ncols;
        if (args.yin_bf16) {
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(args.yin) + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              const uint4 u = __ldg(reinterpret_cast<const uint4*>(src + i));
              const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                yv[i + 2 * j] = __uint_as_float(w[j] << 16);
                yv[i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) yv[i] = (c + i < ncols && live) ? __bfloat162float(src[i]) : 0.f;
          }
        } else {
          const float* src = reinterpret_cast<const float*>(args.yin) + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(src) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 f = __ldg(reinterpret_cast<const float4*>(src + i));
              yv[i] = f.x;
              yv[i + 1] = f.y;
              yv[i + 2] = f.z;
              yv[i + 3] = f.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) yv[i] = (c + i < ncols && live) ? __ldg(src + i) : 0.f;
          }
        }
      };
      // pass 1: t = rowsum(G * y)
      float t = 0.f;
      for (int c = 0; c < 256; c += 32) {
        if (!ok) break;
        tmem_ld32_issue(tb + (uint32_t)c, v);
        tmem_wait(v);
        if (c >= ncols) continue;
        float yv[32];
        load_y(c, yv);
#pragma unroll
        for (int i = 0; i < 32; ++i) t += __uint_as_float(v[i]) * yv[i];
      }
      red[half * BMR + r] = t;
      named_sync(1 + q, 64);
      t = red[r] + red[BMR + r];
      // pass 2: dx = scale * y * (G - t)
      for (int c = 0; c < 256 && ok; c += 32) {
        tmem_ld32_issue(tb + (uint32_t)c, v);
        tmem_wait(v);
        if (c >= ncols || !live) continue;
        float yv[32], d[32];
        load_y(c, yv);
#pragma unroll
        for (int i = 0; i < 32; ++i) d[i] = s * (yv[i] * (__uint_as_float(v[i]) - t));
        const bool full = c + 32 <= ncols;
        if (args.dx) {
          float* dst = args.dx + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(d[i], d[i + 1], d[i + 2], d[i + 3]);
          } else {
            for (int i = 0; i < 32 && c + i < ncols; ++i) dst[i] = d[i];
          }
        }
        if (args.dx_bf16) {
          __nv_bfloat16* dst = args.dx_bf16 + yoff + c;
          if (full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i) = make_uint4(pack_bf16(d[i], d[i + 1]), pack_bf16(d[i + 2], d[i + 3]),
                                                              pack_bf16(d[i + 4], d[i + 5]), pack_bf16(d[i + 6], d[i + 7]));
          } else {
            for (int i = 0; i < 32 && c + i < ncols; ++i) dst[i] = __float2bfloat16_rn(d[i]);
          }
        }
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

static size_t smem_bytes() { return 1024 + 2 * A_BYTES + 4 * B_BYTES + 2 * BMR * 4 + 64; }

template <bool BWD>
static int launch_rows(const void* A, const void* B, int64_t b_out, int64_t b_in, int64_t M, int64_t N, int64_t K, int64_t sA_out,
                       int64_t sA_in, int64_t rsA, int64_t csA, int64_t sB_out, int64_t sB_in, int64_t rsB, int64_t csB, RowArgs a,
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
  B200_REQUIRE(b_out * b_in < 65536 && ceil_div(M, BMR) < INT32_MAX, "attn rows: too many tiles");
  if (M == 0) return B200_OK;
  a.M = M;
  a.N = N;
  a.K = K;
  a.b_in = (int)b_in;
  a.a_bc_out = (b_out == 1 || sA_out == 0);
  a.a_bc_in = (b_in == 1 || sA_in == 0);
  a.b_bc_out = (b_out == 1 || sB_out == 0);
  a.b_bc_in = (b_in == 1 || sB_in == 0);
  const uint64_t aIn = a.a_bc_in ? 1 : b_in, aOut = a.a_bc_out ? 1 : b_out;
  const uint64_t bIn = a.b_bc_in ? 1 : b_in, bOut = a.b_bc_out ? 1 : b_out;
  const uint64_t spanA = (uint64_t)rsA * 2 * M, spanB = (uint64_t)csB * 2 * N;
  const uint64_t sAi = a.a_bc_in ? spanA : (uint64_t)sA_in * 2, sAo = a.a_bc_out ? sAi * aIn : (uint64_t)sA_out * 2;
  const uint64_t sBi = a.b_bc_in ? spanB : (uint64_t)sB_in * 2, sBo = a.b_bc_out ? sBi * bIn : (uint64_t)sB_out * 2;
  CUtensorMap ma, mb;
  int rc = make_map(&ma, A, K, M, aIn, aOut, rsA * 2, sAi, sAo, 64, BMR);
  if (rc) return rc;
  rc = make_map(&mb, B, K, N, bIn, bOut, csB * 2, sBi, sBo, 64, 256);
  if (rc) return rc;
  const size_t smem = smem_bytes();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaFuncSetAttribute(rows_kernel<BWD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  dim3 grid((unsigned)ceil_div(M, BMR), (unsigned)(b_out * b_in));
  rows_kernel<BWD><<<grid, THREADS, smem, s>>>(ma, mb, a);
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
  a.y = y;
  a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y_bf16);
  a.s_out = sY_out;
  a.s_in = sY_in;
  a.ld = ldy;
  return attn::launch_rows<false>(A, B, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, a,
                                  as_stream(stream));
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
  a.yin = y;
  a.yin_bf16 = y_dtype == B200_BF16;
  a.dx = dx;
  a.dx_bf16 = reinterpret_cast<__nv_bfloat16*>(dx_bf16);
  a.s_out = s_out;
  a.s_in = s_in;
  a.ld = ld;
  return attn::launch_rows<true>(A, B, b_out, b_in, M, N, K, sA_out, sA_in, rsA, csA, sB_out, sB_in, rsB, csB, a,
                                 as_stream(stream));
}

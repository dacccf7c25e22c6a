// Shared device / host helpers of the tcgen05 kernels (GEMM, attention rows): bounded
// mbarrier waits, TMA tensor loads and stores, UMMA shared-memory descriptors, single-CTA
// MMA issue and commit, TMEM loads, and the bf16 tensor-map encoder.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"

namespace b200 {
namespace tc {

constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait; false (and device error flag set) on timeout. `sleep_ns` backs off
// between polls (for warps that wait a whole main loop, so they do not take issue slots).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int sleep_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (sleep_ns) __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > WAIT_LIMIT_NS) {
      raise_device_error(B200_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 u;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w) : "r"(addr) : "memory");
  return u;
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

// UMMA shared-memory descriptor, SWIZZLE_128B, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// tcgen05.ld of 32 consecutive fp32 columns of this warp's 32 TMEM lanes (asynchronous:
// the registers are valid after tmem_wait, which names them so no use moves above it)
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%"
      "22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
                 "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
                 "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
                 "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Stage a 32 x 32 chunk (lane = row, `w` = the row's 32 elements packed into 32-bit words)
// into a swizzled buffer: ESZ-byte elements, rows of 32 * ESZ bytes, 16-byte pieces XORed
// by the row index (the 128B / 64B / 32B TMA swizzle patterns), so both the row-per-lane
// writes and the row-contiguous reads are free of bank conflicts.
template <int ESZ>
__device__ __forceinline__ void stage_chunk(uint32_t buf, int lane, const uint32_t (&w)[8 * ESZ]) {
  constexpr int PIECES = 2 * ESZ;  // 16-byte pieces per row
  const uint32_t rb = buf + (uint32_t)lane * (32u * ESZ);
  const uint32_t sw = ESZ == 4 ? (uint32_t)(lane & 7) : (ESZ == 2 ? (uint32_t)((lane >> 1) & 3) : (uint32_t)((lane >> 2) & 1));
#pragma unroll
  for (int j = 0; j < PIECES; ++j)
    st_shared_v4(rb + (((uint32_t)j ^ sw) << 4), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// store `n` (<= 16) bytes of a 16-byte piece at dst: one vector store when whole and aligned
__device__ __forceinline__ void put_piece(uint8_t* dst, uint4 u, int64_t n) {
  if (n >= 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    *reinterpret_cast<uint4*>(dst) = u;
    return;
  }
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if ((reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (4 * k + 4 <= n) reinterpret_cast<uint32_t*>(dst)[k] = w[k];
      else {
        for (int b = 4 * k; b < n && b < 4 * k + 4; ++b) dst[b] = (uint8_t)(w[k] >> (8 * (b & 3)));
        break;
      }
    return;
  }
  for (int b = 0; b < 16 && b < n; ++b) dst[b] = (uint8_t)(w[b >> 2] >> (8 * (b & 3)));
}

// Write the staged chunk back row-contiguously: every warp store instruction covers
// 512 / 32 / ... whole row segments. `base` = element (row0, cbase) of the output,
// `ld` = row stride in elements, `rows` / `cols` = how much of the chunk is inside.
template <int ESZ>
__device__ __forceinline__ void write_chunk(uint32_t buf, int lane, uint8_t* base, int64_t ld, int rows, int64_t cols) {
  constexpr int PIECES = 2 * ESZ;         // 16-byte pieces per row
  constexpr int ROWS_PER = 32 / PIECES;   // rows one instruction covers
  const int j = lane % PIECES;
#pragma unroll
  for (int i = 0; i < PIECES; ++i) {
    const int rr = i * ROWS_PER + lane / PIECES;
    if (rr >= rows) continue;
    const uint32_t sw = ESZ == 4 ? (uint32_t)(rr & 7) : (ESZ == 2 ? (uint32_t)((rr >> 1) & 3) : (uint32_t)((rr >> 2) & 1));
    const uint4 u = ld_shared_v4(buf + (uint32_t)rr * (32u * ESZ) + (((uint32_t)j ^ sw) << 4));
    const int64_t left = (cols - (int64_t)j * (16 / ESZ)) * ESZ;  // bytes of this piece inside the row
    if (left <= 0) continue;
    put_piece(base + ((int64_t)rr * ld + (int64_t)j * (16 / ESZ)) * ESZ, u, left);
  }
}


// ---------------------------------------------------------------------------------
// host side: tensor maps
// ---------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 4-D bf16 tensor map: dims (d0 contiguous, d1, d2, d3) with byte strides s1, s2, s3,
// box (b0, b1, 1, 1). Dims of size 1 get a harmless stride equal to the previous extent.
static int make_map(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1,
                    uint64_t s2, uint64_t s3, uint32_t b0, uint32_t b1) {
  auto enc = get_encode();
  if (!enc) {
    set_error("gemm(bf16): cuTensorMapEncodeTiled unavailable");
    return B200_ERR_CUDA;
  }
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1, s2, s3};
  cuuint32_t box[4] = {b0, b1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gemm(bf16): cuTensorMapEncodeTiled failed (%d): dims %llu %llu %llu %llu strides %llu %llu %llu", (int)r,
              (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, (unsigned long long)d3,
              (unsigned long long)s1, (unsigned long long)s2, (unsigned long long)s3);
    return B200_ERR_ARG;
  }
  return B200_OK;
}

// Row-chunk map over a [b_out, b_in, M, N] tensor: dims (N, M, b_in, b_out), byte strides
// (ldc, sC_in, sC_out) * esize, box 32 columns x `box_rows` rows (an epilogue warp's 32 x 32
// chunk, or a 128-row slab), swizzle matching the staged rows (128 B fp32, 64 B bf16, 32 B
// mask rows). False when TMA cannot address it.
static bool make_store_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t esize, int64_t N, int64_t M,
                           int64_t b_in, int64_t b_out, int64_t ldc, int64_t sC_in, int64_t sC_out, uint32_t box_rows = 32) {
  auto enc = get_encode();
  if (!enc || !base || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const uint64_t rowb = (uint64_t)ldc * esize;
  const uint64_t s2 = b_in > 1 ? (uint64_t)sC_in * esize : rowb * (uint64_t)M;
  const uint64_t s3 = b_out > 1 ? (uint64_t)sC_out * esize : s2 * (uint64_t)b_in;
  if (rowb % 16 || s2 % 16 || s3 % 16 || rowb == 0 || s2 == 0 || s3 == 0) return false;
  if (rowb >= (1ull << 40) || s2 >= (1ull << 40) || s3 >= (1ull << 40)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)b_in, (cuuint64_t)b_out};
  cuuint64_t strides[3] = {rowb, s2, s3};
  cuuint32_t box[4] = {32, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw =
      esize == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : (esize == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  return enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace b200

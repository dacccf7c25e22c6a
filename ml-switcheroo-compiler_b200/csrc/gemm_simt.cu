// Exact-fp32 strided batched GEMM on the CUDA cores, with the fused epilogue
// (alpha, per-column bias, ReLU / GELU, optional ReLU mask). This is the path for the
// fp32 workloads, where bf16 tensor-core rounding would break the 1e-4 tolerance; it
// also takes any operand strides (transposes are stride swaps, never materialised).
#include "common.cuh"

namespace b200 {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16, SG_T = 256;

__device__ __forceinline__ float epilogue_apply(float acc, float alpha, const float* bias, int64_t n, int epi) {
  float v = alpha * acc + (bias ? bias[n] : 0.f);
  if (epi == B200_EPI_RELU) v = v > 0.f ? v : 0.f;
  else if (epi == B200_EPI_GELU) v = gelu_tanh(v);
  return v;
}

__global__ void __launch_bounds__(SG_T) gemm_simt_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                         void* __restrict__ C, int c_dt, int64_t M, int64_t N, int64_t K,
                                                         int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB,
                                                         int64_t csB, int64_t sC, int64_t ldc, float alpha,
                                                         const float* __restrict__ bias, int epi, uint8_t* __restrict__ aux) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Bs[SG_BK][SG_BN + 4];
  const int64_t z = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * SG_BM, n0 = (int64_t)blockIdx.x * SG_BN;
  const float* Az = A + z * sA;
  const float* Bz = B + z * sB;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 4 x 4 outputs each
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += SG_BK) {
    // A tile: SG_BM x SG_BK (1024 elements, 4 per thread)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = threadIdx.x + i * SG_T;
      int mm = e / SG_BK, kk = e % SG_BK;
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? Az[gm * rsA + gk * csA] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = threadIdx.x + i * SG_T;
      int kk = e / SG_BN, nn = e % SG_BN;
      int64_t gk = k0 + kk, gn = n0 + nn;
      Bs[kk][nn] = (gk < K && gn < N) ? Bz[gk * rsB + gn * csB] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float pre = alpha * acc[i][j] + (bias ? bias[gn] : 0.f);
      float v = pre;
      if (epi == B200_EPI_RELU) v = pre > 0.f ? pre : 0.f;
      else if (epi == B200_EPI_GELU) v = gelu_tanh(pre);
      int64_t off = z * sC + gm * ldc + gn;
      store_from_f32(C, off, c_dt, v);
      if (aux) aux[off] = pre > 0.f ? 1 : 0;
    }
  }
}

int gemm_bf16_tcgen05(int c_dt, const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N, int64_t K,
                      int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB, int64_t csB, int64_t sC, int64_t ldc,
                      float alpha, const float* bias, int epi, void* aux, cudaStream_t s);

}  // namespace b200

using namespace b200;

extern "C" int b200_gemm(int ab_dt, int c_dt, const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N,
                         int64_t K, int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB, int64_t csB, int64_t sC,
                         int64_t ldc, float alpha, const float* bias, int epi, void* aux, void* stream) {
  B200_REQUIRE(A && B && C, "gemm: null operand");
  B200_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "gemm: negative size");
  B200_REQUIRE(batch <= 65535, "gemm: batch %lld > 65535", (long long)batch);
  B200_REQUIRE(ldc >= N, "gemm: ldc < N");
  B200_REQUIRE(epi == B200_EPI_NONE || epi == B200_EPI_RELU || epi == B200_EPI_GELU, "gemm: bad epilogue %d", epi);
  if (c_dt != B200_F32 && c_dt != B200_BF16) {
    set_error("gemm: output dtype %d", c_dt);
    return B200_ERR_DTYPE;
  }
  if (batch == 0 || M == 0 || N == 0) return B200_OK;
  cudaStream_t s = as_stream(stream);
  if (ab_dt == B200_F32) {
    dim3 grid((unsigned)ceil_div(N, SG_BN), (unsigned)ceil_div(M, SG_BM), (unsigned)batch);
    B200_REQUIRE(ceil_div(M, SG_BM) <= 65535, "gemm: M too large for the fp32 path");
    gemm_simt_kernel<<<grid, SG_T, 0, s>>>((const float*)A, (const float*)B, C, c_dt, M, N, K, sA, rsA, csA, sB, rsB, csB,
                                           sC, ldc, alpha, bias, epi, (uint8_t*)aux);
    return check_launch("gemm(fp32)");
  }
  if (ab_dt == B200_BF16) {
    return gemm_bf16_tcgen05(c_dt, A, B, C, batch, M, N, K, sA, rsA, csA, sB, rsB, csB, sC, ldc, alpha, bias, epi, aux, s);
  }
  set_error("gemm: operand dtype %d", ab_dt);
  return B200_ERR_DTYPE;
}

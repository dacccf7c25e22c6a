// Conv2D forward / input-grad / weight-grad on the tcgen05 tensor cores (bf16 operands,
// fp32 accumulation), as GEMMs over bf16 staging buffers in a caller-provided workspace:
//
//   fwd   : Y_n[O, P]   = Wp[O, Kp] . Xcol_n[Kp, P]        batched over images n,
//                                                          Wp shared (broadcast A)
//   dgrad : dXcol_n     = Wp^T[Kp, O] . dY_n[O, P]        then a gather col2im
//   wgrad : dW[O, Kp]   = sum_s dYt_s[O, L] . XcolT_s[L, Kp]  split-K over (image, pixel)
//                                                          chunks, then a fixed-order sum
//
// P = OH*OW output pixels, K = C*KH*KW taps, Kp / Pp = K / P rounded up to 8 so every
// staged row is 16-byte aligned for TMA. Outputs are written straight in NCHW / OIHW.
// The reference kernels replaced: Conv2D (numpy/eager/conv.py:462-489), Conv2DInputGrad
// (conv.py:634-697), Conv2DWeightGrad (conv.py:699-764); padding follows
// _compute_conv2d_padding_values (conv.py:590-633), passed in as (pt, pl).
#include "common.cuh"

namespace b200 {

int gemm_bf16_tcgen05(int c_dt, const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N, int64_t K,
                      int64_t sA, int64_t rsA, int64_t csA, int64_t sB, int64_t rsB, int64_t csB, int64_t sC, int64_t ldc,
                      float alpha, const float* bias, int epi, void* aux, cudaStream_t s);

namespace cg {

__host__ __device__ inline int64_t rup(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

struct Dims {
  int64_t N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl;
  __host__ __device__ int64_t K() const { return C * KH * KW; }
  __host__ __device__ int64_t Kp() const { return rup(K(), 8); }
  __host__ __device__ int64_t P() const { return OH * OW; }
  __host__ __device__ int64_t Pp() const { return rup(P(), 8); }
};

__device__ __forceinline__ __nv_bfloat16 bf(float v) { return __float2bfloat16_rn(v); }

// w fp32 [O, K] -> wp bf16 [O, Kp]
__global__ void pack_weight_kernel(const float* __restrict__ w, __nv_bfloat16* __restrict__ wp, int64_t O, int64_t K, int64_t Kp) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < O * Kp; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = e / Kp, k = e % Kp;
    wp[e] = bf(k < K ? w[o * K + k] : 0.f);
  }
}

__device__ __forceinline__ float x_at(const float* __restrict__ x, const Dims& d, int64_t n, int64_t k, int64_t p) {
  if (k >= d.K() || p >= d.P()) return 0.f;
  const int64_t c = k / (d.KH * d.KW), i = (k / d.KW) % d.KH, j = k % d.KW;
  const int64_t oh = p / d.OW, ow = p % d.OW;
  const int64_t h = oh * d.sh - d.pt + i, w = ow * d.sw - d.pl + j;
  if (h < 0 || h >= d.H || w < 0 || w >= d.W) return 0.f;
  return x[((n * d.C + c) * d.H + h) * d.W + w];
}

// x -> col bf16 [N, Kp, Pp]   (fwd operand: rows are taps, contiguous pixels)
__global__ void im2col_kp_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ col, Dims d) {
  const int64_t Kp = d.Kp(), Pp = d.Pp(), total = d.N * Kp * Pp;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = e % Pp, k = (e / Pp) % Kp, n = e / (Pp * Kp);
    col[e] = bf(x_at(x, d, n, k, p));
  }
}

// x -> colT bf16 [Q, Kp], row q = n * Pp + p, Q >= N * Pp (zero rows past the data)
__global__ void im2col_pk_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ colT, Dims d, int64_t Q) {
  const int64_t Kp = d.Kp(), Pp = d.Pp(), total = Q * Kp;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = e % Kp, q = e / Kp;
    const int64_t n = q / Pp, p = q % Pp;
    colT[e] = bf(n < d.N ? x_at(x, d, n, k, p) : 0.f);
  }
}

// dy fp32 [N, O, P] -> bf16 [N, O, Pp]
__global__ void pack_dy_nop_kernel(const float* __restrict__ dy, __nv_bfloat16* __restrict__ out, Dims d) {
  const int64_t P = d.P(), Pp = d.Pp(), total = d.N * d.O * Pp;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = e % Pp, no = e / Pp;
    out[e] = bf(p < P ? dy[no * P + p] : 0.f);
  }
}

// dy fp32 [N, O, P] -> bf16 [S, O, L]: split s holds columns q = s * L + l, q = n * Pp + p
// (zero past the data), so each split is a dense [O, L] K-major GEMM operand
__global__ void pack_dy_sol_kernel(const float* __restrict__ dy, __nv_bfloat16* __restrict__ out, Dims d, int64_t S, int64_t L) {
  const int64_t P = d.P(), Pp = d.Pp(), total = S * d.O * L;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t l = e % L, o = (e / L) % d.O, sidx = e / (L * d.O);
    const int64_t q = sidx * L + l;
    const int64_t n = q / Pp, p = q % Pp;
    out[e] = bf((n < d.N && p < P) ? dy[(n * d.O + o) * P + p] : 0.f);
  }
}

// dxcol fp32 [N, Kp, P] -> dx [N, C, H, W]: every input pixel gathers the taps that read it
__global__ void col2im_kernel(const float* __restrict__ dxcol, float* __restrict__ dx, Dims d) {
  const int64_t total = d.N * d.C * d.H * d.W, Kp = d.Kp(), P = d.P();
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t w = e % d.W, h = (e / d.W) % d.H, c = (e / (d.W * d.H)) % d.C, n = e / (d.W * d.H * d.C);
    float acc = 0.f;
    for (int64_t i = 0; i < d.KH; ++i) {
      const int64_t th = h + d.pt - i;
      if (th < 0 || th % d.sh) continue;
      const int64_t oh = th / d.sh;
      if (oh >= d.OH) continue;
      for (int64_t j = 0; j < d.KW; ++j) {
        const int64_t tw = w + d.pl - j;
        if (tw < 0 || tw % d.sw) continue;
        const int64_t ow = tw / d.sw;
        if (ow >= d.OW) continue;
        const int64_t k = (c * d.KH + i) * d.KW + j;
        acc += dxcol[(n * Kp + k) * P + oh * d.OW + ow];
      }
    }
    dx[e] = acc;
  }
}

// partials [S, O, Kp] -> dw [O, K] (sum over S in order, drop the K padding)
__global__ void wgrad_sum_kernel(const float* __restrict__ part, float* __restrict__ dw, int64_t S, int64_t O, int64_t K, int64_t Kp) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < O * K; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = e / K, k = e % K;
    float acc = 0.f;
    for (int64_t s = 0; s < S; ++s) acc += part[(s * O + o) * Kp + k];
    dw[e] = acc;
  }
}

inline unsigned grid_of(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), (int64_t)num_sms() * 32)); }

// split-K plan for wgrad: S chunks of L (multiple of 64) covering Q = S * L >= N * Pp
inline void wgrad_split(const Dims& d, int64_t& S, int64_t& L) {
  const int64_t total = d.N * d.Pp();
  const int64_t tiles = ceil_div(d.O, 128) * ceil_div(d.Kp(), d.Kp() > 128 ? 256 : 128);
  S = std::max<int64_t>(1, std::min<int64_t>(ceil_div(2 * (int64_t)num_sms(), tiles), ceil_div(total, 512)));
  L = rup(ceil_div(total, S), 64);
  S = ceil_div(total, L);
}

inline size_t ws_bytes(int op, const Dims& d) {
  const int64_t Kp = d.Kp(), Pp = d.Pp();
  if (op == 0) return al256((size_t)d.O * Kp * 2) + al256((size_t)d.N * Kp * Pp * 2);
  if (op == 1) return al256((size_t)d.O * Kp * 2) + al256((size_t)d.N * d.O * Pp * 2) + al256((size_t)d.N * Kp * d.P() * 4);
  int64_t S, L;
  wgrad_split(d, S, L);
  const int64_t Q = S * L;
  return al256((size_t)d.O * Q * 2) + al256((size_t)Q * Kp * 2) + al256((size_t)S * d.O * Kp * 4);
}

inline int check(const void* a, const void* b, const void* c, const Dims& d) {
  B200_REQUIRE(a && b && c, "conv2d(tc): null pointer");
  B200_REQUIRE(d.N >= 0 && d.C >= 1 && d.H >= 1 && d.W >= 1 && d.O >= 1 && d.KH >= 1 && d.KW >= 1 && d.OH >= 1 && d.OW >= 1,
               "conv2d(tc): bad sizes");
  B200_REQUIRE(d.sh >= 1 && d.sw >= 1 && d.pt >= 0 && d.pl >= 0, "conv2d(tc): bad stride/padding");
  B200_REQUIRE(d.N * d.Kp() * d.Pp() < (int64_t)1 << 40, "conv2d(tc): staging too large");
  return B200_OK;
}

}  // namespace cg
}  // namespace b200

using namespace b200;
using namespace b200::cg;

#define B200_CONV_DIMS Dims d{N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl}

extern "C" size_t b200_conv2d_tc_workspace_bytes(int op, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH,
                                                 int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                                                 int64_t pl) {
  B200_CONV_DIMS;
  if (op < 0 || op > 2 || N <= 0) return 0;
  return ws_bytes(op, d);
}

extern "C" int b200_conv2d_fwd_tc(const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                                  int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                                  int64_t pl, void* ws, size_t ws_size, void* stream) {
  B200_CONV_DIMS;
  int rc = check(x, w, y, d);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(ws && ws_size >= ws_bytes(0, d), "conv2d_fwd_tc: workspace %zu < %zu", ws_size, ws_bytes(0, d));
  cudaStream_t s = as_stream(stream);
  const int64_t Kp = d.Kp(), Pp = d.Pp(), P = d.P();
  auto* wp = reinterpret_cast<__nv_bfloat16*>(ws);
  auto* col = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(ws) + al256((size_t)O * Kp * 2));
  pack_weight_kernel<<<grid_of(O * Kp), 256, 0, s>>>(w, wp, O, d.K(), Kp);
  if ((rc = check_launch("conv2d_fwd_tc(pack w)"))) return rc;
  im2col_kp_kernel<<<grid_of(N * Kp * Pp), 256, 0, s>>>(x, col, d);
  if ((rc = check_launch("conv2d_fwd_tc(im2col)"))) return rc;
  // Y_n [O, P] = Wp [O, Kp] (shared) . Xcol_n [Kp, Pp]
  return gemm_bf16_tcgen05(B200_F32, wp, col, y, N, O, P, Kp, 0, Kp, 1, Kp * Pp, Pp, 1, O * P, P, 1.f, nullptr,
                           B200_EPI_NONE, nullptr, s);
}

extern "C" int b200_conv2d_dgrad_tc(const float* dy, const float* w, float* dx, int64_t N, int64_t C, int64_t H, int64_t W,
                                    int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                    int64_t pt, int64_t pl, void* ws, size_t ws_size, void* stream) {
  B200_CONV_DIMS;
  int rc = check(dy, w, dx, d);
  if (rc) return rc;
  if (N == 0) return B200_OK;
  B200_REQUIRE(ws && ws_size >= ws_bytes(1, d), "conv2d_dgrad_tc: workspace %zu < %zu", ws_size, ws_bytes(1, d));
  cudaStream_t s = as_stream(stream);
  const int64_t Kp = d.Kp(), Pp = d.Pp(), P = d.P();
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  auto* wp = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)O * Kp * 2);
  auto* dyp = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)N * O * Pp * 2);
  auto* dxcol = reinterpret_cast<float*>(base);
  pack_weight_kernel<<<grid_of(O * Kp), 256, 0, s>>>(w, wp, O, d.K(), Kp);
  if ((rc = check_launch("conv2d_dgrad_tc(pack w)"))) return rc;
  pack_dy_nop_kernel<<<grid_of(N * O * Pp), 256, 0, s>>>(dy, dyp, d);
  if ((rc = check_launch("conv2d_dgrad_tc(pack dy)"))) return rc;
  // dXcol_n [Kp, P] = Wp^T [Kp, O] (shared, MN-major) . dY_n [O, Pp]
  rc = gemm_bf16_tcgen05(B200_F32, wp, dyp, dxcol, N, Kp, P, O, 0, 1, Kp, O * Pp, Pp, 1, Kp * P, P, 1.f, nullptr, B200_EPI_NONE,
                         nullptr, s);
  if (rc) return rc;
  col2im_kernel<<<grid_of(N * C * H * W), 256, 0, s>>>(dxcol, dx, d);
  return check_launch("conv2d_dgrad_tc(col2im)");
}

extern "C" int b200_conv2d_wgrad_tc(const float* x, const float* dy, float* dw, int64_t N, int64_t C, int64_t H, int64_t W,
                                    int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                    int64_t pt, int64_t pl, void* ws, size_t ws_size, void* stream) {
  B200_CONV_DIMS;
  int rc = check(x, dy, dw, d);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  if (N == 0) {
    cudaMemsetAsync(dw, 0, (size_t)O * d.K() * 4, s);
    return check_launch("conv2d_wgrad_tc(empty)");
  }
  B200_REQUIRE(ws && ws_size >= ws_bytes(2, d), "conv2d_wgrad_tc: workspace %zu < %zu", ws_size, ws_bytes(2, d));
  const int64_t Kp = d.Kp();
  int64_t S, L;
  wgrad_split(d, S, L);
  const int64_t Q = S * L;
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  auto* dyt = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)O * Q * 2);
  auto* colT = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)Q * Kp * 2);
  auto* part = reinterpret_cast<float*>(base);
  pack_dy_sol_kernel<<<grid_of(O * Q), 256, 0, s>>>(dy, dyt, d, S, L);
  if ((rc = check_launch("conv2d_wgrad_tc(pack dy)"))) return rc;
  im2col_pk_kernel<<<grid_of(Q * Kp), 256, 0, s>>>(x, colT, d, Q);
  if ((rc = check_launch("conv2d_wgrad_tc(im2col)"))) return rc;
  // partial_s [O, Kp] = dYt_s [O, L] . colT[s L : (s+1) L, :]
  rc = gemm_bf16_tcgen05(B200_F32, dyt, colT, part, S, O, Kp, L, O * L, L, 1, L * Kp, Kp, 1, O * Kp, Kp, 1.f, nullptr,
                         B200_EPI_NONE, nullptr, s);
  if (rc) return rc;
  wgrad_sum_kernel<<<grid_of(O * d.K()), 256, 0, s>>>(part, dw, S, O, d.K(), Kp);
  return check_launch("conv2d_wgrad_tc(sum)");
}

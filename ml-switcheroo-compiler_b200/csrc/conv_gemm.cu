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

// Staging kernels: blockIdx.y / blockIdx.z pick one tap row k (or output channel) and one
// image (or split), so the tap decode (c, i, j) is block-uniform; threads run along the
// contiguous pixel axis with 32-bit divisions only (offsets stay 64-bit).
struct Tap {
  int c, i, j;
};
__device__ __forceinline__ Tap tap_of(const Dims& d, int k) {
  const int khw = (int)(d.KH * d.KW);
  Tap t;
  t.c = k / khw;
  const int r = k - t.c * khw;
  t.i = r / (int)d.KW;
  t.j = r - t.i * (int)d.KW;
  return t;
}
__device__ __forceinline__ float x_tap(const float* __restrict__ x, const Dims& d, int n, const Tap& t, int p) {
  const int OW = (int)d.OW;
  const int oh = p / OW, ow = p - oh * OW;
  const int h = oh * (int)d.sh - (int)d.pt + t.i, w = ow * (int)d.sw - (int)d.pl + t.j;
  if (h < 0 || h >= (int)d.H || w < 0 || w >= (int)d.W) return 0.f;
  return __ldg(x + ((((int64_t)n * d.C + t.c) * d.H + h) * d.W + w));
}

constexpr int NPB = 8;  // images (or channels) one col2im block walks through

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 c = __floats2bfloat162_rn(v[4], v[5]), e = __floats2bfloat162_rn(v[6], v[7]);
  return make_uint4(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b), *reinterpret_cast<uint32_t*>(&c),
                    *reinterpret_cast<uint32_t*>(&e));
}

// The staging kernels below walk their output as one flat array of 8-element groups:
// every group lies inside one row (Pp and L are multiples of 8), is decoded once, and
// leaves as one 16-byte store; a grid-stride loop covers the groups.

// x -> col bf16 [N, Kp, Pp]   (fwd operand: rows are taps, contiguous pixels)
__global__ void __launch_bounds__(256) im2col_kp_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ col, Dims d) {
  const int64_t Kp = d.Kp(), Pp = d.Pp(), P = d.P(), K = d.K();
  const int64_t groups = d.N * Kp * Pp / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = g * 8;
    const int p0 = (int)(e % Pp);
    const int64_t nk = e / Pp;
    const int k = (int)(nk % Kp), n = (int)(nk / Kp);
    float v[8];
    if (k < K) {
      const Tap t = tap_of(d, k);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (p0 + i < P) ? x_tap(x, d, n, t, p0 + i) : 0.f;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    *reinterpret_cast<uint4*>(col + e) = pack8(v);
  }
}

// x -> col bf16 [S, Kp, L]: split s holds pixels q = s * L + l, q = n * Pp + p (zero past
// the data), so each split is a dense K-major weight-gradient operand
__global__ void __launch_bounds__(256) im2col_kq_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ col, Dims d,
                                                        int64_t L, int64_t S) {
  const int64_t Kp = d.Kp(), Pp = d.Pp(), P = d.P(), K = d.K();
  const int64_t groups = S * Kp * L / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = g * 8;
    const int64_t l0 = e % L, sk = e / L;
    const int k = (int)(sk % Kp);
    const int64_t sidx = sk / Kp;
    const int64_t q0 = sidx * L + l0;  // 8 consecutive pixels of one image (Pp % 8 == 0)
    const int n = (int)(q0 / Pp), p0 = (int)(q0 - (int64_t)n * Pp);
    float v[8];
    if (k < K && n < d.N) {
      const Tap t = tap_of(d, k);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (p0 + i < P) ? x_tap(x, d, n, t, p0 + i) : 0.f;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    *reinterpret_cast<uint4*>(col + e) = pack8(v);
  }
}

// dy fp32 [N, O, P] -> bf16 [N, O, Pp]
__global__ void __launch_bounds__(256) pack_dy_nop_kernel(const float* __restrict__ dy, __nv_bfloat16* __restrict__ out, Dims d) {
  const int64_t P = d.P(), Pp = d.Pp();
  const int64_t groups = d.N * d.O * Pp / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = g * 8;
    const int64_t no = e / Pp;
    const int p0 = (int)(e - no * Pp);
    const float* src = dy + no * P;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (p0 + i < P) ? __ldg(src + p0 + i) : 0.f;
    *reinterpret_cast<uint4*>(out + e) = pack8(v);
  }
}

// dy fp32 [N, O, P] -> bf16 [S, O, L]: split s holds columns q = s * L + l, q = n * Pp + p
// (zero past the data), so each split is a dense [O, L] K-major GEMM operand
__global__ void __launch_bounds__(256) pack_dy_sol_kernel(const float* __restrict__ dy, __nv_bfloat16* __restrict__ out, Dims d,
                                                          int64_t L, int64_t S) {
  const int64_t P = d.P(), Pp = d.Pp(), O = d.O;
  const int64_t groups = S * O * L / 8;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = g * 8;
    const int64_t l0 = e % L, so = e / L;
    const int64_t o = so % O, sidx = so / O;
    const int64_t q0 = sidx * L + l0;
    const int64_t n = q0 / Pp;
    const int p0 = (int)(q0 - n * Pp);
    float v[8];
    if (n < d.N) {
      const float* src = dy + (n * O + o) * P;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (p0 + i < P) ? __ldg(src + p0 + i) : 0.f;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    *reinterpret_cast<uint4*>(out + e) = pack8(v);
  }
}

// dxcol fp32 [N, Kp, P] -> dx [N, C, H, W]: every input pixel gathers the taps that read it
__device__ __forceinline__ void col2im_one(const float* __restrict__ dxcol, float* __restrict__ dx, const Dims& d, int hw, int c,
                                           int n) {
  const int H = (int)d.H, W = (int)d.W;
  const int h = hw / W, w = hw - h * W;
  const int KH = (int)d.KH, KW = (int)d.KW, sh = (int)d.sh, sw = (int)d.sw, OH = (int)d.OH, OW = (int)d.OW;
  const int P = OH * OW;
  const float* base = dxcol + ((int64_t)n * d.Kp()) * P;
  float acc = 0.f;
  for (int i = 0; i < KH; ++i) {
    const int th = h + (int)d.pt - i;
    if (th < 0) break;  // th only decreases as i grows
    const int oh = th / sh;
    if (oh * sh != th || oh >= OH) continue;
    for (int j = 0; j < KW; ++j) {
      const int tw = w + (int)d.pl - j;
      if (tw < 0) break;
      const int ow = tw / sw;
      if (ow * sw != tw || ow >= OW) continue;
      const int k = (c * KH + i) * KW + j;
      acc += __ldg(base + (int64_t)k * P + oh * OW + ow);
    }
  }
  dx[(((int64_t)n * d.C + c) * H) * W + hw] = acc;
}

// grid (ceil(H W / 256), C, ceil(N / NPB))
__global__ void __launch_bounds__(256) col2im_kernel(const float* __restrict__ dxcol, float* __restrict__ dx, Dims d) {
  const int hw = blockIdx.x * 256 + threadIdx.x, c = blockIdx.y;
  if (hw >= (int)(d.H * d.W)) return;
  const int n1 = min((int)d.N, (int)(blockIdx.z + 1) * NPB);
  for (int n = blockIdx.z * NPB; n < n1; ++n) col2im_one(dxcol, dx, d, hw, c, n);
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
  return al256((size_t)d.O * Q * 2) + al256((size_t)S * Kp * L * 2) + al256((size_t)S * d.O * Kp * 4);
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
  im2col_kp_kernel<<<grid_of(N * Kp * Pp / 8), 256, 0, s>>>(x, col, d);
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
  B200_REQUIRE(O <= 65535 && N <= 65535 && C <= 65535, "conv2d_dgrad_tc: too many channels or images");
  pack_dy_nop_kernel<<<grid_of(N * O * Pp / 8), 256, 0, s>>>(dy, dyp, d);
  if ((rc = check_launch("conv2d_dgrad_tc(pack dy)"))) return rc;
  // dXcol_n [Kp, P] = Wp^T [Kp, O] (shared, MN-major) . dY_n [O, Pp]
  rc = gemm_bf16_tcgen05(B200_F32, wp, dyp, dxcol, N, Kp, P, O, 0, 1, Kp, O * Pp, Pp, 1, Kp * P, P, 1.f, nullptr, B200_EPI_NONE,
                         nullptr, s);
  if (rc) return rc;
  col2im_kernel<<<dim3((unsigned)ceil_div(H * W, (int64_t)256), (unsigned)C, (unsigned)ceil_div(N, (int64_t)NPB)), 256, 0, s>>>(
      dxcol, dx, d);
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
  auto* col = reinterpret_cast<__nv_bfloat16*>(base);
  base += al256((size_t)S * Kp * L * 2);
  auto* part = reinterpret_cast<float*>(base);
  pack_dy_sol_kernel<<<grid_of(S * O * L / 8), 256, 0, s>>>(dy, dyt, d, L, S);
  if ((rc = check_launch("conv2d_wgrad_tc(pack dy)"))) return rc;
  im2col_kq_kernel<<<grid_of(S * Kp * L / 8), 256, 0, s>>>(x, col, d, L, S);
  if ((rc = check_launch("conv2d_wgrad_tc(im2col)"))) return rc;
  // partial_s [O, Kp] = dYt_s [O, L] . col_s^T   (col_s [Kp, L]: K-major B operand)
  rc = gemm_bf16_tcgen05(B200_F32, dyt, col, part, S, O, Kp, L, O * L, L, 1, Kp * L, 1, L, O * Kp, Kp, 1.f, nullptr,
                         B200_EPI_NONE, nullptr, s);
  if (rc) return rc;
  wgrad_sum_kernel<<<grid_of(O * d.K()), 256, 0, s>>>(part, dw, S, O, d.K(), Kp);
  return check_launch("conv2d_wgrad_tc(sum)");
}

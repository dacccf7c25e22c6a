// Conv2D forward / input-grad / weight-grad (NCHW x OIHW, stride, explicit zero padding,
// groups = dilation = 1). Direct formulation on the CUDA cores with fp32 accumulation;
// with ab_dtype BF16 the operands are rounded to bf16 before the multiply, matching the
// bf16 conv-math policy of the CNN workload.
#include "common.cuh"

namespace b200 {

__device__ __forceinline__ float rnd(float v, int bf) { return bf ? __bfloat162float(__float2bfloat16_rn(v)) : v; }

__global__ void conv_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y, int64_t N,
                                int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                                int64_t sh, int64_t sw, int64_t pt, int64_t pl, int bf) {
  const int64_t total = N * O * OH * OW;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ow = e % OW, oh = (e / OW) % OH, o = (e / (OW * OH)) % O, n = e / (OW * OH * O);
    float acc = 0.f;
    for (int64_t c = 0; c < C; ++c)
      for (int64_t i = 0; i < KH; ++i) {
        const int64_t h = oh * sh - pt + i;
        if (h < 0 || h >= H) continue;
        for (int64_t j = 0; j < KW; ++j) {
          const int64_t ww = ow * sw - pl + j;
          if (ww < 0 || ww >= W) continue;
          acc = fmaf(rnd(x[((n * C + c) * H + h) * W + ww], bf), rnd(w[((o * C + c) * KH + i) * KW + j], bf), acc);
        }
      }
    y[e] = acc;
  }
}

__global__ void conv_dgrad_kernel(const float* __restrict__ dy, const float* __restrict__ w, float* __restrict__ dx, int64_t N,
                                  int64_t C, int64_t H, int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW,
                                  int64_t sh, int64_t sw, int64_t pt, int64_t pl, int bf) {
  const int64_t total = N * C * H * W;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t ww = e % W, h = (e / W) % H, c = (e / (W * H)) % C, n = e / (W * H * C);
    float acc = 0.f;
    for (int64_t i = 0; i < KH; ++i) {
      const int64_t th = h + pt - i;
      if (th < 0 || th % sh) continue;
      const int64_t oh = th / sh;
      if (oh >= OH) continue;
      for (int64_t j = 0; j < KW; ++j) {
        const int64_t tw = ww + pl - j;
        if (tw < 0 || tw % sw) continue;
        const int64_t ow = tw / sw;
        if (ow >= OW) continue;
        for (int64_t o = 0; o < O; ++o)
          acc = fmaf(rnd(dy[((n * O + o) * OH + oh) * OW + ow], bf), rnd(w[((o * C + c) * KH + i) * KW + j], bf), acc);
      }
    }
    dx[e] = acc;
  }
}

// one CTA per weight element; threads split the N*OH*OW sum, block reduction at the end
__global__ void __launch_bounds__(256) conv_wgrad_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                         float* __restrict__ dw, int64_t N, int64_t C, int64_t H, int64_t W,
                                                         int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh,
                                                         int64_t sw, int64_t pt, int64_t pl, int bf) {
  __shared__ float sred[32];
  const int64_t e = blockIdx.x;
  const int64_t j = e % KW, i = (e / KW) % KH, c = (e / (KW * KH)) % C, o = e / (KW * KH * C);
  float acc = 0.f;
  const int64_t P = N * OH * OW;
  for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
    const int64_t ow = p % OW, oh = (p / OW) % OH, n = p / (OW * OH);
    const int64_t h = oh * sh - pt + i, ww = ow * sw - pl + j;
    if (h < 0 || h >= H || ww < 0 || ww >= W) continue;
    acc = fmaf(rnd(x[((n * C + c) * H + h) * W + ww], bf), rnd(dy[((n * O + o) * OH + oh) * OW + ow], bf), acc);
  }
  const float t = block_sum(acc, sred);
  if (threadIdx.x == 0) dw[e] = t;
}

static unsigned grid_for(int64_t n) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), (int64_t)num_sms() * 16));
}

static int check_conv(const void* a, const void* b, const void* c, int64_t N, int64_t C, int64_t H, int64_t W, int64_t O,
                      int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt, int64_t pl,
                      int ab) {
  B200_REQUIRE(a && b && c, "conv2d: null pointer");
  B200_REQUIRE(N >= 0 && C >= 1 && H >= 1 && W >= 1 && O >= 1 && KH >= 1 && KW >= 1 && OH >= 0 && OW >= 0,
               "conv2d: bad sizes");
  B200_REQUIRE(sh >= 1 && sw >= 1 && pt >= 0 && pl >= 0, "conv2d: bad stride/padding");
  B200_REQUIRE((OH - 1) * sh + KH <= H + 2 * pt + sh && (OW - 1) * sw + KW <= W + 2 * pl + sw, "conv2d: output too large");
  if (ab != B200_F32 && ab != B200_BF16) {
    set_error("conv2d: math dtype %d", ab);
    return B200_ERR_DTYPE;
  }
  return B200_OK;
}

}  // namespace b200

using namespace b200;

extern "C" int b200_conv2d_fwd(int ab, const float* x, const float* w, float* y, int64_t N, int64_t C, int64_t H, int64_t W,
                               int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw, int64_t pt,
                               int64_t pl, void* stream) {
  int rc = check_conv(x, w, y, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl, ab);
  if (rc) return rc;
  const int64_t total = N * O * OH * OW;
  if (total == 0) return B200_OK;
  conv_fwd_kernel<<<grid_for(total), 256, 0, as_stream(stream)>>>(x, w, y, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl,
                                                                  ab == B200_BF16);
  return check_launch("conv2d_fwd");
}

extern "C" int b200_conv2d_dgrad(int ab, const float* dy, const float* w, float* dx, int64_t N, int64_t C, int64_t H,
                                 int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                 int64_t pt, int64_t pl, void* stream) {
  int rc = check_conv(dy, w, dx, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl, ab);
  if (rc) return rc;
  const int64_t total = N * C * H * W;
  if (total == 0) return B200_OK;
  conv_dgrad_kernel<<<grid_for(total), 256, 0, as_stream(stream)>>>(dy, w, dx, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl,
                                                                    ab == B200_BF16);
  return check_launch("conv2d_dgrad");
}

extern "C" int b200_conv2d_wgrad(int ab, const float* x, const float* dy, float* dw, int64_t N, int64_t C, int64_t H,
                                 int64_t W, int64_t O, int64_t KH, int64_t KW, int64_t OH, int64_t OW, int64_t sh, int64_t sw,
                                 int64_t pt, int64_t pl, void* stream) {
  int rc = check_conv(x, dy, dw, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl, ab);
  if (rc) return rc;
  const int64_t total = O * C * KH * KW;
  B200_REQUIRE(total <= 2147483647LL, "conv2d_wgrad: too many weights");
  conv_wgrad_kernel<<<(unsigned)total, 256, 0, as_stream(stream)>>>(x, dy, dw, N, C, H, W, O, KH, KW, OH, OW, sh, sw, pt, pl,
                                                                   ab == B200_BF16);
  return check_launch("conv2d_wgrad");
}

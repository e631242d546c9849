// 1-D convolution (cross-correlation) over a batch of (C_in, T) signals, as an
// implicit GEMM on the CUDA cores: out[b][co][t] = bias[co] +
//   sum_{ci < C_in/g, j < k} W[co][ci][j] * x[b][g*C_in/g + ci][t*stride + j*dil - pad_l]
// Replaces cv3cpu/ops.py:165-219 (conv1d, im2col + BLAS) for the plain-weight
// case; zero padding is implicit in the index test, the right pad only sets T_out.
// Tile: 64 output channels x 64 frames per CTA, 4x4 per thread, K-steps of 16
// (ci, j) pairs staged through shared memory.
#include "common.cuh"

namespace {

constexpr int TC = 64, TT = 64, TK = 16;

__global__ void __launch_bounds__(256)
conv1d_kernel(const float* __restrict__ x, int cin, int t_in, const float* __restrict__ w, int cout, int cin_g,
              int k, int stride, int dil, int pad_l, int groups, const float* __restrict__ bias, float* __restrict__ y,
              int t_out) {
  __shared__ float Ws[TK][TC + 4];
  __shared__ float Xs[TK][TT + 4];
  const int cout_g = cout / groups;
  const int g = blockIdx.z % groups, b = blockIdx.z / groups;
  const int co0 = blockIdx.y * TC, t0 = blockIdx.x * TT;
  const int kk_total = cin_g * k;
  const float* xb = x + ((int64_t)b * cin + (int64_t)g * cin_g) * t_in;
  const float* wg = w + (int64_t)g * cout_g * kk_total;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < kk_total; k0 += TK) {
    for (int i = threadIdx.x; i < TC * TK; i += 256) {
      const int r = i / TK, c = i - r * TK;
      const int co = co0 + r, kk = k0 + c;
      Ws[c][r] = (co < cout_g && kk < kk_total) ? wg[(int64_t)co * kk_total + kk] : 0.f;
    }
    for (int i = threadIdx.x; i < TK * TT; i += 256) {
      const int c = i / TT, tt = i - c * TT;
      const int kk = k0 + c, t = t0 + tt;
      float v = 0.f;
      if (kk < kk_total && t < t_out) {
        const int ci = kk / k, j = kk - ci * k;
        const int ti = t * stride + j * dil - pad_l;
        if (ti >= 0 && ti < t_in) v = xb[(int64_t)ci * t_in + ti];
      }
      Xs[c][tt] = v;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < TK; ++c) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = Ws[c][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Xs[c][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* yb = y + ((int64_t)b * cout + (int64_t)g * cout_g) * t_out;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int co = co0 + ty * 4 + i;
    if (co >= cout_g) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = t0 + tx * 4 + j;
      if (t >= t_out) continue;
      float o = acc[i][j];
      if (bias) o += bias[g * cout_g + co];
      yb[(int64_t)co * t_out + t] = o;
    }
  }
}

}  // namespace

extern "C" int cv3_conv1d(const float* x, int64_t batch, int64_t cin, int64_t t_in, const float* w, int64_t cout,
                          int64_t k, int64_t stride, int64_t dilation, int64_t groups, int64_t pad_left,
                          int64_t pad_right, const float* bias, float* y, int64_t t_out, void* stream) {
  CV3_REQUIRE(batch >= 0 && cin > 0 && cout > 0 && k > 0 && stride > 0 && dilation > 0 && groups > 0,
              CV3_ERR_VALUE, "conv1d: bad geometry");
  CV3_REQUIRE(cin % groups == 0 && cout % groups == 0, CV3_ERR_VALUE,
              "conv1d: channels %lld/%lld not divisible by groups %lld", (long long)cin, (long long)cout,
              (long long)groups);
  CV3_REQUIRE(pad_left >= 0 && pad_right >= 0, CV3_ERR_VALUE, "conv1d: negative padding");
  const int64_t span = dilation * (k - 1) + 1;
  const int64_t expect = (t_in + pad_left + pad_right - span) / stride + 1;
  CV3_REQUIRE(t_out == (expect > 0 ? expect : 0), CV3_ERR_VALUE, "conv1d: t_out %lld != %lld",
              (long long)t_out, (long long)expect);
  if (batch == 0 || t_out == 0) return CV3_OK;
  CV3_REQUIRE(t_in < (1LL << 30) && cin * k < (1LL << 30), CV3_ERR_VALUE, "conv1d: too large");
  dim3 grid((unsigned)((t_out + TT - 1) / TT), (unsigned)((cout / groups + TC - 1) / TC), (unsigned)(batch * groups));
  CV3_REQUIRE(grid.y <= 65535 && grid.z <= 65535, CV3_ERR_VALUE, "conv1d: grid too large");
  conv1d_kernel<<<grid, 256, 0, cv3::as_stream(stream)>>>(x, (int)cin, (int)t_in, w, (int)cout, (int)(cin / groups),
                                                          (int)k, (int)stride, (int)dilation, (int)pad_left,
                                                          (int)groups, bias, y, (int)t_out);
  return cv3::check_launch("conv1d");
}

// Elementwise activations and row reductions (norms, softmax), fp32.
// Each follows the arithmetic order of the reference op it replaces
// (cv3cpu/ops.py:30-118); transcendentals use CUDA's IEEE-accurate single
// precision functions (no fast-math), the snake its own branch-free squared sine
// (snake.cuh).
#include "common.cuh"
#include "snake.cuh"

namespace {


__global__ void unary_kernel(int act, float p, const float* __restrict__ x, int64_t n, float* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = act_apply(act, p, x[i]);
}

__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, int dim, float eps,
                                float* __restrict__ y) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * dim;
  float* yr = y + (int64_t)blockIdx.x * dim;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i] * xr[i];
  s = block_sum(s, red);
  const float r = 1.0f / sqrtf(s / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = (xr[i] * r) * w[i];
}

__global__ void layer_norm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                  const float* __restrict__ b, int dim, float eps, float* __restrict__ y) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * dim;
  float* yr = y + (int64_t)blockIdx.x * dim;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i];
  const float mu = block_sum(s, red) / (float)dim;
  float v = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float c = xr[i] - mu;
    v += c * c;
  }
  const float sd = sqrtf(block_sum(v, red) / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float o = (xr[i] - mu) / sd;
    if (w) o = o * w[i];
    if (b) o = o + b[i];
    yr[i] = o;
  }
}

__global__ void softmax_kernel(const float* __restrict__ x, int dim, int lg, float* __restrict__ y) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * dim;
  float* yr = y + (int64_t)blockIdx.x * dim;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) m = fmaxf(m, xr[i]);
  m = block_max(m, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += expf(xr[i] - m);
  s = block_sum(s, red);
  if (lg) {
    const float ls = logf(s);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = (xr[i] - m) - ls;
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = expf(xr[i] - m) / s;
  }
}

__global__ void snake_kernel(const float* __restrict__ x, const float* __restrict__ alpha, int64_t channels, int64_t t,
                             int64_t total, float* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float a = alpha[(i / t) % channels];
    const float v = x[i];
    y[i] = cv3snake::snake_combine(v, cv3snake::inv_alpha(a), cv3snake::sin_sq(__fmul_rn(a, v)));
  }
}

int row_threads(int64_t dim) {
  int t = 32;
  while (t < dim && t < 1024) t <<= 1;
  return t;
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)cv3::sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" int cv3_unary(int act, float param, const float* x, int64_t n, float* y, void* stream) {
  CV3_REQUIRE(act >= CV3_ACT_SILU && act <= CV3_ACT_EXP, CV3_ERR_VALUE, "unary: unknown activation %d", act);
  CV3_REQUIRE(n >= 0, CV3_ERR_VALUE, "unary: negative size");
  if (n == 0) return CV3_OK;
  unary_kernel<<<grid_for(n, 256), 256, 0, cv3::as_stream(stream)>>>(act, param, x, n, y);
  return cv3::check_launch("unary");
}

extern "C" int cv3_rms_norm(const float* x, const float* w, int64_t rows, int64_t dim, float eps, float* y,
                            void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0 && rows < (1LL << 31) && dim < (1LL << 31), CV3_ERR_VALUE, "rms_norm: bad shape");
  if (rows == 0) return CV3_OK;
  rms_norm_kernel<<<(unsigned)rows, row_threads(dim), 0, cv3::as_stream(stream)>>>(x, w, (int)dim, eps, y);
  return cv3::check_launch("rms_norm");
}

extern "C" int cv3_layer_norm(const float* x, const float* w, const float* b, int64_t rows, int64_t dim,
                              float eps, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0 && rows < (1LL << 31) && dim < (1LL << 31), CV3_ERR_VALUE, "layer_norm: bad shape");
  if (rows == 0) return CV3_OK;
  layer_norm_kernel<<<(unsigned)rows, row_threads(dim), 0, cv3::as_stream(stream)>>>(x, w, b, (int)dim, eps, y);
  return cv3::check_launch("layer_norm");
}

extern "C" int cv3_softmax(const float* x, int64_t rows, int64_t dim, int lg, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0 && rows < (1LL << 31) && dim < (1LL << 31), CV3_ERR_VALUE, "softmax: bad shape");
  if (rows == 0) return CV3_OK;
  softmax_kernel<<<(unsigned)rows, row_threads(dim), 0, cv3::as_stream(stream)>>>(x, (int)dim, lg, y);
  return cv3::check_launch("softmax");
}

extern "C" int cv3_snake(const float* x, const float* alpha, int64_t batch, int64_t channels, int64_t t, float* y,
                         void* stream) {
  CV3_REQUIRE(batch >= 0 && channels > 0 && t >= 0, CV3_ERR_VALUE, "snake: bad shape");
  const int64_t total = batch * channels * t;
  if (total == 0) return CV3_OK;
  snake_kernel<<<grid_for(total, 256), 256, 0, cv3::as_stream(stream)>>>(x, alpha, channels, t, total, y);
  return cv3::check_launch("snake");
}

// DiT flow-estimator glue kernels (cv3cpu/models/dit.py, cv3cpu/models/flow.py).
//
// Activations are token-major [batch][frames][channels]; the mel-side tensors
// (x, mu, cond and the velocity) keep the reference's channel-major (80, N)
// layout and are converted inside the kernels that touch them, so no separate
// transpose pass runs per step.  Elementwise formulas keep the reference's
// operation order (explicit round-to-nearest multiply/add where NumPy would
// round twice) so that only GEMM/attention summation order differs.
#include "common.cuh"
#include "planes.cuh"

namespace {

__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }

// cat[b][n][0:80|80:160|160:240|240:320] = x, cond, mu (channel-major inputs), spk
// for the CFG batch: b = 2u keeps utterance u's conditioning, b = 2u+1 zeroes it
// (flow.py:71-77, dit.py:92-97).
__global__ void input_cat_kernel(const float* __restrict__ x, const float* __restrict__ cond,
                                 const float* __restrict__ mu, const float* __restrict__ spk, int utts, int n,
                                 int mel, int spk_dim, float* __restrict__ out) {
  const int width = 3 * mel + spk_dim;
  const int64_t total = (int64_t)2 * utts * n * width;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % width);
    const int64_t r = i / width;
    const int t = (int)(r % n);
    const int b = (int)(r / n);
    const int u = b >> 1;
    const bool uncond = b & 1;
    float v;
    if (c < mel) v = x[((int64_t)u * mel + c) * n + t];
    else if (c < 2 * mel) v = uncond ? 0.f : cond[((int64_t)u * mel + (c - mel)) * n + t];
    else if (c < 3 * mel) v = uncond ? 0.f : mu[((int64_t)u * mel + (c - 2 * mel)) * n + t];
    else v = uncond ? 0.f : spk[(int64_t)u * spk_dim + (c - 3 * mel)];
    out[i] = v;
  }
}

// y = layer_norm(h, eps) * (1 + scale) + shift, no affine (dit.py:168-169, ops.py:107-118).
// One CTA per row; scale/shift rows chosen by row / rows_per_group.
__global__ void ln_modulate_kernel(const float* __restrict__ h, int dim, float eps, const float* __restrict__ scale,
                                   const float* __restrict__ shift, int64_t rows_per_group, int64_t mod_stride,
                                   float* __restrict__ y) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const float* x = h + r * dim;
  float* o = y + r * dim;
  const int64_t g = rows_per_group > 0 ? r / rows_per_group : 0;
  const float* sc = scale + g * mod_stride;
  const float* sh = shift + g * mod_stride;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += x[i];
  const float mu = block_sum(s, red) / (float)dim;
  float v = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float c = x[i] - mu;
    v += c * c;
  }
  const float sd = sqrtf(block_sum(v, red) / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    const float nrm = (x[i] - mu) / sd;
    o[i] = add(mul(nrm, add(1.0f, sc[i])), sh[i]);
  }
}

// ln_modulate_kernel for dim = 128 * V: one warp per row, the row in registers (V
// float4 per lane, one coalesced read), mean and variance by warp shuffles (no
// block barriers), same formulas; 8 rows per CTA.  PLANES: the result goes out as
// activation planes (planes.cuh) for cv3_tc_gemm_q8_planes instead of fp32 -- float4
// j of a lane holds columns 4 (lane + 32 j) .., so each half warp covers one 64-wide
// group, whose exponent is a 16-lane max.
template <int V, bool PLANES>
__global__ void __launch_bounds__(256) ln_modulate_warp_kernel(const float* __restrict__ h, int64_t rows, float eps,
                                                               const float* __restrict__ scale,
                                                               const float* __restrict__ shift,
                                                               int64_t rows_per_group, int64_t mod_stride,
                                                               float* __restrict__ y, __half* __restrict__ planes,
                                                               int8_t* __restrict__ exps, int64_t lde) {
  constexpr int DIM = 128 * V;
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float4* x4 = reinterpret_cast<const float4*>(h + r * DIM);
  float4 v[V];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    v[j] = x4[lane + 32 * j];
    s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  }
  const float mu = warp_sum(s) / (float)DIM;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const float a = v[j].x - mu, b = v[j].y - mu, c = v[j].z - mu, d = v[j].w - mu;
    q += (a * a + b * b) + (c * c + d * d);
  }
  const float sd = sqrtf(warp_sum(q) / (float)DIM + eps);
  const int64_t g = rows_per_group > 0 ? r / rows_per_group : 0;
  const float4* sc4 = reinterpret_cast<const float4*>(scale + g * mod_stride);
  const float4* sh4 = reinterpret_cast<const float4*>(shift + g * mod_stride);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const float4 sc = __ldg(sc4 + lane + 32 * j), sh = __ldg(sh4 + lane + 32 * j);
    float4 o;
    o.x = add(mul((v[j].x - mu) / sd, add(1.0f, sc.x)), sh.x);
    o.y = add(mul((v[j].y - mu) / sd, add(1.0f, sc.y)), sh.y);
    o.z = add(mul((v[j].z - mu) / sd, add(1.0f, sc.z)), sh.z);
    o.w = add(mul((v[j].w - mu) / sd, add(1.0f, sc.w)), sh.w);
    if (!PLANES) {
      reinterpret_cast<float4*>(y + r * DIM)[lane + 32 * j] = o;
    } else {
      float am = fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w)));
#pragma unroll
      for (int m = 1; m < 16; m <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, m));
      const int e = cv3p::group_exponent(am);
      const float f = cv3p::pow2f(e);
      const int g = 2 * j + (lane >> 4), c = 4 * (lane & 15);
      uint32_t h0, l0, h1, l1;
      cv3p::split_pair(o.x * f, o.y * f, h0, l0);
      cv3p::split_pair(o.z * f, o.w * f, h1, l1);
      __half* pr = planes + r * (2 * DIM) + 128 * g + c;
      *reinterpret_cast<uint2*>(pr) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(pr + 64) = make_uint2(l0, l1);
      if ((lane & 15) == 0) exps[(int64_t)g * lde + r] = (int8_t)e;
    }
  }
}

// h += gate * y  (dit.py:170, :173): rows of width dim, gate per group of rows.
__global__ void gate_residual_kernel(float* __restrict__ h, const float* __restrict__ y, const float* __restrict__ gate,
                                     int64_t rows, int dim, int64_t rows_per_group, int64_t gate_stride) {
  const int64_t total = rows * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / dim;
    const int c = (int)(i - r * dim);
    const int64_t g = rows_per_group > 0 ? r / rows_per_group : 0;
    h[i] = add(h[i], mul(gate[g * gate_stride + c], y[i]));
  }
}

// Interleaved-pair rotation of channels [0, width) of q and k inside fused qkv
// rows (dit.py:32-54): (x0, x1) -> (x0 c0 - x1 s0, x1 c1 + x0 s1), position =
// row % frames, tables [frames][width].
__global__ void partial_rope_kernel(float* __restrict__ qkv, int64_t rows, int64_t ld, int64_t k_off, int frames,
                                    int width, const float* __restrict__ cosT, const float* __restrict__ sinT) {
  const int pairs = width / 2;
  const int64_t total = rows * pairs * 2;  // q and k
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int which = (int)(i % 2);
    const int64_t j = i / 2;
    const int p = (int)(j % pairs);
    const int64_t r = j / pairs;
    const int n = (int)(r % frames);
    float* v = qkv + r * ld + (which ? k_off : 0) + 2 * p;
    const float x0 = v[0], x1 = v[1];
    const float c0 = cosT[(int64_t)n * width + 2 * p], c1 = cosT[(int64_t)n * width + 2 * p + 1];
    const float s0 = sinT[(int64_t)n * width + 2 * p], s1 = sinT[(int64_t)n * width + 2 * p + 1];
    v[0] = add(mul(x0, c0), mul(-x1, s0));
    v[1] = add(mul(x1, c1), mul(x0, s1));
  }
}

// [batch][rows][cols] -> [batch][cols][rows] (optionally accumulating into out).
__global__ void transpose_kernel(const float* __restrict__ in, int rows, int cols, float* __restrict__ out, int acc) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const float* ib = in + (int64_t)b * rows * cols;
  float* ob = out + (int64_t)b * rows * cols;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int r = r0 + dy, c = c0 + threadIdx.x;
    tile[dy][threadIdx.x] = (r < rows && c < cols) ? ib[(int64_t)r * cols + c] : 0.f;
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int c = c0 + dy, r = r0 + threadIdx.x;
    if (r < rows && c < cols) {
      float* p = ob + (int64_t)c * rows + r;
      *p = acc ? add(*p, tile[threadIdx.x][dy]) : tile[threadIdx.x][dy];
    }
  }
}

// Euler step with classifier-free guidance (flow.py:86-87):
// x[u][c][n] += dt * ((1 + cfg) * d[2u][n][c] - cfg * d[2u+1][n][c]),
// d token-major [2U][frames][mel], x channel-major [U][mel][frames].
__global__ void cfg_euler_kernel(float* __restrict__ x, const float* __restrict__ d, int utts, int mel, int frames,
                                 float c1, float c2, float dt) {
  const int64_t total = (int64_t)utts * mel * frames;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % frames);
    const int64_t r = i / frames;
    const int c = (int)(r % mel);
    const int u = (int)(r / mel);
    const float d0 = d[((int64_t)(2 * u) * frames + n) * mel + c];
    const float d1 = d[((int64_t)(2 * u + 1) * frames + n) * mel + c];
    const float dphi = sub(mul(c1, d0), mul(c2, d1));
    x[i] = add(x[i], mul(dt, dphi));
  }
}

// x / max(||x||_2, 1e-12) per row (flow.py:105-106).
__global__ void l2_normalize_kernel(const float* __restrict__ x, int dim, float* __restrict__ y) {
  __shared__ float red[32];
  const float* r = x + (int64_t)blockIdx.x * dim;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += r[i] * r[i];
  const float nrm = fmaxf(sqrtf(block_sum(s, red)), 1e-12f);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) y[(int64_t)blockIdx.x * dim + i] = r[i] / nrm;
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)cv3::sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

int row_threads(int64_t dim) {
  int t = 32;
  while (t < dim && t < 1024) t <<= 1;
  return t;
}

}  // namespace

extern "C" int cv3_dit_input_cat(const float* x, const float* cond, const float* mu, const float* spk, int64_t utts,
                                 int64_t frames, int64_t mel, int64_t spk_dim, float* out, void* stream) {
  CV3_REQUIRE(utts >= 0 && frames >= 0 && mel > 0 && spk_dim > 0, CV3_ERR_VALUE, "dit_input_cat: bad shape");
  const int64_t total = 2 * utts * frames * (3 * mel + spk_dim);
  if (total == 0) return CV3_OK;
  input_cat_kernel<<<grid_for(total, 256), 256, 0, cv3::as_stream(stream)>>>(x, cond, mu, spk, (int)utts, (int)frames,
                                                                             (int)mel, (int)spk_dim, out);
  return cv3::check_launch("dit_input_cat");
}

extern "C" int cv3_ln_modulate(const float* h, int64_t rows, int64_t dim, float eps, const float* scale,
                               const float* shift, int64_t rows_per_group, int64_t mod_stride, float* y,
                               void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0 && rows < (1LL << 31), CV3_ERR_VALUE, "ln_modulate: bad shape");
  if (rows == 0) return CV3_OK;
  const bool al = (((uintptr_t)h | (uintptr_t)y | (uintptr_t)scale | (uintptr_t)shift) & 15) == 0 && mod_stride % 4 == 0;
  if (al && (dim == 1024 || dim == 512)) {
    const unsigned grid = (unsigned)((rows + 7) / 8);
    if (dim == 1024)
      ln_modulate_warp_kernel<8, false><<<grid, 256, 0, cv3::as_stream(stream)>>>(
          h, rows, eps, scale, shift, rows_per_group, mod_stride, y, nullptr, nullptr, 0);
    else
      ln_modulate_warp_kernel<4, false><<<grid, 256, 0, cv3::as_stream(stream)>>>(
          h, rows, eps, scale, shift, rows_per_group, mod_stride, y, nullptr, nullptr, 0);
    return cv3::check_launch("ln_modulate");
  }
  ln_modulate_kernel<<<(unsigned)rows, row_threads(dim), 0, cv3::as_stream(stream)>>>(
      h, (int)dim, eps, scale, shift, rows_per_group, mod_stride, y);
  return cv3::check_launch("ln_modulate");
}

extern "C" int cv3_ln_modulate_planes(const float* h, int64_t rows, int64_t dim, float eps, const float* scale,
                                      const float* shift, int64_t rows_per_group, int64_t mod_stride, void* planes,
                                      int8_t* exps, int64_t lde, void* stream) {
  CV3_REQUIRE(rows >= 0 && rows < (1LL << 31) && (dim == 1024 || dim == 512), CV3_ERR_UNSUPPORTED,
              "ln_modulate_planes: dim 512 or 1024");
  CV3_REQUIRE(lde >= rows && lde % 16 == 0, CV3_ERR_VALUE, "ln_modulate_planes: lde >= rows, a multiple of 16");
  CV3_REQUIRE((((uintptr_t)h | (uintptr_t)planes | (uintptr_t)scale | (uintptr_t)shift) & 15) == 0 &&
                  mod_stride % 4 == 0,
              CV3_ERR_VALUE, "ln_modulate_planes: 16-byte aligned operands");
  if (rows == 0) return CV3_OK;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  __half* pl = static_cast<__half*>(planes);
  if (dim == 1024)
    ln_modulate_warp_kernel<8, true><<<grid, 256, 0, cv3::as_stream(stream)>>>(
        h, rows, eps, scale, shift, rows_per_group, mod_stride, nullptr, pl, exps, lde);
  else
    ln_modulate_warp_kernel<4, true><<<grid, 256, 0, cv3::as_stream(stream)>>>(
        h, rows, eps, scale, shift, rows_per_group, mod_stride, nullptr, pl, exps, lde);
  return cv3::check_launch("ln_modulate_planes");
}

extern "C" int cv3_gate_residual(float* h, const float* y, const float* gate, int64_t rows, int64_t dim,
                                 int64_t rows_per_group, int64_t gate_stride, void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0, CV3_ERR_VALUE, "gate_residual: bad shape");
  if (rows == 0) return CV3_OK;
  gate_residual_kernel<<<grid_for(rows * dim, 256), 256, 0, cv3::as_stream(stream)>>>(h, y, gate, rows, (int)dim,
                                                                                     rows_per_group, gate_stride);
  return cv3::check_launch("gate_residual");
}

extern "C" int cv3_partial_rope(float* qkv, int64_t rows, int64_t ld, int64_t k_offset, int64_t frames,
                                int64_t width, const float* cos_table, const float* sin_table, void* stream) {
  CV3_REQUIRE(rows >= 0 && frames > 0 && width > 0 && width % 2 == 0 && ld >= k_offset + width, CV3_ERR_VALUE,
              "partial_rope: bad shape");
  if (rows == 0) return CV3_OK;
  partial_rope_kernel<<<grid_for(rows * width, 256), 256, 0, cv3::as_stream(stream)>>>(
      qkv, rows, ld, k_offset, (int)frames, (int)width, cos_table, sin_table);
  return cv3::check_launch("partial_rope");
}

extern "C" int cv3_transpose(const float* in, int64_t batch, int64_t rows, int64_t cols, float* out, int accumulate,
                             void* stream) {
  CV3_REQUIRE(batch >= 0 && rows >= 0 && cols >= 0 && batch <= 65535, CV3_ERR_VALUE, "transpose: bad shape");
  if (batch * rows * cols == 0) return CV3_OK;
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
  CV3_REQUIRE(grid.y <= 65535, CV3_ERR_VALUE, "transpose: too many rows");
  transpose_kernel<<<grid, dim3(32, 8), 0, cv3::as_stream(stream)>>>(in, (int)rows, (int)cols, out, accumulate);
  return cv3::check_launch("transpose");
}

extern "C" int cv3_cfg_euler(float* x, const float* d, int64_t utts, int64_t mel, int64_t frames, double cfg_rate,
                             float dt, void* stream) {
  CV3_REQUIRE(utts >= 0 && mel > 0 && frames >= 0, CV3_ERR_VALUE, "cfg_euler: bad shape");
  if (utts * frames == 0) return CV3_OK;
  // (1.0 + cfg) and cfg are Python floats in the reference, rounded to float32
  // when they scale a float32 array.
  const float c1 = (float)(1.0 + cfg_rate), c2 = (float)cfg_rate;
  cfg_euler_kernel<<<grid_for(utts * mel * frames, 256), 256, 0, cv3::as_stream(stream)>>>(
      x, d, (int)utts, (int)mel, (int)frames, c1, c2, dt);
  return cv3::check_launch("cfg_euler");
}

extern "C" int cv3_l2_normalize(const float* x, int64_t rows, int64_t dim, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && dim > 0, CV3_ERR_VALUE, "l2_normalize: bad shape");
  if (rows == 0) return CV3_OK;
  l2_normalize_kernel<<<(unsigned)rows, row_threads(dim), 0, cv3::as_stream(stream)>>>(x, (int)dim, y);
  return cv3::check_launch("l2_normalize");
}

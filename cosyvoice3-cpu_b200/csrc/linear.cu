// Linear layers: the q8 weight-streaming GEMV/skinny GEMM, the fp32 SIMT GEMM
// and the q8 dequantiser.
//
// q8 kernel (replaces cv3cpu/quant.py:156-204): HBM-bound.  Each warp owns RW
// weight rows; its lanes stride along K in 16-byte chunks (16 int8 = a quarter
// of one 64-wide scale block), so a warp reads 512 contiguous bytes of a row
// per step and every chunk's loads for all RW rows are issued before any math
// (8 independent 16-byte loads in flight per lane).  int8 is
// widened with one byte-permute + one exact add (2^23 + b + 128 - (2^23 + 128)),
// partial dots are taken per chunk, multiplied by the chunk's fp16 scale and
// summed; a warp shuffle reduces the row.  x rows (<= 8 per pass) sit in
// shared memory, zero-padded to Kp.
#include "common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// 16 int8 weights of one chunk -> 16 floats (exact).
__device__ __forceinline__ void widen16(const int4 w, float f[16]) {
  const uint32_t words[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u,
                             (uint32_t)w.z ^ 0x80808080u, (uint32_t)w.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t bits = __byte_perm(words[i], 0x4B000000u, 0x7440u | b);
      f[4 * i + b] = __int_as_float(bits) - 8388736.0f;  // 2^23 + 128
    }
  }
}

// M: x rows held per pass (rows >= mm are zero and not written).  RW: weight
// rows per warp.  Each lane keeps UNR*RW = 8 16-byte loads in flight.
template <int M, int RW>
__global__ void __launch_bounds__(kThreads)
q8_gemv_kernel(const float* __restrict__ x, int64_t ldx, int mm, int k, const int8_t* __restrict__ q,
               const uint16_t* __restrict__ sc, int n, int kp, const float* __restrict__ bias,
               const float* residual, float* y, int64_t ldy) {
  constexpr int UNR = 8 / RW;
  extern __shared__ float xs[];  // [M][kp]
  for (int i = threadIdx.x; i < M * kp; i += blockDim.x) {
    const int m = i / kp, c = i - m * kp;
    xs[i] = (c < k && m < mm) ? x[(int64_t)m * ldx + c] : 0.f;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int row0 = warp * RW;
  if (row0 >= n) return;
  const int chunks = kp >> 4;
  const int nb = kp >> 6;

  float acc[RW][M];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

  for (int c0 = 0; c0 < chunks; c0 += 32 * UNR) {
    int4 w[UNR][RW];
#pragma unroll
    for (int j = 0; j < UNR; ++j) {
      const int c = c0 + lane + 32 * j;
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const int row = min(row0 + r, n - 1);
        w[j][r] = c < chunks ? ld_stream16(q + (int64_t)row * kp + c * 16) : make_int4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int j = 0; j < UNR; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c < chunks) {
        float f[RW][16];
        float s[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          widen16(w[j][r], f[r]);
          s[r] = h2f(sc[(int64_t)min(row0 + r, n - 1) * nb + (c >> 2)]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float xv[16];
          const float4* src = reinterpret_cast<const float4*>(xs + m * kp + c * 16);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 t = src[v];
            xv[4 * v] = t.x; xv[4 * v + 1] = t.y; xv[4 * v + 2] = t.z; xv[4 * v + 3] = t.w;
          }
#pragma unroll
          for (int r = 0; r < RW; ++r) {
            float p = 0.f;
#pragma unroll
            for (int e = 0; e < 16; ++e) p = fmaf(f[r][e], xv[e], p);
            acc[r][m] = fmaf(p, s[r], acc[r][m]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[r][m]);
      const int row = row0 + r;
      if (lane == 0 && row < n && m < mm) {
        float o = v;
        if (bias) o += bias[row];
        if (residual) o += residual[(int64_t)m * ldy + row];
        y[(int64_t)m * ldy + row] = o;
      }
    }
  }
}

template <int M, int RW>
int launch_q8(const float* x, int64_t ldx, int mm, int k, const int8_t* q, const uint16_t* sc, int n, int kp,
              const float* bias, const float* res, float* y, int64_t ldy, cudaStream_t st) {
  const int smem = M * kp * 4;
  auto fn = q8_gemv_kernel<M, RW>;
  if (smem > 48 * 1024) {
    int rc = cv3::allow_smem((const void*)fn, smem);
    if (rc) return rc;
  }
  const int warps = (n + RW - 1) / RW;
  const int grid = (warps + kWarps - 1) / kWarps;
  fn<<<grid, kThreads, smem, st>>>(x, ldx, mm, k, q, sc, n, kp, bias, res, y, ldy);
  return cv3::check_launch("q8_gemv");
}

template <int M>
int dispatch_rw(const float* x, int64_t ldx, int mm, int k, const int8_t* q, const uint16_t* sc, int n, int kp,
                const float* bias, const float* res, float* y, int64_t ldy, cudaStream_t st) {
  // Enough warps for two per SM scheduler first, then more rows per warp.
  const int sms = cv3::sm_count();
  if (M <= 2 && n >= sms * kWarps * 4 * 2)
    return launch_q8<M, 4>(x, ldx, mm, k, q, sc, n, kp, bias, res, y, ldy, st);
  if (M <= 4 && n >= sms * kWarps * 2 * 2)
    return launch_q8<M, 2>(x, ldx, mm, k, q, sc, n, kp, bias, res, y, ldy, st);
  return launch_q8<M, 1>(x, ldx, mm, k, q, sc, n, kp, bias, res, y, ldy, st);
}

// ---------------------------------------------------------------------------
// q4 ("tiny" profile, cv3cpu/quant.py:70-86, 124-131): a 32-wide block of a
// row is 16 bytes -- byte j holds code j (low nibble) and code j + 16 (high
// nibble) -- and one fp16 scale; w = (code - 8) * scale, exact in fp32.  Each
// lane takes whole 16-byte blocks (a warp reads 512 contiguous bytes of a row
// per step), widens the 32 codes exactly, dots them with x and applies the
// block's scale; a warp shuffle reduces the row.  Same structure as q8.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void widen_q4(const int4 w, float f[32]) {
  const uint32_t words[4] = {(uint32_t)w.x, (uint32_t)w.y, (uint32_t)w.z, (uint32_t)w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (words[i] >> (8 * b)) & 0xFFu;
      f[4 * i + b] = (float)(int)(byte & 0xFu) - 8.0f;   // code j
      f[16 + 4 * i + b] = (float)(int)(byte >> 4) - 8.0f;  // code j + 16
    }
}

template <int M, int RW>
__global__ void __launch_bounds__(kThreads)
q4_gemv_kernel(const float* __restrict__ x, int64_t ldx, int mm, int k, const uint8_t* __restrict__ q,
               const uint16_t* __restrict__ sc, int n, int kp, const float* __restrict__ bias,
               const float* residual, float* y, int64_t ldy) {
  constexpr int UNR = 8 / RW;
  extern __shared__ float xs[];  // [M][kp]
  for (int i = threadIdx.x; i < M * kp; i += blockDim.x) {
    const int m = i / kp, c = i - m * kp;
    xs[i] = (c < k && m < mm) ? x[(int64_t)m * ldx + c] : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int row0 = warp * RW;
  if (row0 >= n) return;
  const int blocks = kp >> 5;  // 32-wide blocks = 16-byte chunks of a row
  float acc[RW][M];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  for (int c0 = 0; c0 < blocks; c0 += 32 * UNR) {
    int4 w[UNR][RW];
#pragma unroll
    for (int j = 0; j < UNR; ++j) {
      const int c = c0 + lane + 32 * j;
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const int row = min(row0 + r, n - 1);
        w[j][r] = c < blocks ? ld_stream16(q + (int64_t)row * (kp / 2) + c * 16) : make_int4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int j = 0; j < UNR; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c < blocks) {
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          float f[32];
          widen_q4(w[j][r], f);
          const float s = h2f(sc[(int64_t)min(row0 + r, n - 1) * blocks + c]);
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float4* src = reinterpret_cast<const float4*>(xs + m * kp + c * 32);
            float p = 0.f;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 t = src[v];
              p = fmaf(f[4 * v], t.x, p);
              p = fmaf(f[4 * v + 1], t.y, p);
              p = fmaf(f[4 * v + 2], t.z, p);
              p = fmaf(f[4 * v + 3], t.w, p);
            }
            acc[r][m] = fmaf(p, s, acc[r][m]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[r][m]);
      const int row = row0 + r;
      if (lane == 0 && row < n && m < mm) {
        float o = v;
        if (bias) o += bias[row];
        if (residual) o += residual[(int64_t)m * ldy + row];
        y[(int64_t)m * ldy + row] = o;
      }
    }
  }
}

template <int M>
int launch_q4(const float* x, int64_t ldx, int mm, int k, const uint8_t* q, const uint16_t* sc, int n, int kp,
              const float* bias, const float* res, float* y, int64_t ldy, cudaStream_t st) {
  const int smem = M * kp * 4;
  const int sms = cv3::sm_count();
  const bool two = M <= 4 && n >= sms * kWarps * 2 * 2;  // enough rows for two per warp
  auto fn = two ? q4_gemv_kernel<M, 2> : q4_gemv_kernel<M, 1>;
  if (smem > 48 * 1024) {
    int rc = cv3::allow_smem((const void*)fn, smem);
    if (rc) return rc;
  }
  const int rw = two ? 2 : 1;
  const int grid = ((n + rw - 1) / rw + kWarps - 1) / kWarps;
  fn<<<grid, kThreads, smem, st>>>(x, ldx, mm, k, q, sc, n, kp, bias, res, y, ldy);
  return cv3::check_launch("q4_gemv");
}

__global__ void q4_dequant_kernel(const uint8_t* __restrict__ q, const uint16_t* __restrict__ sc, int64_t n,
                                  int64_t kp, int64_t k, float* __restrict__ out) {
  const int64_t total = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k, c = i - r * k;
    const int64_t blk = c >> 5, j = c & 31;
    const uint8_t byte = q[r * (kp / 2) + blk * 16 + (j & 15)];
    const int code = j < 16 ? (byte & 0xF) : (byte >> 4);
    out[i] = ((float)code - 8.0f) * h2f(sc[r * (kp / 32) + blk]);
  }
}

// ---------------------------------------------------------------------------
// fp32 SIMT GEMM: y = x w^T (+bias)(+residual); 64x64 tile, 4x4 per thread.
// ---------------------------------------------------------------------------
constexpr int BM = 64, BN = 64, BK = 16;

__global__ void __launch_bounds__(256)
sgemm_nt_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w, int64_t ldw,
                int m, int n, int k, const float* __restrict__ bias, const float* residual,
                float* y, int64_t ldy) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, c = i - r * BK;
      const int gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < m && gk < k) ? x[(int64_t)gm * ldx + gk] : 0.f;
      const int gn = n0 + r;
      Bs[c][r] = (gn < n && gk < k) ? w[(int64_t)gn * ldw + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
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
    const int gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= n) continue;
      float o = acc[i][j];
      if (bias) o += bias[gn];
      if (residual) o += residual[(int64_t)gm * ldy + gn];
      y[(int64_t)gm * ldy + gn] = o;
    }
  }
}

__global__ void q8_dequant_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ sc, int64_t n,
                                  int64_t kp, int64_t k, float* __restrict__ out) {
  const int64_t total = n * k;
  const int64_t nb = kp / 64;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k, c = i - r * k;
    out[i] = (float)q[r * kp + c] * h2f(sc[r * nb + c / 64]);
  }
}

}  // namespace

extern "C" int cv3_q8_linear(const float* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                             const uint16_t* scales, int64_t n, int64_t kp, const float* bias,
                             const float* residual, float* y, int64_t ldy, void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0, CV3_ERR_VALUE, "q8_linear: negative size");
  CV3_REQUIRE(kp % 64 == 0 && kp >= k && kp - k < 64, CV3_ERR_VALUE,
              "q8_linear: padded K %lld does not match K %lld", (long long)kp, (long long)k);
  CV3_REQUIRE(ldx >= k && ldy >= n, CV3_ERR_VALUE, "q8_linear: leading dimension too small");
  CV3_REQUIRE(((uintptr_t)q & 15) == 0, CV3_ERR_VALUE, "q8_linear: payload must be 16-byte aligned");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(n < (1LL << 31) && kp < (1LL << 20), CV3_ERR_VALUE, "q8_linear: shape too large");
  CV3_REQUIRE(kp * 8 * 4 <= 200 * 1024, CV3_ERR_VALUE, "q8_linear: padded K %lld too large", (long long)kp);
  cudaStream_t st = cv3::as_stream(stream);
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mm = (int)((m - m0) < 8 ? (m - m0) : 8);
    const float* xp = x + m0 * ldx;
    const float* rp = residual ? residual + m0 * ldy : nullptr;
    float* yp = y + m0 * ldy;
    int rc;
    if (mm == 1) rc = dispatch_rw<1>(xp, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rp, yp, ldy, st);
    else if (mm == 2) rc = dispatch_rw<2>(xp, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rp, yp, ldy, st);
    else if (mm <= 4) rc = dispatch_rw<4>(xp, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rp, yp, ldy, st);
    else rc = dispatch_rw<8>(xp, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rp, yp, ldy, st);
    if (rc) return rc;
  }
  return CV3_OK;
}

extern "C" int cv3_q4_linear(const float* x, int64_t m, int64_t k, int64_t ldx, const uint8_t* q,
                             const uint16_t* scales, int64_t n, int64_t kp, const float* bias, const float* residual,
                             float* y, int64_t ldy, void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0, CV3_ERR_VALUE, "q4_linear: negative size");
  CV3_REQUIRE(kp % 32 == 0 && kp >= k && kp - k < 32, CV3_ERR_VALUE,
              "q4_linear: padded K %lld does not match K %lld (32-wide blocks)", (long long)kp, (long long)k);
  CV3_REQUIRE(ldx >= k && ldy >= n, CV3_ERR_VALUE, "q4_linear: leading dimension too small");
  CV3_REQUIRE(((uintptr_t)q & 15) == 0, CV3_ERR_VALUE, "q4_linear: payload must be 16-byte aligned");
  CV3_REQUIRE(n < (1LL << 31) && kp < (1LL << 20), CV3_ERR_VALUE, "q4_linear: shape too large");
  CV3_REQUIRE(kp * 8 * 4 <= 200 * 1024, CV3_ERR_VALUE, "q4_linear: padded K %lld too large", (long long)kp);
  if (m == 0 || n == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  for (int64_t m0 = 0; m0 < m; m0 += 8) {  // 8 x rows per pass
    const int mm = (int)std::min<int64_t>(8, m - m0);
    const float* xr = x + m0 * ldx;
    const float* rr = residual ? residual + m0 * ldy : nullptr;
    float* yr = y + m0 * ldy;
    int rc = mm <= 1   ? launch_q4<1>(xr, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rr, yr, ldy, st)
             : mm <= 2 ? launch_q4<2>(xr, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rr, yr, ldy, st)
             : mm <= 4 ? launch_q4<4>(xr, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rr, yr, ldy, st)
                       : launch_q4<8>(xr, ldx, mm, (int)k, q, scales, (int)n, (int)kp, bias, rr, yr, ldy, st);
    if (rc) return rc;
  }
  return CV3_OK;
}

extern "C" int cv3_q4_dequant(const uint8_t* q, const uint16_t* scales, int64_t n, int64_t kp, int64_t k, float* out,
                              void* stream) {
  CV3_REQUIRE(n >= 0 && k >= 0 && kp % 32 == 0 && kp >= k, CV3_ERR_VALUE, "q4_dequant: bad shape");
  if (n == 0 || k == 0) return CV3_OK;
  int64_t grid = (n * k + 255) / 256;
  if (grid > cv3::sm_count() * 32) grid = cv3::sm_count() * 32;
  q4_dequant_kernel<<<(unsigned)grid, 256, 0, cv3::as_stream(stream)>>>(q, scales, n, kp, k, out);
  return cv3::check_launch("q4_dequant");
}

extern "C" int cv3_f32_linear(const float* x, int64_t m, int64_t k, int64_t ldx, const float* w, int64_t n,
                              int64_t ldw, const float* bias, const float* residual, float* y, int64_t ldy,
                              void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0, CV3_ERR_VALUE, "f32_linear: negative size");
  CV3_REQUIRE(ldx >= k && ldw >= k && ldy >= n, CV3_ERR_VALUE, "f32_linear: leading dimension too small");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CV3_ERR_VALUE, "f32_linear: too large");
  dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
  CV3_REQUIRE(grid.y <= 65535, CV3_ERR_VALUE, "f32_linear: too many rows");
  sgemm_nt_kernel<<<grid, 256, 0, cv3::as_stream(stream)>>>(x, ldx, w, ldw, (int)m, (int)n, (int)k, bias,
                                                             residual, y, ldy);
  return cv3::check_launch("f32_linear");
}

extern "C" int cv3_q8_dequant(const int8_t* q, const uint16_t* scales, int64_t n, int64_t kp, int64_t k,
                              float* out, void* stream) {
  CV3_REQUIRE(n >= 0 && k >= 0 && kp % 64 == 0 && kp >= k, CV3_ERR_VALUE, "q8_dequant: bad shape");
  if (n == 0 || k == 0) return CV3_OK;
  const int64_t total = n * k;
  int64_t blocks = (total + 255) / 256;
  if (blocks > cv3::sm_count() * 32) blocks = cv3::sm_count() * 32;
  q8_dequant_kernel<<<(unsigned)blocks, 256, 0, cv3::as_stream(stream)>>>(q, scales, n, kp, k, out);
  return cv3::check_launch("q8_dequant");
}

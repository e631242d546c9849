// Batched decode GEMV for q8 weights (the LM's per-token linears, M <= 8 rows).
//
// y[m][row] = epilogue( sum_k xn[m][k] * q[row][k] * s[row][k/64] )
//
// Layout of the work: a CTA owns 32 weight rows (one per lane) and a K range;
// its 8 warps split that range, every lane streams its own row 16 bytes at a
// time (eight 16-byte loads in flight per lane) while the matching activation
// values are read from shared memory as broadcasts (all lanes of a warp use the
// same k), so each weight byte costs M FMAs and no per-lane activation traffic.
// Small matrices also split K across CTAs (grid.y); the partial sums go to a
// caller workspace and the last CTA of a row tile to arrive adds them in a fixed
// order -- deterministic, no float atomics.
//
// Fusions (cv3cpu/models/qwen2.py:155-177, llm.py:74-78):
//   * optional RMSNorm of x while it is staged (x*(1/sqrt(mean(x^2)+eps)))*w,
//   * bias, residual add (y may alias the residual),
//   * SwiGLU pairs: weight rows interleaved (2i = gate_i, 2i+1 = up_i) give
//     y[m][i] = silu(gate) * up directly.
#include "common.cuh"

namespace {

constexpr int kWarps = 4;   // 128-thread CTAs: every row tile of the LM shapes fits one wave
constexpr int kRows = 32;
constexpr int kUnroll = 8;

__device__ __forceinline__ void widen16(const int4 w, float f[16]) {
  const uint32_t words[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u,
                             (uint32_t)w.z ^ 0x80808080u, (uint32_t)w.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < 4; ++b) f[4 * i + b] = __int_as_float(__byte_perm(words[i], 0x4B000000u, 0x7440u | b)) - 8388736.0f;
}

struct GemvArgs {
  const float* x; int64_t ldx; int mm; int k;
  const int8_t* q; const uint16_t* sc; int n; int kp;
  const float* bias; const float* residual; float* y; int64_t ldy;
  const float* norm_w; float eps;
  int swiglu;
  int splits; int kps;          // K splits across CTAs and elements per split (multiple of 16)
  float* partial; int* counter;  // [splits][M][n] and [n/32] (zero on entry, left zero)
};

template <int M>
__global__ void __launch_bounds__(kWarps * 32)
q8_decode_gemv_kernel(GemvArgs a) {
  extern __shared__ float xs[];            // [M][xw] staged activations (xw = K range or whole rows)
  __shared__ float part[kWarps][M][kRows];
  __shared__ float rnorm[M];
  __shared__ int last_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * kRows, split = blockIdx.y;
  const int k0 = split * a.kps;
  const int klen = max(0, min(a.kps, a.kp - k0));
  // with a fused RMSNorm every CTA needs whole rows for the mean of squares
  const int xw = a.norm_w ? a.kp : a.kps;
  const int xoff = a.norm_w ? k0 : 0;      // where this CTA's K range starts inside xs rows
  const int xbase = a.norm_w ? 0 : k0;     // first column of x staged

  // -- stage x: float4 loads issued in independent batches of 8 per thread ------------
  {
    const int vec_row = xw / 4;
    const int total = M * vec_row;
    constexpr int T = kWarps * 32;
    for (int i0 = 0; i0 < total; i0 += 8 * T) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * T + tid;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < total) {
          const int m = i / vec_row, c = (i - m * vec_row) * 4 + xbase;
          if (m < a.mm && c + 3 < a.k) v[u] = *reinterpret_cast<const float4*>(a.x + (int64_t)m * a.ldx + c);
          else if (m < a.mm)
            for (int e = 0; e < 4; ++e)
              if (c + e < a.k) reinterpret_cast<float*>(&v[u])[e] = a.x[(int64_t)m * a.ldx + c + e];
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * T + tid;
        if (i < total) reinterpret_cast<float4*>(xs)[i] = v[u];
      }
    }
  }
  __syncthreads();
  if (a.norm_w) {
    for (int m = warp; m < M; m += kWarps) {
      float s = 0.f;
      for (int c = lane; c < a.k; c += 32) {
        const float v = xs[m * xw + c];
        s += v * v;
      }
      s = warp_sum(s);
      if (lane == 0) rnorm[m] = 1.0f / sqrtf(s / (float)a.k + a.eps);
    }
    __syncthreads();
    // scale in place, float4 at a time; the norm weights come in as independent
    // float4 loads (one batch per thread), never one dependent load per element
    const int vec_row = xw / 4;
    for (int c4 = tid; c4 < vec_row; c4 += kWarps * 32) {
      const int c = c4 * 4;
      float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c + 3 < a.k) w4 = *reinterpret_cast<const float4*>(a.norm_w + c);
      else
        for (int e = 0; e < 4; ++e)
          if (c + e < a.k) reinterpret_cast<float*>(&w4)[e] = a.norm_w[c + e];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float4* p = reinterpret_cast<float4*>(xs + m * xw) + c4;
        float4 v = *p;
        const float r = rnorm[m];
        v.x = (v.x * r) * w4.x;
        v.y = (v.y * r) * w4.y;
        v.z = (v.z * r) * w4.z;
        v.w = (v.w * r) * w4.w;
        *p = v;
      }
    }
    __syncthreads();
  }

  // -- this warp's slice of the CTA's K range, one weight row per lane ---------------
  const int pieces = (klen + 15) / 16;
  const int per_warp = (pieces + kWarps - 1) / kWarps;
  const int p0 = warp * per_warp, p1 = min(pieces, p0 + per_warp);
  const int row = row0 + lane;
  const int rowc = min(row, a.n - 1);
  const int8_t* qrow = a.q + (int64_t)rowc * a.kp + k0;
  const uint16_t* srow = a.sc + (int64_t)rowc * (a.kp >> 6);
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.f;
  for (int p = p0; p < p1; p += kUnroll) {
    int4 w[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      w[u] = (p + u < p1) ? ld_stream16(qrow + (p + u) * 16) : make_int4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (p + u < p1) {
        const int c = (p + u) * 16;  // offset inside the CTA's K range
        const float s = h2f(srow[(k0 + c) >> 6]);
        float f[16];
        widen16(w[u], f);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float4* xv = reinterpret_cast<const float4*>(xs + m * xw + xoff + c);
          float d = 0.f;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 t = xv[v];
            d = fmaf(f[4 * v], t.x, d);
            d = fmaf(f[4 * v + 1], t.y, d);
            d = fmaf(f[4 * v + 2], t.z, d);
            d = fmaf(f[4 * v + 3], t.w, d);
          }
          acc[m] = fmaf(d, s, acc[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) part[warp][m][lane] = acc[m];
  __syncthreads();

  // -- reduce the warps (fixed order), then the K splits -------------------------------
  // thread -> (m, r = lane) pairs, kWarps rows of m per pass; a warp always holds one m
  constexpr int kPasses = (M + kWarps - 1) / kWarps;
  float vsum[kPasses];
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int m = warp + ps * kWarps;
    float v = 0.f;
    if (m < M) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += part[w][m][lane];
    }
    vsum[ps] = v;
  }
  if (a.splits > 1) {
    const int gr = row0 + lane;
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
      const int m = warp + ps * kWarps;
      if (m < M && gr < a.n) a.partial[((int64_t)split * M + m) * a.n + gr] = vsum[ps];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = (atomicAdd(&a.counter[blockIdx.x], 1) == a.splits - 1);
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
      const int m = warp + ps * kWarps;
      float v = 0.f;
      if (m < M && gr < a.n) {
        // issue the partial loads in groups of 8 before summing them in order
        for (int s0 = 0; s0 < a.splits; s0 += 8) {
          float t[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            t[u] = (s0 + u < a.splits) ? __ldcg(&a.partial[((int64_t)(s0 + u) * M + m) * a.n + gr]) : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (s0 + u < a.splits) v += t[u];
        }
      }
      vsum[ps] = v;
    }
    if (tid == 0) a.counter[blockIdx.x] = 0;  // ready for the next launch
  }

  // -- epilogue ------------------------------------------------------------------------
  const int gr = row0 + lane;
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int m = warp + ps * kWarps;
    float v = vsum[ps];
    if (m < M && gr < a.n && a.bias) v += a.bias[gr];
    if (a.swiglu) {
      // rows 2i (gate) and 2i+1 (up) sit in neighbouring lanes
      const float up = __shfl_down_sync(0xffffffffu, v, 1);
      if (m < a.mm && gr < a.n && (lane & 1) == 0) {
        const float g = v;
        a.y[(int64_t)m * a.ldy + gr / 2] = (g / (1.0f + expf(-g))) * up;
      }
    } else if (m < a.mm && gr < a.n) {
      float o = v;
      if (a.residual) o = o + a.residual[(int64_t)m * a.ldy + gr];
      a.y[(int64_t)m * a.ldy + gr] = o;
    }
  }
}

template <int M>
int launch(const GemvArgs& a, cudaStream_t st) {
  const int smem = M * (a.norm_w ? a.kp : a.kps) * 4;
  auto fn = q8_decode_gemv_kernel<M>;
  if (smem > 48 * 1024) {
    int rc = cv3::allow_smem((const void*)fn, smem);
    if (rc) return rc;
  }
  dim3 grid((unsigned)((a.n + kRows - 1) / kRows), (unsigned)a.splits);
  fn<<<grid, kWarps * 32, smem, st>>>(a);
  return cv3::check_launch("q8_decode_gemv");
}

}  // namespace

extern "C" int cv3_q8_decode_gemv(const float* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                                  const uint16_t* scales, int64_t n, int64_t kp, const float* bias,
                                  const float* residual, const float* norm_w, float eps, int swiglu, float* y,
                                  int64_t ldy, int64_t splits, float* workspace, int64_t workspace_floats,
                                  int* counters, void* stream) {
  CV3_REQUIRE(m >= 1 && m <= 8, CV3_ERR_VALUE, "q8_decode_gemv: 1..8 rows per call (got %lld)", (long long)m);
  CV3_REQUIRE(n > 0 && k > 0 && kp % 64 == 0 && kp >= k && kp - k < 64, CV3_ERR_VALUE,
              "q8_decode_gemv: padded K %lld does not match K %lld", (long long)kp, (long long)k);
  CV3_REQUIRE(ldx >= k, CV3_ERR_VALUE, "q8_decode_gemv: ldx too small");
  CV3_REQUIRE(swiglu ? (n % 2 == 0 && ldy >= n / 2 && !residual) : ldy >= n, CV3_ERR_VALUE,
              "q8_decode_gemv: bad output layout");
  CV3_REQUIRE(((uintptr_t)q & 15) == 0 && n < (1LL << 30) && kp < (1LL << 20), CV3_ERR_VALUE,
              "q8_decode_gemv: payload alignment or size");
  CV3_REQUIRE(splits >= 1 && splits <= 64, CV3_ERR_VALUE, "q8_decode_gemv: 1..64 K splits");
  GemvArgs a{x, ldx, (int)m, (int)k, q, scales, (int)n, (int)kp, bias, residual, y, ldy, norm_w, eps, swiglu,
             (int)splits, 0, workspace, counters};
  a.kps = (int)((kp / splits + 15) / 16 * 16);
  a.splits = (int)((kp + a.kps - 1) / a.kps);
  CV3_REQUIRE((norm_w ? kp : a.kps) * 8 * 4 <= 200 * 1024, CV3_ERR_VALUE, "q8_decode_gemv: K range per CTA too large");
  CV3_REQUIRE(ldx % 4 == 0 && ((uintptr_t)x & 15) == 0, CV3_ERR_VALUE, "q8_decode_gemv: x rows must be 16-byte aligned");
  if (a.splits > 1) {
    CV3_REQUIRE(workspace && counters && workspace_floats >= (int64_t)a.splits * 8 * n, CV3_ERR_VALUE,
                "q8_decode_gemv: K splits need a workspace of splits*8*n floats and n/32 zeroed counters");
  }
  cudaStream_t st = cv3::as_stream(stream);
  switch (m) {
    case 1: return launch<1>(a, st);
    case 2: return launch<2>(a, st);
    case 3: case 4: return launch<4>(a, st);
    default: return launch<8>(a, st);
  }
}

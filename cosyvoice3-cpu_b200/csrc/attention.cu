// Scaled dot-product attention, fp32, exact softmax semantics of
// cv3cpu/ops.py:267-310 (GQA by head grouping, masks: none / causal(offset) /
// chunk(size, left)).  Tensors are addressed by strides, so both the
// reference's (H, N, D) layout and the models' token-major (B, N, H*D) layout
// are read in place:  elem(b, h, n, d) = base + b*sb + h*sh + n*sn + d.
//
// Two kernels:
//  * prefill/full: one thread per query, 128 queries per CTA; 64-key K/V tiles
//    staged in shared memory and read as broadcasts; per tile the scores are
//    kept in shared memory, the running max/sum rescaled once per tile.
//  * decode (<= 4 queries): one CTA per (batch, head, query); scores of all
//    keys in shared memory, then block max, exp, sum and a V pass with
//    coalesced rows.
#include "common.cuh"

namespace {

struct AttnArgs {
  const float* q; const float* k; const float* v; float* o;
  int64_t qsb, qsh, qsn;
  int64_t ksb, ksh, ksn;
  int64_t vsb, vsh, vsn;
  int64_t osb, osh, osn;
  int heads, kv_heads, n, m, d;
  float scale;
  int mask_kind;   // 0 none, 1 causal, 2 chunk
  int mask_a, mask_b;
};

__device__ __forceinline__ bool allowed(const AttnArgs& a, int qi, int kj) {
  if (a.mask_kind == 1) return kj <= qi + a.mask_a;
  if (a.mask_kind == 2) {
    const int size = a.mask_a, left = a.mask_b;
    const int c = qi / size;
    const int end = (c + 1) * size;
    const int start = left < 0 ? 0 : max((c - left) * size, 0);
    return kj < end && kj >= start;
  }
  return true;
}

constexpr int QT = 128;  // queries per CTA (one per thread)
constexpr int KT = 32;   // keys per tile
constexpr int DMAX = 64;

__global__ void __launch_bounds__(QT)
attn_full_kernel(AttnArgs a) {
  __shared__ float4 Ks[KT][DMAX / 4];
  __shared__ float4 Vs[KT][DMAX / 4];
  __shared__ float S[KT][QT];
  const int bh = blockIdx.y;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int hk = h / (a.heads / a.kv_heads);
  const int qi = blockIdx.x * QT + threadIdx.x;
  const bool live = qi < a.n;
  const float* qp = a.q + b * a.qsb + h * a.qsh + (int64_t)(live ? qi : 0) * a.qsn;
  float qv[DMAX], ov[DMAX];
#pragma unroll
  for (int d = 0; d < DMAX; ++d) {
    qv[d] = (d < a.d && live) ? qp[d] * a.scale : 0.f;
    ov[d] = 0.f;
  }
  float mrun = -INFINITY, lrun = 0.f;
  const float* kb = a.k + b * a.ksb + hk * a.ksh;
  const float* vb = a.v + b * a.vsb + hk * a.vsh;
  // K/V tiles are fetched one tile ahead into registers (float4, all loads of a
  // tile in flight together) so their latency overlaps the current tile's math.
  constexpr int F4 = KT * DMAX / 4 / QT;  // float4 of K (and of V) per thread per tile
  float4 kpre[F4], vpre[F4];
  auto fetch = [&](int j0) {
#pragma unroll
    for (int u = 0; u < F4; ++u) {
      const int f = threadIdx.x + u * QT;
      const int r = f / (DMAX / 4), c = (f % (DMAX / 4)) * 4;
      const int j = j0 + r;
      const bool ok = j < a.m && c < a.d;
      kpre[u] = ok ? *reinterpret_cast<const float4*>(kb + (int64_t)j * a.ksn + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      vpre[u] = ok ? *reinterpret_cast<const float4*>(vb + (int64_t)j * a.vsn + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  fetch(0);
  for (int j0 = 0; j0 < a.m; j0 += KT) {
    __syncthreads();
#pragma unroll
    for (int u = 0; u < F4; ++u) {
      const int f = threadIdx.x + u * QT;
      Ks[f / (DMAX / 4)][f % (DMAX / 4)] = kpre[u];
      Vs[f / (DMAX / 4)][f % (DMAX / 4)] = vpre[u];
    }
    __syncthreads();
    if (j0 + KT < a.m) fetch(j0 + KT);
    float tmax = -INFINITY;
    for (int r = 0; r < KT; ++r) {
      const int j = j0 + r;
      float s = -INFINITY;
      if (j < a.m && allowed(a, qi, j)) {
        // four independent partial sums: the dot product is a 16-deep chain, not 64
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < DMAX / 4; ++d4) {
          const float4 kv = Ks[r][d4];
          s0 = fmaf(qv[4 * d4], kv.x, s0);
          s1 = fmaf(qv[4 * d4 + 1], kv.y, s1);
          s2 = fmaf(qv[4 * d4 + 2], kv.z, s2);
          s3 = fmaf(qv[4 * d4 + 3], kv.w, s3);
        }
        s = (s0 + s1) + (s2 + s3);
      }
      S[r][threadIdx.x] = s;
      tmax = fmaxf(tmax, s);
    }
    const float mnew = fmaxf(mrun, tmax);
    if (mnew == -INFINITY) continue;  // nothing visible yet
    const float corr = expf(mrun - mnew);
    lrun *= corr;
#pragma unroll
    for (int d = 0; d < DMAX; ++d) ov[d] *= corr;
    for (int r = 0; r < KT; ++r) {
      const float p = expf(S[r][threadIdx.x] - mnew);
      lrun += p;
#pragma unroll
      for (int d4 = 0; d4 < DMAX / 4; ++d4) {
        const float4 vv = Vs[r][d4];
        ov[4 * d4] = fmaf(p, vv.x, ov[4 * d4]);
        ov[4 * d4 + 1] = fmaf(p, vv.y, ov[4 * d4 + 1]);
        ov[4 * d4 + 2] = fmaf(p, vv.z, ov[4 * d4 + 2]);
        ov[4 * d4 + 3] = fmaf(p, vv.w, ov[4 * d4 + 3]);
      }
    }
    mrun = mnew;
  }
  if (!live) return;
  float* op = a.o + b * a.osb + h * a.osh + (int64_t)qi * a.osn;
  const float inv = 1.0f / lrun;
#pragma unroll
  for (int d = 0; d < DMAX; ++d)
    if (d < a.d) op[d] = ov[d] * inv;
}

constexpr int DT = 256;

__global__ void __launch_bounds__(DT)
attn_decode_kernel(AttnArgs a) {
  extern __shared__ float sm[];  // [m] scores, then 4*DMAX partials
  __shared__ float qs[DMAX];
  __shared__ float red[32];
  const int qi = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int hk = h / (a.heads / a.kv_heads);
  const float* qp = a.q + b * a.qsb + h * a.qsh + (int64_t)qi * a.qsn;
  if (threadIdx.x < DMAX) qs[threadIdx.x] = threadIdx.x < a.d ? qp[threadIdx.x] * a.scale : 0.f;
  __syncthreads();
  const float* kb = a.k + b * a.ksb + hk * a.ksh;
  const float* vb = a.v + b * a.vsb + hk * a.vsh;
  float lmax = -INFINITY;
  for (int j = threadIdx.x; j < a.m; j += DT) {
    float s = -INFINITY;
    if (allowed(a, qi, j)) {
      s = 0.f;
      const float* kr = kb + (int64_t)j * a.ksn;
      for (int d = 0; d < a.d; ++d) s = fmaf(qs[d], kr[d], s);
    }
    sm[j] = s;
    lmax = fmaxf(lmax, s);
  }
  const float mx = block_max(lmax, red);
  float lsum = 0.f;
  for (int j = threadIdx.x; j < a.m; j += DT) {
    const float p = (mx == -INFINITY) ? 0.f : expf(sm[j] - mx);
    sm[j] = p;
    lsum += p;
  }
  const float sum = block_sum(lsum, red);  // also orders the sm[] writes above
  float* part = sm + a.m;
  const int d = threadIdx.x % DMAX, grp = threadIdx.x / DMAX;  // 4 groups of 64
  float acc = 0.f;
  if (d < a.d)
    for (int j = grp; j < a.m; j += DT / DMAX) acc = fmaf(sm[j], vb[(int64_t)j * a.vsn + d], acc);
  part[grp * DMAX + d] = acc;
  __syncthreads();
  if (threadIdx.x < a.d) {
    float o = 0.f;
#pragma unroll
    for (int g = 0; g < DT / DMAX; ++g) o += part[g * DMAX + threadIdx.x];
    a.o[b * a.osb + h * a.osh + (int64_t)qi * a.osn + threadIdx.x] = o / sum;
  }
}

}  // namespace

extern "C" int cv3_attention(const float* q, int64_t qsb, int64_t qsh, int64_t qsn,
                             const float* k, int64_t ksb, int64_t ksh, int64_t ksn,
                             const float* v, int64_t vsb, int64_t vsh, int64_t vsn,
                             float* o, int64_t osb, int64_t osh, int64_t osn,
                             int64_t batch, int64_t heads, int64_t kv_heads, int64_t n, int64_t m, int64_t d,
                             float scale, int mask_kind, int64_t mask_a, int64_t mask_b, void* stream) {
  CV3_REQUIRE(batch >= 0 && heads > 0 && kv_heads > 0 && n >= 0 && m >= 0, CV3_ERR_VALUE, "attention: bad shape");
  CV3_REQUIRE(heads % kv_heads == 0, CV3_ERR_VALUE, "%lld query heads is not a multiple of %lld kv heads",
              (long long)heads, (long long)kv_heads);
  CV3_REQUIRE(d >= 1 && d <= DMAX, CV3_ERR_UNSUPPORTED, "attention: head dim %lld > %d not built", (long long)d, DMAX);
  CV3_REQUIRE(d % 4 == 0 && ksn % 4 == 0 && vsn % 4 == 0 && ksh % 4 == 0 && vsh % 4 == 0 && ksb % 4 == 0 &&
                  vsb % 4 == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0,
              CV3_ERR_UNSUPPORTED, "attention: head dim, key/value strides and bases must be 16-byte multiples");
  CV3_REQUIRE(mask_kind >= 0 && mask_kind <= 2, CV3_ERR_VALUE, "attention: unknown mask kind %d", mask_kind);
  CV3_REQUIRE(mask_kind != 2 || mask_a > 0, CV3_ERR_VALUE, "attention: chunk size must be positive");
  if (batch == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(m > 0, CV3_ERR_VALUE, "attention: no keys");
  CV3_REQUIRE(n < (1LL << 30) && m < (1LL << 30) && batch * heads <= 65535, CV3_ERR_VALUE, "attention: too large");
  AttnArgs a{q, k, v, o, qsb, qsh, qsn, ksb, ksh, ksn, vsb, vsh, vsn, osb, osh, osn,
             (int)heads, (int)kv_heads, (int)n, (int)m, (int)d, scale, mask_kind, (int)mask_a, (int)mask_b};
  cudaStream_t st = cv3::as_stream(stream);
  if (n <= 4) {
    const int64_t smem = (m + 4 * DMAX) * 4;
    CV3_REQUIRE(smem <= 200 * 1024, CV3_ERR_UNSUPPORTED, "attention: %lld keys exceed the decode kernel", (long long)m);
    if (smem > 48 * 1024) {
      int rc = cv3::allow_smem((const void*)attn_decode_kernel, (int)smem);
      if (rc) return rc;
    }
    dim3 grid((unsigned)n, (unsigned)(batch * heads));
    attn_decode_kernel<<<grid, DT, (size_t)smem, st>>>(a);
    return cv3::check_launch("attention_decode");
  }
  dim3 grid((unsigned)((n + QT - 1) / QT), (unsigned)(batch * heads));
  attn_full_kernel<<<grid, QT, 0, st>>>(a);
  return cv3::check_launch("attention_full");
}

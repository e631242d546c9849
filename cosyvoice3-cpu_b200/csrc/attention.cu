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
#include "tc_common.cuh"

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

template <bool VEC>
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
      kpre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      vpre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok && VEC) {
        kpre[u] = *reinterpret_cast<const float4*>(kb + (int64_t)j * a.ksn + c);
        vpre[u] = *reinterpret_cast<const float4*>(vb + (int64_t)j * a.vsn + c);
      } else if (ok) {
        float* kp = reinterpret_cast<float*>(&kpre[u]);
        float* vp = reinterpret_cast<float*>(&vpre[u]);
        for (int e = 0; e < 4 && c + e < a.d; ++e) {
          kp[e] = kb[(int64_t)j * a.ksn + c + e];
          vp[e] = vb[(int64_t)j * a.vsn + c + e];
        }
      }
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

// ---------------------------------------------------------------------------
// Tensor-core path for head dim 64: flash-attention tiling on tcgen05, 3xTF32.
//
// CTA = one (batch, head) and 128 queries; keys in 64-key tiles through a
// 3-stage TMA ring (K and V read in place through 4-D tensor maps over the
// strided layout).  10 warps:
//   warp 0     TMA producer (K and V tiles, SWIZZLE_128B);
//   warp 1     MMA issuer: S_t = Q.K_t^T into TMEM, O_t = P_t.V_t into TMEM,
//              both as hi*lo + lo*hi + hi*hi tf32 products (fp32-accurate);
//              S_{t+2} is issued right behind O_t so the tensor pipe has work
//              while the softmax warps handle tile t+1;
//   warps 2-5  softmax, one query row per thread (= TMEM lane): running max,
//              P_t = 2^(s*log2e - m*log2e) split into tf32 hi/lo and written
//              back to TMEM, the row sum, and the rescale factor alpha_t of the
//              running output (shared memory);
//   warps 6-9  the scaled Q rows into TMEM once; then per tile the K tile split
//              in place into hi/lo, the V tile transposed and split (tf32 MMAs
//              take K-major operands only), and the fold o = o*alpha_u + O_u of
//              an earlier tile's output into registers; finally o / l stored.
// TMEM columns: Q hi | Q lo | S/P-hi x2 | P-lo x2 | O x2 (512).  Q and P are
// the A operands straight from TMEM; K and the transposed V are K-major B
// operands in shared memory.  Every wait is bounded; on a timeout the CTA
// records an error (cv3_tc_attention_status), drains what it issued and exits.
// ---------------------------------------------------------------------------
namespace tc {

using namespace cv3tc;

constexpr int BQ = 128, BKV = 64, HD = 64, STAGES = 3;
constexpr int HALF = BKV * 32 * 4;  // 8 KB: 64 keys x 32 floats (one TMA box, 128-byte rows)
constexpr int TILE = 2 * HALF;      // 16 KB: 64 keys x 64 floats
constexpr int STAGE = 4 * TILE;     // K hi | K lo | V hi | V lo
constexpr int THREADS = 320;
constexpr uint32_t C_QHI = 0, C_QLO = 64, C_S = 128, C_PLO = 256, C_O = 384;
constexpr uint32_t ID_S = idesc_tf32(BQ, BKV);
constexpr uint32_t ID_PV = idesc_tf32(BQ, HD);
constexpr float LOG2E = 1.4426950408889634f;

// byte offset of element (row, col) of a [rows][64] fp32 tile held as two
// 32-column TMA boxes of [rows][128 B] with the 128-byte swizzle (16-byte
// chunks XOR row % 8); boxes HALF bytes apart
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return (uint32_t)((col >> 5) * HALF + row * 128 + ((((col & 31) >> 2) ^ (row & 7)) << 4) + (col & 3) * 4);
}

struct Bars {
  uint64_t kfull[STAGES], vfull[STAGES], kconv[STAGES], vconv[STAGES], kempty[STAGES], vempty[STAGES];
  uint64_t sfull[2], pready[2], ofull[2], ofree[2], aready[4];
  uint64_t qready, done;
  uint32_t tmem;
  int abort_flag;
  int issued_k[STAGES], issued_v[STAGES];
  float alpha[4][BQ];  // rescale factor of the running output, per tile (mod 4) and row
  float lfin[BQ];      // final softmax denominators
};
constexpr int SMEM = STAGES * STAGE + 1024 + (int)sizeof(Bars);

__device__ int g_attn_err = 0;

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, int code) {
  return cv3tc::mbar_wait(bar, parity, &g_attn_err, code);
}

template <int MASK>
__device__ __forceinline__ bool visible(const AttnArgs& a, int qi, int kj) {
  if (MASK == 1) return kj <= qi + a.mask_a;
  if (MASK == 2) {
    const int c = qi / a.mask_a;
    const int start = a.mask_b < 0 ? 0 : max((c - a.mask_b) * a.mask_a, 0);
    return kj < (c + 1) * a.mask_a && kj >= start;
  }
  return true;
}

template <int MASK>
__global__ void __launch_bounds__(THREADS, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& B = *reinterpret_cast<Bars*>(smem + STAGES * STAGE);
  volatile int* abort_flag = &B.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int hk = h / (a.heads / a.kv_heads);
  const int q0 = blockIdx.x * BQ;
  const int qlast = min(a.n, q0 + BQ) - 1;
  // keys any query of this CTA may see
  int kbeg = 0, kend = a.m;
  if (MASK == 1) {
    kend = (int)min((long long)a.m, (long long)qlast + a.mask_a + 1);
  } else if (MASK == 2) {
    kend = (int)min((long long)a.m, ((long long)qlast / a.mask_a + 1) * a.mask_a);
    if (a.mask_b >= 0) kbeg = max((q0 / a.mask_a - a.mask_b) * a.mask_a, 0);
  }
  const int tbeg = kbeg / BKV;
  const int nt = kend > kbeg ? (kend + BKV - 1) / BKV - tbeg : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&B.kfull[s], 1);
      mbar_init(&B.vfull[s], 1);
      mbar_init(&B.kconv[s], 4);
      mbar_init(&B.vconv[s], 4);
      mbar_init(&B.kempty[s], 1);
      mbar_init(&B.vempty[s], 1);
      B.issued_k[s] = -1;
      B.issued_v[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.sfull[i], 1);
      mbar_init(&B.pready[i], 4);
      mbar_init(&B.ofull[i], 1);
      mbar_init(&B.ofree[i], 4);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&B.aready[i], 4);
    mbar_init(&B.qready, 4);
    mbar_init(&B.done, 1);
    B.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = B.tmem;

  if (warp == 0) {
    // ---- TMA producer ----------------------------------------------------------------
    if (lane == 0) {
      for (int t = 0; t < nt; ++t) {
        const int s = t % STAGES;
        const uint32_t r = (uint32_t)(t / STAGES);
        const int key0 = (tbeg + t) * BKV;
        uint8_t* st = smem + s * STAGE;
        if (*abort_flag || !bwait(&B.kempty[s], (r & 1) ^ 1, 1)) {
          *abort_flag = 1;
          break;
        }
        B.issued_k[s] = (int)r;
        mbar_expect_tx(&B.kfull[s], TILE);
        tma_load_4d(st, &kmap, &B.kfull[s], 0, key0, hk, b);
        tma_load_4d(st + HALF, &kmap, &B.kfull[s], 32, key0, hk, b);
        if (*abort_flag || !bwait(&B.vempty[s], (r & 1) ^ 1, 2)) {
          *abort_flag = 1;
          break;
        }
        B.issued_v[s] = (int)r;
        mbar_expect_tx(&B.vfull[s], TILE);
        tma_load_4d(st + 2 * TILE, &vmap, &B.vfull[s], 0, key0, hk, b);
        tma_load_4d(st + 2 * TILE + HALF, &vmap, &B.vfull[s], 32, key0, hk, b);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: the whole warp runs the loop, one elected lane issues ------------------
    {
      // every lane waits; the outcome is made warp-uniform before any MMA
      auto ready = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
        const bool ok = !*abort_flag && bwait(bar, parity, code);
        return __all_sync(0xffffffffu, ok);
      };
      auto issue_s = [&](int t) -> bool {
        const int s = t % STAGES;
        const uint32_t r = (uint32_t)(t / STAGES);
        if (!ready(&B.kconv[s], r & 1, 3)) return false;
        fence_after();
        const uint32_t khi = smem_u32(smem + s * STAGE), klo = khi + TILE;
        const uint32_t d = tmem + C_S + 64u * (t & 1);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * HALF + (kk & 3) * 32);
          mma_ts(d, tmem + C_QHI + 8 * kk, desc_k_sw128(klo + off), ID_S, kk > 0 ? 1u : 0u);
          mma_ts(d, tmem + C_QLO + 8 * kk, desc_k_sw128(khi + off), ID_S, 1u);
          mma_ts(d, tmem + C_QHI + 8 * kk, desc_k_sw128(khi + off), ID_S, 1u);
        }
        mma_commit(&B.sfull[t & 1]);
        mma_commit(&B.kempty[s]);
        return true;
      };
      auto issue_pv = [&](int t) -> bool {
        const int s = t % STAGES;
        const uint32_t r = (uint32_t)(t / STAGES);
        if (!ready(&B.pready[t & 1], (uint32_t)(t >> 1) & 1, 4)) return false;
        if (!ready(&B.vconv[s], r & 1, 5)) return false;
        if (t >= 2 && !ready(&B.ofree[t & 1], (uint32_t)((t - 2) >> 1) & 1, 6)) return false;
        fence_after();
        const uint32_t vhi = smem_u32(smem + s * STAGE + 2 * TILE), vlo = vhi + TILE;
        const uint32_t d = tmem + C_O + 64u * (t & 1);
        const uint32_t phi = tmem + C_S + 64u * (t & 1), plo = tmem + C_PLO + 64u * (t & 1);
#pragma unroll
        for (int kk = 0; kk < BKV / 8; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * HALF + (kk & 3) * 32);
          mma_ts(d, phi + 8 * kk, desc_k_sw128(vlo + off), ID_PV, kk > 0 ? 1u : 0u);
          mma_ts(d, plo + 8 * kk, desc_k_sw128(vhi + off), ID_PV, 1u);
          mma_ts(d, phi + 8 * kk, desc_k_sw128(vhi + off), ID_PV, 1u);
        }
        mma_commit(&B.ofull[t & 1]);
        mma_commit(&B.vempty[s]);
        return true;
      };
      bool ok = nt == 0 || ready(&B.qready, 0, 7);
      if (ok && nt > 0) {
        fence_after();
        ok = issue_s(0) && (nt < 2 || issue_s(1));
        for (int t = 0; ok && t < nt; ++t) ok = issue_pv(t) && (t + 2 >= nt || issue_s(t + 2));
      }
      if (!ok && lane == 0) *abort_flag = 1;
      mma_commit(&B.done);  // arrives once everything issued above has completed
    }
  } else if (warp < 6) {
    // ---- softmax (warps 2-5) -------------------------------------------------------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float mrun = -INFINITY, l = 0.f;
    for (int t = 0; t < nt; ++t) {
      const int key0 = (tbeg + t) * BKV;
      // S_t done also means O_{t-2} is done (the pipe runs in issue order), so the
      // P-lo buffer of this parity is free again
      bool go = !*abort_flag && bwait(&B.sfull[t & 1], (uint32_t)(t >> 1) & 1, 11);
      go = __all_sync(0xffffffffu, go);
      if (!go) {
        *abort_flag = 1;
        break;
      }
      fence_after();
      float sv[BKV];
      tmem_ld64(tmem + lane_base + C_S + 64u * (t & 1), sv);
      if (MASK != 0 || key0 + BKV > a.m) {
#pragma unroll
        for (int j = 0; j < BKV; ++j)
          if (key0 + j >= a.m || !visible<MASK>(a, qi, key0 + j)) sv[j] = -INFINITY;
      }
      float mx[BKV / 2];
#pragma unroll
      for (int j = 0; j < BKV / 2; ++j) mx[j] = fmaxf(sv[j], sv[j + BKV / 2]);
#pragma unroll
      for (int w = BKV / 4; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) mx[j] = fmaxf(mx[j], mx[j + w]);
      const float mnew = fmaxf(mrun, mx[0]);
      const float mlog = mnew == -INFINITY ? 0.f : mnew * LOG2E;
      const float alpha = mrun == -INFINITY ? 0.f : ex2(fmaf(mrun, LOG2E, -mlog));
      float lo[BKV];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < BKV; ++j) {
        const float p = ex2(fmaf(sv[j], LOG2E, -mlog));
        ps[j & 3] += p;
        sv[j] = tf32_hi(p);
        lo[j] = p - sv[j];
      }
      tmem_st64(tmem + lane_base + C_S + 64u * (t & 1), sv);
      tmem_st64(tmem + lane_base + C_PLO + 64u * (t & 1), lo);
      l = l * alpha + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
      mrun = mnew;
      B.alpha[t & 3][row] = alpha;
      if (t == nt - 1) B.lfin[row] = l;
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&B.pready[t & 1]);
        mbar_arrive(&B.aready[t & 3]);
      }
    }
  } else {
    // ---- Q into TMEM; K/V tiles split; output folds (warps 6-9) ---------------------------
    const int quarter = warp & 3;
    const int cw = warp - 6;          // converter warp 0..3
    const int ctid = threadIdx.x - 192;
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    if (nt > 0) {
      const float* qp = a.q + (int64_t)b * a.qsb + (int64_t)h * a.qsh + (int64_t)min(qi, a.n - 1) * a.qsn;
      float hi[HD], lo[HD];
#pragma unroll
      for (int c4 = 0; c4 < HD / 4; ++c4) {
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < a.n) x = *reinterpret_cast<const float4*>(qp + c4 * 4);
        const float xs[4] = {x.x * a.scale, x.y * a.scale, x.z * a.scale, x.w * a.scale};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[c4 * 4 + e] = tf32_hi(xs[e]);
          lo[c4 * 4 + e] = xs[e] - hi[c4 * 4 + e];
        }
      }
      tmem_st64(tmem + lane_base + C_QHI, hi);
      tmem_st64(tmem + lane_base + C_QLO, lo);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.qready);
    }
    float o[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] = 0.f;
    bool ok = true;
    // o = o * alpha_u + O_u, then hand the O buffer back to the MMA warp
#define CV3_FOLD(u)                                                                               \
  {                                                                                               \
    const int u_ = (u);                                                                           \
    bool go_ = !*abort_flag && bwait(&B.aready[u_ & 3], (uint32_t)(u_ >> 2) & 1, 10) &&           \
               bwait(&B.ofull[u_ & 1], (uint32_t)(u_ >> 1) & 1, 12);                              \
    go_ = __all_sync(0xffffffffu, go_);                                                           \
    if (!go_) {                                                                                   \
      ok = false;                                                                                 \
    } else {                                                                                      \
      fence_after();                                                                              \
      const float al_ = B.alpha[u_ & 3][row];                                                     \
      float ov_[HD];                                                                              \
      tmem_ld64(tmem + lane_base + C_O + 64u * (u_ & 1), ov_);                                    \
      _Pragma("unroll") for (int c = 0; c < HD; ++c) o[c] = fmaf(o[c], al_, ov_[c]);              \
      fence_before();                                                                             \
      __syncwarp();                                                                               \
      if (lane == 0) mbar_arrive(&B.ofree[u_ & 1]);                                               \
    }                                                                                             \
  }
    for (int t = 0; ok && t < nt; ++t) {
      const int s = t % STAGES;
      const uint32_t r = (uint32_t)(t / STAGES);
      uint8_t* st = smem + s * STAGE;
      bool go = !*abort_flag && bwait(&B.kfull[s], r & 1, 8);
      go = __all_sync(0xffffffffu, go);
      if (!go) {
        ok = false;
        break;
      }
      split_tile(reinterpret_cast<float*>(st), reinterpret_cast<float*>(st + TILE), TILE, ctid, 128);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.kconv[s]);
      go = !*abort_flag && bwait(&B.vfull[s], r & 1, 9);
      go = __all_sync(0xffffffffu, go);
      if (!go) {
        ok = false;
        break;
      }
      {
        // V_t arrives as [key][d]; the MMA wants V_t^T [d][key] as a K-major operand,
        // so the tile is transposed while it is split.  Reads: float4 along d, eight
        // consecutive keys per quarter-warp (distinct swizzled chunks); writes: a warp
        // covers 32 consecutive keys of one d row (32 distinct banks).  All reads
        // finish (barrier of the four converter warps) before the in-place writes.
        uint8_t* vraw = st + 2 * TILE;
        uint8_t* vlo = st + 3 * TILE;
        float4 rv[2][4];
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4)
            rv[kb][i4] = *reinterpret_cast<const float4*>(vraw + swz(lane + 32 * kb, 4 * (cw * 4 + i4)));
        asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int i4 = 0; i4 < 4; ++i4) {
            const float xv[4] = {rv[kb][i4].x, rv[kb][i4].y, rv[kb][i4].z, rv[kb][i4].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t off = swz(4 * (cw * 4 + i4) + e, lane + 32 * kb);
              const float hv = tf32_hi(xv[e]);
              *reinterpret_cast<float*>(vraw + off) = hv;
              *reinterpret_cast<float*>(vlo + off) = xv[e] - hv;
            }
          }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.vconv[s]);
      if (t >= 2) CV3_FOLD(t - 2);
    }
    if (ok && nt >= 2) CV3_FOLD(nt - 2);
    if (ok && nt >= 1) CV3_FOLD(nt - 1);
#undef CV3_FOLD
    if (!ok) *abort_flag = 1;
    if (ok && qi < a.n) {
      const float inv = 1.0f / B.lfin[row];
      float* op = a.o + (int64_t)b * a.osb + (int64_t)h * a.osh + (int64_t)qi * a.osn;
#pragma unroll
      for (int c4 = 0; c4 < HD / 4; ++c4)
        reinterpret_cast<float4*>(op)[c4] =
            make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv, o[4 * c4 + 2] * inv, o[4 * c4 + 3] * inv);
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      if (*abort_flag) {
        // let every issued TMA copy land before the shared memory is released
        for (int s = 0; s < STAGES; ++s) {
          if (B.issued_k[s] >= 0) bwait(&B.kfull[s], (uint32_t)B.issued_k[s] & 1, 13);
          if (B.issued_v[s] >= 0) bwait(&B.vfull[s], (uint32_t)B.issued_v[s] & 1, 14);
        }
      }
      bwait(&B.done, 0, 15);  // every MMA (and its barrier arrivals) finished
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// 4-D map (head dim, keys, kv heads, batch) over a strided K or V; size-1 modes
// get a nominal stride (they are never stepped).
int make_kv_map(CUtensorMap* map, const float* base, int64_t m, int64_t kv_heads, int64_t batch, int64_t sn, int64_t sh,
                int64_t sb) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  CV3_REQUIRE(encode != nullptr, CV3_ERR_CUDA, "attention: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)m, (cuuint64_t)kv_heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(sn * 4), (cuuint64_t)((kv_heads > 1 ? sh : sn) * 4),
                           (cuuint64_t)((batch > 1 ? sb : sn) * 4)};
  for (int i = 0; i < 3; ++i)
    CV3_REQUIRE(strides[i] > 0 && strides[i] % 16 == 0 && strides[i] < (1ull << 40), CV3_ERR_VALUE,
                "attention: key/value stride not usable by TMA");
  cuuint32_t box[4] = {32, (cuuint32_t)BKV, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CV3_REQUIRE(r == CUDA_SUCCESS, CV3_ERR_CUDA, "attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CV3_OK;
}

int launch(const AttnArgs& a, int64_t batch, cudaStream_t st) {
  CUtensorMap km, vm;
  int rc = make_kv_map(&km, a.k, a.m, a.kv_heads, batch, a.ksn, a.ksh, a.ksb);
  if (rc) return rc;
  rc = make_kv_map(&vm, a.v, a.m, a.kv_heads, batch, a.vsn, a.vsh, a.vsb);
  if (rc) return rc;
  auto fn = a.mask_kind == 1 ? attn_tc_kernel<1> : (a.mask_kind == 2 ? attn_tc_kernel<2> : attn_tc_kernel<0>);
  rc = cv3::allow_smem((const void*)fn, SMEM);
  if (rc) return rc;
  dim3 grid((unsigned)((a.n + BQ - 1) / BQ), (unsigned)(batch * a.heads));
  fn<<<grid, THREADS, SMEM, st>>>(km, vm, a);
  return cv3::check_launch("attention_tc");
}

}  // namespace tc

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
  const bool kv16 = d % 4 == 0 && ksn % 4 == 0 && vsn % 4 == 0 && ksh % 4 == 0 && vsh % 4 == 0 && ksb % 4 == 0 &&
                   vsb % 4 == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0;
  const bool qo16 = qsn % 4 == 0 && qsh % 4 == 0 && qsb % 4 == 0 && ((uintptr_t)q & 15) == 0 && osn % 4 == 0 &&
                    osh % 4 == 0 && osb % 4 == 0 && ((uintptr_t)o & 15) == 0;
  if (d == tc::HD && kv16 && qo16) return tc::launch(a, batch, st);
  dim3 grid((unsigned)((n + QT - 1) / QT), (unsigned)(batch * heads));
  if (kv16) attn_full_kernel<true><<<grid, QT, 0, st>>>(a);
  else attn_full_kernel<false><<<grid, QT, 0, st>>>(a);
  return cv3::check_launch("attention_full");
}

extern "C" int cv3_tc_attention_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, tc::g_attn_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(tc::g_attn_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

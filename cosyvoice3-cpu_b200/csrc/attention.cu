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
// Tensor-core path for head dim 64: flash-attention tiling on tcgen05 with fp16
// operands carrying fp32 precision.
//
// Every fp32 operand enters as two fp16 parts, hi = fp16(x * 2^e) and
// lo = fp16(x * 2^e - hi), with e a power of two chosen per query row (Q), per
// 64-key tile (K and V) or not at all (P, which lies in [0, 1]): 22 significant
// bits relative to the row's / tile's largest value.  Products are hi*hi + hi*lo
// + lo*hi in kind::f16 (K = 16 per MMA: half the instructions of 3xTF32, whose
// K is 8), accumulated in fp32; the scales come off in the softmax (per row and
// tile) and in the output fold (per tile).  Measured against fp64 this matches
// the 3xTF32 scheme it replaces.
//
// CTA = one (batch, head) and 128 queries; keys in 64-key tiles through a
// 3-stage TMA ring (K and V read in place through 4-D tensor maps over the
// strided layout).  10 warps:
//   warp 0     TMA producer (K and V tiles as fp32, SWIZZLE_128B);
//   warp 1     MMA issuer: S_t = Q.K_t^T into TMEM, O_t = P_t.V_t into TMEM;
//              S_{t+2} is issued right behind O_t so the tensor pipe has work
//              while the softmax warps handle tile t+1;
//   warps 2-5  softmax, one query row per thread (= TMEM lane): running max,
//              P_t = 2^(s*log2e - m*log2e) split into fp16 hi/lo written back
//              over S_t in TMEM, the row sum, and the rescale factor alpha_t of
//              the running output (shared memory); then K_{t+2} as fp16 hi/lo
//              tiles (UMMA K-major, 128 B swizzle) with the tile's exponent;
//   warps 6-9  the scaled Q rows into TMEM once; then per tile V as fp16 hi/lo
//              tiles in its stored [key][dim] order (an MN-major B operand of
//              P.V) with the tile's exponent, and the fold o = o*alpha +
//              O_u*2^-e_v(u) of an earlier tile's output into registers;
//              finally o / l stored.
// TMEM columns: Q hi | Q lo (32 each: two fp16 per column) | S/P x2 | O x2.
// Q and P are the A operands straight from TMEM; K (K-major) and V (MN-major)
// are B operands in shared memory.  Every wait is bounded; on a timeout the CTA records an error
// (cv3_tc_attention_status), drains what it issued and exits.
// ---------------------------------------------------------------------------
namespace tc {

using namespace cv3tc;

constexpr int BQ = 128, BKV = 64, HD = 64, STAGES = 3;
constexpr int HALF = BKV * 32 * 4;  // 8 KB: 64 keys x 32 floats (one TMA box, 128-byte rows)
constexpr int TILE = 2 * HALF;      // 16 KB: 64 keys x 64 floats
constexpr int T16 = BKV * HD * 2;   // 8 KB: a 64 x 64 fp16 tile, 128-byte rows
// stage: K fp32 | V fp32 | K hi | K lo | V hi | V lo
constexpr int ST_K = 0, ST_V = TILE, ST_KH = 2 * TILE, ST_KL = ST_KH + T16, ST_VH = ST_KL + T16, ST_VL = ST_VH + T16;
constexpr int STAGE = ST_VL + T16;  // 64 KB
constexpr int THREADS = 320;
constexpr uint32_t C_QHI = 0, C_QLO = 32, C_S = 64, C_O = 192;
constexpr uint32_t ID_S = (1u << 4) | ((uint32_t)(BKV >> 3) << 17) | ((uint32_t)(BQ >> 4) << 24);  // f16 x f16 -> f32
// P.V: B = V as stored, [key][dim] -- MN-major (bit 16), 8-key x 128 B swizzle atoms
constexpr uint32_t ID_PV = (1u << 4) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(BQ >> 4) << 24);
constexpr float LOG2E = 1.4426950408889634f;

// byte offset of element (row, col) of a [rows][64] fp32 tile held as two
// 32-column TMA boxes of [rows][128 B] with the 128-byte swizzle (16-byte
// chunks XOR row % 8); boxes HALF bytes apart
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return (uint32_t)((col >> 5) * HALF + row * 128 + ((((col & 31) >> 2) ^ (row & 7)) << 4) + (col & 3) * 4);
}

// byte offset of the 16-byte chunk holding fp16 elements [8 c, 8 c + 8) of row `row`
// of a [rows][64] fp16 tile in the UMMA K-major 128 B-swizzled layout
__device__ __forceinline__ uint32_t swz16(int row, int c) { return (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4)); }

// the exponent e with max * 2^e in [2^14, 2^15) (0 for an all-zero block), clamped
__device__ __forceinline__ int scale_exp(float amax) {
  if (!(amax > 0.f)) return 0;
  const int e = 14 - (((__float_as_int(amax) >> 23) & 0xFF) - 127);
  return e > 126 ? 126 : (e < -126 ? -126 : e);
}

__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// (a0, a1) -> fp16 hi and lo pairs, a0 in the low halves
__device__ __forceinline__ void split2(float a0, float a1, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(a1), "f"(a0));
  const __half2 h = *reinterpret_cast<const __half2*>(&hi);
  const float r0 = a0 - __low2float(h), r1 = a1 - __high2float(h);
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

// 32 lanes x 32 columns of packed words into TMEM
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// 12 kind::f16 MMAs (4 k-steps x hi*lo, lo*hi, hi*hi) into d, A from TMEM (hi at ah, lo
// at al; 8 columns per k-step), B from shared memory (descriptors bh, bl; BSTEP per
// k-step in 16-byte units: 2 for a K-major tile, 128 for two 8-row atoms of an MN-major
// one), one elected lane; d is overwritten by the first
template <int BSTEP>
__device__ __forceinline__ void mma12(uint32_t d, uint32_t ah, uint32_t al, uint64_t bh, uint64_t bl, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b32 a1, a2, a3, c1, c2, c3;\n\t"
      ".reg .b64 h1, h2, h3, l1, l2, l3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, %5, %5;\n\tsetp.eq.b32 pt, %5, %5;\n\t"
      "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
      "add.u32 c1, %2, 8;\n\tadd.u32 c2, %2, 16;\n\tadd.u32 c3, %2, 24;\n\t"
      "add.s64 h1, %3, %7;\n\tadd.s64 h2, %3, %8;\n\tadd.s64 h3, %3, %9;\n\t"
      "add.s64 l1, %4, %7;\n\tadd.s64 l2, %4, %8;\n\tadd.s64 l3, %4, %9;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %4, %6, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], l1, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [c1], h1, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], h1, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], l2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [c2], h2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], h2, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], l3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [c3], h3, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], h3, %6, pt;\n\t}" ::"r"(d),
      "r"(ah), "r"(al), "l"(bh), "l"(bl), "r"(0), "r"(idesc), "n"(BSTEP), "n"(2 * BSTEP), "n"(3 * BSTEP)
      : "memory");
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
  float qf[BQ];        // 2^-e of each query row's scaling
  float kf[8], vf[8];  // 2^-e of each key / value tile's scaling (tile mod 8)
  float red[2][4];     // the converter warps' tile maxima (K, V)
};
constexpr int SMEM = STAGES * STAGE + 1024 + (int)sizeof(Bars);

// The four warps of a role (softmax: named barrier 2, converters: 1) agree on `ok`: a
// barrier over their 128 threads that every thread reaches, so they leave together.
__device__ __forceinline__ bool agree128(bool ok, int bar) {
  uint32_t all;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(all)
      : "r"((uint32_t)ok), "r"(bar)
      : "memory");
  return all != 0;
}

// the largest of the four warps' values m (named barrier `bar` + four shared slots)
__device__ __forceinline__ float max128(float m, float* red4, int w, int lane, int bar) {
  m = warp_max(m);
  if (lane == 0) red4[w] = m;
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  return fmaxf(fmaxf(red4[0], red4[1]), fmaxf(red4[2], red4[3]));
}

// A K or V tile (fp32 [key][dim], as TMA wrote it at `src`) -> fp16 hi / lo tiles at `dh`
// / `dl`, [key][dim] rows of 128 B with the 128 B swizzle -- K-major for K (dims are its
// MMA K), MN-major for V (keys are its MMA K) -- scaled by the tile's exponent (2^-e into
// *kf); thread i of the 128 takes key i / 2, dims 32 (i % 2) .. + 31
__device__ __forceinline__ void convert_rows(uint8_t* st, int src, int dh, int dl, int i, float* kf, float* red4, int w,
                                             int lane, int bar) {
  const int kr = i >> 1, kh = i & 1;
  float kv[32];
  float am = 0.f;
#pragma unroll
  for (int i4 = 0; i4 < 8; ++i4) {
    const float4 x = *reinterpret_cast<const float4*>(st + src + swz(kr, 32 * kh + 4 * i4));
    kv[4 * i4] = x.x;
    kv[4 * i4 + 1] = x.y;
    kv[4 * i4 + 2] = x.z;
    kv[4 * i4 + 3] = x.w;
    am = fmaxf(fmaxf(am, fmaxf(fabsf(x.x), fabsf(x.y))), fmaxf(fabsf(x.z), fabsf(x.w)));
  }
  const int e = scale_exp(max128(am, red4, w, lane, bar));
  const float sc = pow2i(e);
  if (i == 0) *kf = pow2i(-e);
#pragma unroll
  for (int c = 0; c < 4; ++c) {  // 8 dims per 16-byte chunk
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split2(kv[8 * c + 2 * j] * sc, kv[8 * c + 2 * j + 1] * sc, hi[j], lo[j]);
    const uint32_t off = swz16(kr, 4 * kh + c);
    *reinterpret_cast<uint4*>(st + dh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(st + dl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

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
        tma_load_4d(st + ST_K, &kmap, &B.kfull[s], 0, key0, hk, b);
        tma_load_4d(st + ST_K + HALF, &kmap, &B.kfull[s], 32, key0, hk, b);
        if (*abort_flag || !bwait(&B.vempty[s], (r & 1) ^ 1, 2)) {
          *abort_flag = 1;
          break;
        }
        B.issued_v[s] = (int)r;
        mbar_expect_tx(&B.vfull[s], TILE);
        tma_load_4d(st + ST_V, &vmap, &B.vfull[s], 0, key0, hk, b);
        tma_load_4d(st + ST_V + HALF, &vmap, &B.vfull[s], 32, key0, hk, b);
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
      auto sbuf = [&](int t) -> uint32_t { return tmem + C_S + 64u * (uint32_t)(t & 1); };
      constexpr uint64_t T16D = T16 >> 4;  // the lo tile, in descriptor address units
      auto issue_s = [&](int t) -> bool {
        const int s = t % STAGES;
        if (!ready(&B.kconv[s], (uint32_t)(t / STAGES) & 1, 3)) return false;
        fence_after();
        const uint64_t kd = desc_k_sw128(smem_u32(smem + s * STAGE + ST_KH));
        mma12<2>(sbuf(t), tmem + C_QHI, tmem + C_QLO, kd, kd + T16D, ID_S);
        mma_commit(&B.sfull[t & 1]);
        mma_commit(&B.kempty[s]);
        return true;
      };
      auto issue_pv = [&](int t) -> bool {
        const int s = t % STAGES;
        if (!ready(&B.pready[t & 1], (uint32_t)(t >> 1) & 1, 4)) return false;
        if (!ready(&B.vconv[s], (uint32_t)(t / STAGES) & 1, 5)) return false;
        if (t >= 2 && !ready(&B.ofree[t & 1], (uint32_t)((t - 2) >> 1) & 1, 6)) return false;
        fence_after();
        const uint64_t vd = desc_k_sw128(smem_u32(smem + s * STAGE + ST_VH));
        // P hi in columns 0-31 of the S buffer, P lo in 32-63
        mma12<128>(tmem + C_O + 64u * (t & 1), sbuf(t), sbuf(t) + 32, vd, vd + T16D, ID_PV);
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
    const int sw = warp - 2, stid = threadIdx.x - 64;  // softmax warp 0..3, thread 0..127
    // the softmax warps also turn each K tile into fp16 parts: tiles 0 and 1 first, then
    // tile t + 2 right after the softmax of tile t (S_{t+2} is issued after O_t, which
    // waits for that softmax anyway)
    auto conv_k = [&](int t) -> bool {
      const int s = t % STAGES;
      if (!agree128(!*abort_flag && bwait(&B.kfull[s], (uint32_t)(t / STAGES) & 1, 8), 2)) return false;
      convert_rows(smem + s * STAGE, ST_K, ST_KH, ST_KL, stid, &B.kf[t & 7], B.red[0], sw, lane, 2);
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.kconv[s]);
      return true;
    };
    bool sok = nt == 0 || (conv_k(0) && (nt < 2 || conv_k(1)));
    // Q's row scale is written before qready, which the first S waited for
    float qf = 0.f;
    for (int t = 0; sok && t < nt; ++t) {
      const int key0 = (tbeg + t) * BKV;
      // S_t done also means O_{t-2}, the last reader of this buffer's P, is done (the
      // pipe runs in issue order)
      if (!agree128(!*abort_flag && bwait(&B.sfull[t & 1], (uint32_t)(t >> 1) & 1, 11), 2)) {
        sok = false;
        break;
      }
      fence_after();
      if (t == 0) qf = B.qf[row];
      const float f = qf * B.kf[t & 7];  // S = S' * 2^-(e_q + e_k)
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
      const float mnew = fmaxf(mrun, mx[0] * f);
      const float mlog = mnew == -INFINITY ? 0.f : mnew * LOG2E;
      const float alpha = mrun == -INFINITY ? 0.f : ex2(fmaf(mrun, LOG2E, -mlog));
      const float fl = f * LOG2E;
      uint32_t ph[BKV / 2], pl[BKV / 2];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < BKV; j += 2) {
        const float p0 = ex2(fmaf(sv[j], fl, -mlog)), p1 = ex2(fmaf(sv[j + 1], fl, -mlog));
        ps[j & 3] += p0;
        ps[(j + 1) & 3] += p1;
        split2(p0, p1, ph[j / 2], pl[j / 2]);
      }
      tmem_st32u(tmem + lane_base + C_S + 64u * (t & 1), ph);
      tmem_st32u(tmem + lane_base + C_S + 64u * (t & 1) + 32, pl);
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
      if (t + 2 < nt && !conv_k(t + 2)) sok = false;
    }
    if (!sok) *abort_flag = 1;
  } else {
    // ---- Q into TMEM; V tiles to fp16 parts; output folds (warps 6-9) ----------------------
    const int quarter = warp & 3;
    const int cw = warp - 6;          // converter warp 0..3
    const int ctid = threadIdx.x - 192;
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    if (nt > 0) {
      const float* qp = a.q + (int64_t)b * a.qsb + (int64_t)h * a.qsh + (int64_t)min(qi, a.n - 1) * a.qsn;
      float xs[HD];
      float am = 0.f;
#pragma unroll
      for (int c4 = 0; c4 < HD / 4; ++c4) {
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < a.n) x = *reinterpret_cast<const float4*>(qp + c4 * 4);
        xs[4 * c4] = x.x * a.scale;
        xs[4 * c4 + 1] = x.y * a.scale;
        xs[4 * c4 + 2] = x.z * a.scale;
        xs[4 * c4 + 3] = x.w * a.scale;
#pragma unroll
        for (int e = 0; e < 4; ++e) am = fmaxf(am, fabsf(xs[4 * c4 + e]));
      }
      const int e = scale_exp(am);
      const float sc = pow2i(e);
      uint32_t hi[HD / 2], lo[HD / 2];
#pragma unroll
      for (int j = 0; j < HD; j += 2) split2(xs[j] * sc, xs[j + 1] * sc, hi[j / 2], lo[j / 2]);
      B.qf[row] = pow2i(-e);
      tmem_st32u(tmem + lane_base + C_QHI, hi);
      tmem_st32u(tmem + lane_base + C_QLO, lo);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.qready);
    }
    float o[HD];
#pragma unroll
    for (int c = 0; c < HD; ++c) o[c] = 0.f;
    bool ok = true;
    // o = o * alpha_u + O_u * 2^-e_v(u), then hand the O buffer back to the MMA warp
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
      const float vf_ = B.vf[u_ & 7];                                                             \
      float ov_[HD];                                                                              \
      tmem_ld64(tmem + lane_base + C_O + 64u * (u_ & 1), ov_);                                    \
      _Pragma("unroll") for (int c = 0; c < HD; ++c) o[c] = fmaf(o[c], al_, ov_[c] * vf_);        \
      fence_before();                                                                             \
      __syncwarp();                                                                               \
      if (lane == 0) mbar_arrive(&B.ofree[u_ & 1]);                                               \
    }                                                                                             \
  }
    // every converter warp reaches each agreement (a failed fold included), so the four
    // leave the loop together and no named barrier waits for a warp that has left
    for (int t = 0; t < nt; ++t) {
      const int s = t % STAGES;
      const uint32_t r = (uint32_t)(t / STAGES);
      uint8_t* st = smem + s * STAGE;
      if (!agree128(ok && !*abort_flag && bwait(&B.vfull[s], r & 1, 9), 1)) {
        ok = false;
        break;
      }
      convert_rows(st, ST_V, ST_VH, ST_VL, ctid, &B.vf[t & 7], B.red[1], cw, lane, 1);
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

// The balanced DiT's linears on the 5th-generation tensor cores with the int8 weights
// used as they are stored (cv3cpu/quant.py:90-136: W[n][k] = q[n][k] * s[n][k / 64],
// q int8, s fp16; ops.linear -> quant.qmatmul, cv3cpu/quant.py:156-204):
//
//   C[M][N] = epilogue( sum_g s[n][g] * (A[M][64 g .. 64 g + 63] . q[n][64 g .. 64 g + 63]) )
//
// Why not dequantise and run fp32 (3xTF32): q is exactly representable in fp16, so the
// weight side needs no split at all; only the fp32 activations do.  Each 64-wide K group
// of an A row is scaled by a power of two that brings its largest element into
// [2^14, 2^15) and split into two fp16 parts, hi = fp16(a) and lo = fp16(a - hi) -- 22
// significant bits, the precision the 3xTF32 split gives A.  The group's partial sum
// P = A_hi . q + A_lo . q accumulates in fp32 in TMEM (kind::f16, 8 MMAs per group
// where 3xTF32 on dequantised weights issues 24 tf32 MMAs), and the epilogue warps
// promote it: acc[m][n] += P * 2^-e[m][g] * s[n][g] in fp32 registers.
//
// Persistent CTAs (one per SM) walk 128 x 128 output tiles; 14 warps (18 with A given
// as activation planes: no converters, sixteen promotion warps of 32 columns):
//   warp 0     TMA: per K group the A fp32 tile (two 32-wide SWIZZLE_128B boxes) and the
//              q tile (fp16, converted once at load); a stage is free again once the
//              converters have read A and the MMAs B;
//   warp 1     MMA issuer: per group 4 k-steps x (hi, lo) into the group's accumulator
//              (four in TMEM: the MMAs run up to three groups ahead of the promotion);
//   warps 2-5  converters: thread = A row: the row's 64 values, their exponent, the
//              hi / lo fp16 planes in the UMMA K-major SWIZZLE_128B layout;
//   warps 6-13 promotion and epilogue, two per TMEM lane quarter (64 columns each):
//              fold each group into fp32 registers, then bias / GELU-tanh / gated
//              residual and the stores (256-bit: a whole 32-byte sector of the row per
//              thread and instruction) while the MMA warp starts the next tile.
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel records an error
// (cv3_tc_gemm_q8_status), stops issuing work, lets what it issued finish and exits.
#include <algorithm>

#include "planes.cuh"
#include "tc_common.cuh"

namespace {

using namespace cv3tc;

constexpr int BM = 128, BN = 128, KG = 64;  // KG: one scale group
constexpr int STAGES = 3;                            // fp32 A: converted in the kernel
constexpr int STAGES_P = 3;                          // pre-split A planes: hi | lo | B per stage (3 measured faster than 2 or 4)
constexpr int TILE_A = BM * KG * 4;                  // 32 KB: two 32-wide fp32 boxes
constexpr int TILE_B = BN * KG * 2;                  // 16 KB: fp16 weights
constexpr int STAGE_BYTES = TILE_A + TILE_B;        // A | B (1 KB multiples: SW128 tiles)
constexpr int PLANES_AT = STAGES * STAGE_BYTES;      // 2 buffers x (hi | lo), 16 KB each
constexpr int PLANE = BM * KG * 2;                   // 16 KB
// warps: 0 TMA, 1 MMA; fp32 A: 2-5 converters, 6-13 promotion (64 columns each);
// pre-split A: 2-17 promotion (32 columns each: four warps per TMEM lane quarter)
template <bool P> struct Layout {
  static constexpr int THREADS = P ? 576 : 448;
  static constexpr int PW0 = P ? 2 : 6;    // first promotion warp
  static constexpr int NPW = P ? 16 : 8;   // promotion warps
  static constexpr int EPI_COLS = P ? 32 : 64;
};
constexpr int NACC = 4;  // TMEM accumulators (one per K group in flight), 128 columns each
constexpr int NSIDE = 8;                       // side ring: per group the tile's scales and exponents
constexpr int SIDE_BYTES = BN * 4 + BM;        // 512 B fp32 scales | 128 B int8 exponents
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);  // f16 x f16 -> f32

__device__ int g_q8_err = 0;

struct Bars {
  uint64_t full[STAGES_P], empty[STAGES_P], afull[2], aempty[2], pfull[NACC], pempty[NACC], done;
  uint64_t sfull[NSIDE], sempty[NSIDE];
  int sissued[NSIDE];
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES_P];
  // per (group mod 8, row): the power of two the converters scaled by.  Depth: converter
  // g waits for MMA g-2, which waits for the promotion of g-2-NACC, so the slot of
  // group g is rewritten only after its promotion when the depth is >= NACC + 2
  int ex[8][BM];
  float xmax[4][BM];  // mode 4 with 32-column threads: each column quarter's row maxima
};
constexpr int SIDE_AT = PLANES_AT + 4 * PLANE;   // after both layouts' stages / planes
constexpr int SMEM_BYTES = SIDE_AT + NSIDE * SIDE_BYTES + 1024 + (int)sizeof(Bars);

struct Epi {
  int mode;  // 0: +bias; 1: gelu_tanh(+bias); 2: h += gate * (+bias); 3: h += (+bias);
             // 4: gelu_tanh(+bias) written as activation planes (oplanes, oexps, olde)
  const float* bias;
  const float* gate;
  int64_t rows_per_group, gate_stride;
  __half* oplanes;
  int8_t* oexps;
  int64_t olde;
};

__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  const float inner = x + 0.044715f * x * x * x;
  return 0.5f * x * (1.0f + tanhf(c * inner));
}

// 32 lanes x 16 consecutive columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])::"memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive columns, without waiting (see tmem_wait64)
__device__ __forceinline__ void tmem_issue32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// wait for the issued TMEM loads; naming every destination register keeps their uses
// after the wait
__device__ __forceinline__ void tmem_wait64(uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                 "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]),
                 "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]),
                 "+r"(a[29]), "+r"(a[30]), "+r"(a[31]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]),
                 "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]),
                 "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]),
                 "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]),
                 "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31])::"memory");
}

__device__ __forceinline__ uint32_t f2h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void h22f(uint32_t h, float& lo, float& hi) {
  __half2 v = *reinterpret_cast<__half2*>(&h);
  lo = __low2float(v);
  hi = __high2float(v);
}

// the exponent e with max|x| * 2^e in [2^14, 2^15), clamped to [-126, 126]
__device__ __forceinline__ int group_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  const int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
  const int s = 14 - e;
  return s > 126 ? 126 : (s < -126 ? -126 : s);
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// 256-bit global accesses (sm_100): a thread writes or reads a whole 32-byte sector of
// its row at once (32-byte aligned addresses)
__device__ __forceinline__ void st8(void* p, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t a4,
                                    uint32_t a5, uint32_t a6, uint32_t a7) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a0), "r"(a1), "r"(a2), "r"(a3),
               "r"(a4), "r"(a5), "r"(a6), "r"(a7)
               : "memory");
}

__device__ __forceinline__ void ld8(const float* p, float* v) {
  asm volatile("ld.global.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p)
               : "memory");
}

// One K group's MMAs: 4 k-steps of 16, A hi and A lo into the group's accumulator d,
// the weights from one descriptor; then the commits that free the stage, the A planes
// and hand the accumulator to the promotion.
template <bool PLANES_BAR>
__device__ __forceinline__ void issue_group(uint32_t d, uint64_t ahi, uint64_t alo, uint64_t b,
                                            uint64_t* bar_stage, uint64_t* bar_planes, uint64_t* bar_acc) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t"
      ".reg .b64 h1, h2, h3, l1, l2, l3, b1, b2, b3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, %5, %5;\n\tsetp.eq.b32 pt, %5, %5;\n\t"
      "add.s64 h1, %1, 2;\n\tadd.s64 h2, %1, 4;\n\tadd.s64 h3, %1, 6;\n\t"
      "add.s64 l1, %2, 2;\n\tadd.s64 l2, %2, 4;\n\tadd.s64 l3, %2, 6;\n\t"
      "add.s64 b1, %3, 2;\n\tadd.s64 b2, %3, 4;\n\tadd.s64 b3, %3, 6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %3, %4, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %3, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], h1, b1, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], l1, b1, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], h2, b2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], l2, b2, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], h3, b3, %4, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], l3, b3, %4, pt;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%6];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t}" ::"r"(d),
      "l"(ahi), "l"(alo), "l"(b), "r"(IDESC), "r"(0), "r"(smem_u32(bar_stage)), "r"(smem_u32(bar_acc))
      : "memory");
  if (PLANES_BAR) mma_commit(bar_planes);
}

// PRESPLIT: A arrives as activation planes (planes.cuh) by TMA -- hi | lo | B per
// stage, three stages, no converter warps; the promotion reads the exponents from
// pexp.  Otherwise A is fp32 and the converter warps split it.
template <bool PRESPLIT>
__global__ void __launch_bounds__(Layout<PRESPLIT>::THREADS, 1)
tc_gemm_q8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_e, int M, int N,
                  int K, float* __restrict__ C, int64_t ldc, Epi ep) {
  constexpr int NST = PRESPLIT ? STAGES_P : STAGES;
  constexpr int EPI_COLS = Layout<PRESPLIT>::EPI_COLS, NPW = Layout<PRESPLIT>::NPW, PW0 = Layout<PRESPLIT>::PW0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& S = *reinterpret_cast<Bars*>(smem + SIDE_AT + NSIDE * SIDE_BYTES);
  uint8_t* side = smem + SIDE_AT;
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = K / KG;
  const int tiles_n = N / BN;
  const int ntiles = tiles_n * ((M + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], PRESPLIT ? 1 : 1 + 4);  // MMA commit (B, and A planes), converter warps (fp32 A)
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.afull[i], 4);
      mbar_init(&S.aempty[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&S.pfull[i], 1);
      mbar_init(&S.pempty[i], NPW);
    }
    for (int i = 0; i < NSIDE; ++i) {
      mbar_init(&S.sfull[i], 1);
      mbar_init(&S.sempty[i], NPW);
      S.sissued[i] = -1;
    }
    mbar_init(&S.done, 1);
    S.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S.tmem;
  // warp-uniform wait: one try_wait and a vote when the phase has completed already
  auto ready = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (__all_sync(0xffffffffu, mbar_test(bar, parity))) return true;
    const bool ok = !*abort_flag && mbar_wait(bar, parity, &g_q8_err, code);
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      int g = 0;
      bool go = true;
      for (int tile = blockIdx.x; go && tile < ntiles; tile += gridDim.x) {
        const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
        for (int kg = 0; kg < ng; ++kg, ++g) {
          const int s = g % NST;
          const uint32_t r = (uint32_t)(g / NST);
          if (*abort_flag || !mbar_wait(&S.empty[s], (r & 1) ^ 1, &g_q8_err, 1)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          S.issued[s] = (int)r;
          mbar_expect_tx(&S.full[s], TILE_A + TILE_B);
          if (PRESPLIT) {
            tma_load_2d(st, &map_a, &S.full[s], 2 * KG * kg, m0);            // hi plane of the group
            tma_load_2d(st + PLANE, &map_a, &S.full[s], 2 * KG * kg + KG, m0);  // lo plane
          } else {
            tma_load_2d(st, &map_a, &S.full[s], kg * KG, m0);
            tma_load_2d(st + TILE_A / 2, &map_a, &S.full[s], kg * KG + KG / 2, m0);
          }
          tma_load_2d(st + TILE_A, &map_b, &S.full[s], kg * KG, n0);
          // the promotion's per-group constants: scales (and the planes' exponents)
          const int sl = g % NSIDE;
          if (!mbar_wait(&S.sempty[sl], ((uint32_t)(g / NSIDE) & 1) ^ 1, &g_q8_err, 10)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          uint8_t* sd = side + sl * SIDE_BYTES;
          S.sissued[sl] = g / NSIDE;
          mbar_expect_tx(&S.sfull[sl], PRESPLIT ? SIDE_BYTES : BN * 4);
          tma_load_2d(sd, &map_s, &S.sfull[sl], n0, kg);
          if (PRESPLIT) tma_load_2d(sd + BN * 4, &map_e, &S.sfull[sl], m0, kg);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % NST;
        const uint32_t r = (uint32_t)(g / NST);
        const int b = g & 1;
        const uint32_t u = (uint32_t)(g >> 1);
        const int ai = g % NACC;
        if (!ready(&S.full[s], r & 1, 2) || (!PRESPLIT && !ready(&S.afull[b], u & 1, 3)) ||
            (g >= NACC && !ready(&S.pempty[ai], (uint32_t)(g / NACC - 1) & 1, 4))) {
          ok = false;
          break;
        }
        fence_after();
        const uint64_t dah =
            desc_k_sw128(smem_u32(PRESPLIT ? smem + s * STAGE_BYTES : smem + PLANES_AT + b * 2 * PLANE));
        const uint64_t dal = dah + (PLANE >> 4);
        const uint64_t db = desc_k_sw128(smem_u32(smem + s * STAGE_BYTES + TILE_A));
        issue_group<!PRESPLIT>(tmem + ai * 128, dah, dal, db, &S.empty[s], &S.aempty[b], &S.pfull[ai]);
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.done);  // also on abort: arrives once whatever was issued has completed
  } else if (!PRESPLIT && warp < 6) {
    // ---- converters: thread = A row (idle with pre-split planes) ----
    const int row = (warp - 2) * 32 + lane;
    bool ok = !PRESPLIT;
    int g = 0;
    for (int tile = blockIdx.x; !PRESPLIT && ok && tile < ntiles; tile += gridDim.x) {
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % NST;
        const int b = g & 1;
        const uint32_t u = (uint32_t)(g >> 1);
        if (!ready(&S.full[s], (uint32_t)(g / NST) & 1, 5)) {
          ok = false;
          break;
        }
        // the row's 64 fp32 values: box h holds K 32h .. 32h + 31, 16-byte chunk j of a
        // 128-byte row at physical chunk j ^ (row % 8)
        float x[64];
        const uint8_t* st = smem + s * STAGE_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 v =
                *reinterpret_cast<const float4*>(st + h * (TILE_A / 2) + row * 128 + ((j ^ (row & 7)) << 4));
            x[32 * h + 4 * j] = v.x;
            x[32 * h + 4 * j + 1] = v.y;
            x[32 * h + 4 * j + 2] = v.z;
            x[32 * h + 4 * j + 3] = v.w;
          }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);  // this warp's rows of A are read
        float am = 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i) am = fmaxf(am, fabsf(x[i]));
        const int e = group_exponent(am);
        const float sc = pow2f(e);
        if (!ready(&S.aempty[b], (u & 1) ^ 1, 6)) {
          ok = false;
          break;
        }
        uint8_t* phi = smem + PLANES_AT + b * 2 * PLANE + row * 128;
        uint8_t* plo = phi + PLANE;
        // fp16 chunk j holds K 8j .. 8j + 7 (physical chunk j ^ (row % 8))
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = x[8 * j + 2 * q] * sc, a1 = x[8 * j + 2 * q + 1] * sc;  // exact: powers of two
            hw[q] = f2h2(a0, a1);
            float h0, h1;
            h22f(hw[q], h0, h1);
            lw[q] = f2h2(a0 - h0, a1 - h1);
          }
          const int pc = (j ^ (row & 7)) << 4;
          *reinterpret_cast<uint4*>(phi + pc) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(plo + pc) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        S.ex[g & 7][row] = e;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.afull[b]);
      }
    }
    if (!ok && !PRESPLIT) *abort_flag = 1;
  } else {
    // ---- promotion and epilogue: thread = output row (its TMEM lane), 64 columns ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int cbase = (warp - PW0) / 4 * EPI_COLS;
    const uint32_t lane_base = ((uint32_t)(quarter * 32) << 16) + (uint32_t)cbase;
    const bool vec = (ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(C) & 31) == 0);  // 32-byte rows pieces
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.f;
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % NST;
        const int ai = g % NACC;
        if (!ready(&S.pfull[ai], (uint32_t)(g / NACC) & 1, 7)) {
          ok = false;
          break;
        }
        fence_after();
        const int sl = g % NSIDE;
        if (!ready(&S.sfull[sl], (uint32_t)(g / NSIDE) & 1, 11)) {
          ok = false;
          break;
        }
        const uint8_t* sd = side + sl * SIDE_BYTES;
        const float f = pow2f(PRESPLIT ? -(int)reinterpret_cast<const int8_t*>(sd + BN * 4)[row] : -S.ex[g & 7][row]);
        const float* scl = reinterpret_cast<const float*>(sd) + cbase;  // the same for every lane
#pragma unroll
        for (int c0 = 0; c0 < EPI_COLS; c0 += 32) {
          float pv[32];
          tmem_ld32(tmem + lane_base + ai * 128 + c0, pv);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 sv = *reinterpret_cast<const float4*>(scl + c0 + 4 * q);
            acc[c0 + 4 * q] = fmaf(pv[4 * q] * f, sv.x, acc[c0 + 4 * q]);
            acc[c0 + 4 * q + 1] = fmaf(pv[4 * q + 1] * f, sv.y, acc[c0 + 4 * q + 1]);
            acc[c0 + 4 * q + 2] = fmaf(pv[4 * q + 2] * f, sv.z, acc[c0 + 4 * q + 2]);
            acc[c0 + 4 * q + 3] = fmaf(pv[4 * q + 3] * f, sv.w, acc[c0 + 4 * q + 3]);
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&S.pempty[ai]);
          mbar_arrive(&S.sempty[sl]);
        }
      }
      const int grow = m0 + row;
      if (PRESPLIT && ep.mode == 4) {
        // GELU-tanh, then the tile's columns as planes for the next GEMM: a 64-wide group
        // spans two 32-column threads of the same row, which exchange their maxima
        float am = 0.f;
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) {
          acc[j] = gelu_tanh(ep.bias ? __fadd_rn(acc[j], __ldg(ep.bias + n0 + cbase + j)) : acc[j]);
          am = fmaxf(am, fabsf(acc[j]));
        }
        const int cq = cbase / 32;
        S.xmax[cq][row] = am;
        // every promotion thread reaches this barrier each tile, also after a failed wait
        // (then it leaves with the others: the barrier also agrees on ok)
        uint32_t all_ok;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(all_ok)
            : "r"((uint32_t)ok), "n"(NPW * 32)
            : "memory");
        am = fmaxf(am, S.xmax[cq ^ 1][row]);
        asm volatile("bar.sync 1, %0;" ::"n"(NPW * 32) : "memory");
        ok = all_ok != 0;
        if (!ok) break;
        if (grow >= M) continue;
        const int e = cv3p::group_exponent(am);
        const float f = cv3p::pow2f(e);
        const int gg = (n0 + cbase) / KG, half = cq & 1;
        __half* ph = ep.oplanes + (int64_t)grow * (2 * N) + 2 * KG * gg + 32 * half;
        // 16 columns per 256-bit store (the planes rows are 32-byte aligned: N % 8 == 0)
#pragma unroll
        for (int q = 0; q < EPI_COLS / 16; ++q) {
          uint32_t h[8], l[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) cv3p::split_pair(acc[16 * q + 2 * t] * f, acc[16 * q + 2 * t + 1] * f, h[t], l[t]);
          st8(ph + 16 * q, h[0], h[1], h[2], h[3], h[4], h[5], h[6], h[7]);
          st8(ph + KG + 16 * q, l[0], l[1], l[2], l[3], l[4], l[5], l[6], l[7]);
        }
        if (half == 0) ep.oexps[(int64_t)gg * ep.olde + grow] = (int8_t)e;
        continue;
      }
      if (!ok) break;
      if (grow >= M) continue;
      float* crow = C + (int64_t)grow * ldc + n0 + cbase;
      const float* gate = ep.mode == 2 ? ep.gate + (ep.rows_per_group > 0 ? grow / ep.rows_per_group : 0) *
                                                     ep.gate_stride + n0 + cbase
                                       : nullptr;
      // chunks of 16 columns with every load (bias, gate, residual row) before the chunk's
      // stores: the residual is C itself
#pragma unroll
      for (int c0 = 0; c0 < EPI_COLS; c0 += 16) {
        float bv[16], gv[16], cv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bv[j] = ep.bias ? __ldg(ep.bias + n0 + cbase + c0 + j) : 0.f;
          gv[j] = ep.mode == 2 ? __ldg(gate + c0 + j) : 0.f;
          cv[j] = 0.f;
        }
        if (ep.mode >= 2) {
          if (vec) {
            ld8(crow + c0, cv);
            ld8(crow + c0 + 8, cv + 8);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) cv[j] = crow[c0 + j];
          }
        }
        float o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = acc[c0 + j];
          if (ep.bias) y = __fadd_rn(y, bv[j]);
          if (ep.mode == 1) y = gelu_tanh(y);
          else if (ep.mode == 2) y = __fadd_rn(cv[j], __fmul_rn(gv[j], y));
          else if (ep.mode == 3) y = __fadd_rn(cv[j], y);
          o[j] = y;
        }
        if (vec) {
#pragma unroll
          for (int q = 0; q < 2; ++q)
            st8(crow + c0 + 8 * q, __float_as_uint(o[8 * q]), __float_as_uint(o[8 * q + 1]), __float_as_uint(o[8 * q + 2]),
                __float_as_uint(o[8 * q + 3]), __float_as_uint(o[8 * q + 4]), __float_as_uint(o[8 * q + 5]),
                __float_as_uint(o[8 * q + 6]), __float_as_uint(o[8 * q + 7]));
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) crow[c0 + j] = o[j];
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      if (*abort_flag)
        for (int s = 0; s < NST; ++s)
          if (S.issued[s] >= 0) mbar_wait(&S.full[s], (uint32_t)S.issued[s] & 1, &g_q8_err, 8);
      if (*abort_flag)
        for (int i = 0; i < NSIDE; ++i)
          if (S.sissued[i] >= 0) mbar_wait(&S.sfull[i], (uint32_t)S.sissued[i] & 1, &g_q8_err, 12);
      mbar_wait(&S.done, 0, &g_q8_err, 9);  // every MMA (and its barrier arrivals) finished
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

int map_2d(CUtensorMap* map, CUtensorMapDataType type, int esize, const void* ptr, int64_t rows, int64_t cols,
           int64_t ld, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  CV3_REQUIRE(encode != nullptr, CV3_ERR_CUDA, "tc_gemm_q8: cuTensorMapEncodeTiled is unavailable");
  CV3_REQUIRE(((uintptr_t)ptr & 15) == 0, CV3_ERR_VALUE, "tc_gemm_q8: operand base must be 16-byte aligned");
  CV3_REQUIRE((ld * esize) % 16 == 0, CV3_ERR_VALUE, "tc_gemm_q8: row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, type, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CV3_REQUIRE(r == CUDA_SUCCESS, CV3_ERR_CUDA, "tc_gemm_q8: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CV3_OK;
}

// fp32 rows -> activation planes: one warp per row, two values per lane per group
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int64_t ldx, int64_t rows,
                                                         int k, __half* __restrict__ planes, int8_t* __restrict__ exps,
                                                         int64_t lde) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* xr = x + r * ldx;
  __half* pr = planes + r * (2 * (int64_t)k);
  for (int g = 0; g < k / KG; ++g) {
    const float2 v = *reinterpret_cast<const float2*>(xr + KG * g + 2 * lane);
    const float am = warp_max(fmaxf(fabsf(v.x), fabsf(v.y)));
    const int e = cv3p::group_exponent(am);
    const float f = cv3p::pow2f(e);
    uint32_t h, l;
    cv3p::split_pair(v.x * f, v.y * f, h, l);
    *reinterpret_cast<uint32_t*>(pr + 2 * KG * g + 2 * lane) = h;
    *reinterpret_cast<uint32_t*>(pr + 2 * KG * g + KG + 2 * lane) = l;
    if (lane == 0) exps[(int64_t)g * lde + r] = (int8_t)e;
  }
}

// q int8 [n][k] -> fp16 [n][k] (exact); scales fp16 [n][k/64] -> fp32 [k/64][n]
__global__ void q8_prepare_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ sc, int64_t n, int64_t k,
                                  __half* __restrict__ w16, float* __restrict__ st) {
  const int64_t total = n * k, ks = k / 64;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    w16[i] = __int2half_rn((int)q[i]);
    if (i < n * ks) {
      const int64_t r = i / ks, g = i - r * ks;
      st[g * n + r] = h2f(sc[i]);
    }
  }
}

}  // namespace

extern "C" int cv3_q8_gemm_prepare(const int8_t* q, const uint16_t* scales, int64_t n, int64_t k, void* w16,
                                   float* scales_t, void* stream) {
  CV3_REQUIRE(n > 0 && k > 0 && k % 64 == 0, CV3_ERR_VALUE, "q8_gemm_prepare: K must be a positive multiple of 64");
  int64_t grid = (n * k + 255) / 256;
  if (grid > cv3::sm_count() * 16) grid = cv3::sm_count() * 16;
  q8_prepare_kernel<<<(unsigned)grid, 256, 0, cv3::as_stream(stream)>>>(q, scales, n, k, static_cast<__half*>(w16),
                                                                         scales_t);
  return cv3::check_launch("q8_gemm_prepare");
}

namespace {

int launch_q8(bool presplit, const CUtensorMap& ma, const void* w16, const float* scales_t, const int8_t* pexp,
              int64_t lde, float* c, int64_t ldc, int64_t m, int64_t n, int64_t k, const Epi& ep, void* stream) {
  CUtensorMap mb, ms, me;
  int rc = map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w16, n, k, k, KG, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = map_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, scales_t, k / KG, n, n, BN, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (presplit) {
    rc = map_2d(&me, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, pexp, k / KG, lde, lde, BM, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    me = ms;  // (not read)
  }
  const void* fn = presplit ? (const void*)tc_gemm_q8_kernel<true> : (const void*)tc_gemm_q8_kernel<false>;
  rc = cv3::allow_smem(fn, SMEM_BYTES);
  if (rc) return rc;
  const int64_t ntiles = (n / BN) * ((m + BM - 1) / BM);
  CV3_REQUIRE(ntiles < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_q8: too many tiles");
  const int grid = (int)std::min<int64_t>(ntiles, cv3::sm_count());
  if (presplit)
    tc_gemm_q8_kernel<true><<<grid, Layout<true>::THREADS, SMEM_BYTES, cv3::as_stream(stream)>>>(
        ma, mb, ms, me, (int)m, (int)n, (int)k, c, ldc, ep);
  else
    tc_gemm_q8_kernel<false><<<grid, Layout<false>::THREADS, SMEM_BYTES, cv3::as_stream(stream)>>>(
        ma, mb, ms, me, (int)m, (int)n, (int)k, c, ldc, ep);
  return cv3::check_launch("tc_gemm_q8");
}

}  // namespace

extern "C" int cv3_tc_gemm_q8(const float* a, int64_t lda, const void* w16, const float* scales_t, float* c,
                              int64_t ldc, int64_t m, int64_t n, int64_t k, int mode, const float* bias,
                              const float* gate, int64_t rows_per_group, int64_t gate_stride, void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0 && mode >= 0 && mode <= 3, CV3_ERR_VALUE, "tc_gemm_q8: bad arguments");
  CV3_REQUIRE(mode != 2 || gate != nullptr, CV3_ERR_VALUE, "tc_gemm_q8: gated residual needs a gate");
  CV3_REQUIRE(n % BN == 0 && k % KG == 0, CV3_ERR_VALUE, "tc_gemm_q8: N a multiple of %d and K of %d", BN, KG);
  CV3_REQUIRE(lda >= k && ldc >= n && lda % 4 == 0, CV3_ERR_VALUE, "tc_gemm_q8: leading dimensions");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(k > 0 && m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_q8: sizes");
  CUtensorMap ma;
  int rc = map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a, m, k, lda, KG / 2, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Epi ep{mode, bias, gate, rows_per_group, gate_stride, nullptr, nullptr, 0};
  return launch_q8(false, ma, w16, scales_t, nullptr, 0, c, ldc, m, n, k, ep, stream);
}

extern "C" int cv3_tc_gemm_q8_planes(const void* planes, const int8_t* exps, int64_t lde, const void* w16,
                                     const float* scales_t, float* c, int64_t ldc, int64_t m, int64_t n, int64_t k,
                                     int mode, const float* bias, const float* gate, int64_t rows_per_group,
                                     int64_t gate_stride, void* out_planes, int8_t* out_exps, int64_t out_lde,
                                     void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0 && mode >= 0 && mode <= 4, CV3_ERR_VALUE, "tc_gemm_q8_planes: bad arguments");
  CV3_REQUIRE(mode != 2 || gate != nullptr, CV3_ERR_VALUE, "tc_gemm_q8_planes: gated residual needs a gate");
  CV3_REQUIRE(n % BN == 0 && k % KG == 0, CV3_ERR_VALUE, "tc_gemm_q8_planes: N a multiple of %d and K of %d", BN,
              KG);
  CV3_REQUIRE(lde >= m && lde % 16 == 0 && exps != nullptr, CV3_ERR_VALUE,
              "tc_gemm_q8_planes: exponents [k/64][lde], lde >= m and a multiple of 16");
  CV3_REQUIRE(mode == 4 ? (out_planes && out_exps && out_lde >= m && out_lde % 16 == 0 &&
                           ((uintptr_t)out_planes & 31) == 0)
                        : ldc >= n,
              CV3_ERR_VALUE,
              "tc_gemm_q8_planes: output (mode 4: 32-byte aligned planes [m][2n] and exponents [n/64][out_lde])");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(k > 0 && m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 30), CV3_ERR_VALUE, "tc_gemm_q8_planes: sizes");
  CUtensorMap ma;
  int rc = map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, planes, m, 2 * k, 2 * k, KG, BM,
                  CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Epi ep{mode, bias, gate, rows_per_group, gate_stride, static_cast<__half*>(out_planes), out_exps, out_lde};
  return launch_q8(true, ma, w16, scales_t, exps, lde, c, ldc, m, n, k, ep, stream);
}

extern "C" int cv3_q8_split_rows(const float* x, int64_t ldx, int64_t rows, int64_t k, void* planes, int8_t* exps,
                                 int64_t lde, void* stream) {
  CV3_REQUIRE(rows >= 0 && k > 0 && k % KG == 0 && ldx >= k && ldx % 2 == 0 && lde >= rows && lde % 16 == 0,
              CV3_ERR_VALUE, "q8_split_rows: K a multiple of 64, lde >= rows and a multiple of 16");
  CV3_REQUIRE(((uintptr_t)x & 7) == 0 && ((uintptr_t)planes & 3) == 0, CV3_ERR_VALUE, "q8_split_rows: alignment");
  if (rows == 0) return CV3_OK;
  split_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, cv3::as_stream(stream)>>>(
      x, ldx, rows, (int)k, static_cast<__half*>(planes), exps, lde);
  return cv3::check_launch("q8_split_rows");
}

extern "C" int cv3_tc_gemm_q8_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_q8_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_q8_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

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
// Persistent CTAs (one per SM) walk 128 x 128 output tiles; 14 warps:
//   warp 0     TMA: per K group the A fp32 tile (two 32-wide SWIZZLE_128B boxes) and the
//              q tile (fp16, converted once at load); a stage is free again once the
//              converters have read A and the MMAs B;
//   warp 1     MMA issuer: per group 4 k-steps x (hi, lo) into the group's accumulator
//              (four in TMEM: the MMAs run up to three groups ahead of the promotion);
//   warps 2-5  converters: thread = A row: the row's 64 values, their exponent, the
//              hi / lo fp16 planes in the UMMA K-major SWIZZLE_128B layout;
//   warps 6-13 promotion and epilogue, two per TMEM lane quarter (64 columns each):
//              fold each group into fp32 registers, then bias / GELU-tanh / gated
//              residual and the stores while the MMA warp starts the next tile.
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel records an error
// (cv3_tc_gemm_q8_status), stops issuing work, lets what it issued finish and exits.
#include <algorithm>

#include "tc_common.cuh"

namespace {

using namespace cv3tc;

constexpr int BM = 128, BN = 128, KG = 64;  // KG: one scale group
constexpr int STAGES = 3;
constexpr int TILE_A = BM * KG * 4;                  // 32 KB: two 32-wide fp32 boxes
constexpr int TILE_B = BN * KG * 2;                  // 16 KB: fp16 weights
constexpr int STAGE_BYTES = TILE_A + TILE_B;        // A | B (1 KB multiples: SW128 tiles)
constexpr int PLANES_AT = STAGES * STAGE_BYTES;      // 2 buffers x (hi | lo), 16 KB each
constexpr int PLANE = BM * KG * 2;                   // 16 KB
constexpr int THREADS = 448;
constexpr int EPI_COLS = 64;
constexpr int NACC = 4;  // TMEM accumulators (one per K group in flight), 128 columns each
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);  // f16 x f16 -> f32

__device__ int g_q8_err = 0;

struct Bars {
  uint64_t full[STAGES], empty[STAGES], afull[2], aempty[2], pfull[NACC], pempty[NACC], done;
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES];
  // per (group mod 8, row): the power of two the converters scaled by.  Depth: converter
  // g waits for MMA g-2, which waits for the promotion of g-2-NACC, so the slot of
  // group g is rewritten only after its promotion when the depth is >= NACC + 2
  int ex[8][BM];
};
constexpr int SMEM_BYTES = PLANES_AT + 4 * PLANE + 1024 + (int)sizeof(Bars);

struct Epi {
  int mode;  // 0: +bias; 1: gelu_tanh(+bias); 2: h += gate * (+bias); 3: h += (+bias)
  const float* bias;
  const float* gate;
  int64_t rows_per_group, gate_stride;
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

// One K group's MMAs: 4 k-steps of 16, A hi and A lo into the group's accumulator d,
// the weights from one descriptor; then the commits that free the stage, the A planes
// and hand the accumulator to the promotion.
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
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%8];\n\t}" ::"r"(d),
      "l"(ahi), "l"(alo), "l"(b), "r"(IDESC), "r"(0), "r"(smem_u32(bar_stage)), "r"(smem_u32(bar_planes)),
      "r"(smem_u32(bar_acc))
      : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_q8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const float* __restrict__ scales_t, int M, int N, int K, float* __restrict__ C, int64_t ldc,
                  Epi ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& S = *reinterpret_cast<Bars*>(smem + PLANES_AT + 4 * PLANE);
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = K / KG;
  const int tiles_n = N / BN;
  const int ntiles = tiles_n * ((M + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1 + 4);  // MMA commit (B), four converter warps (A)
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.afull[i], 4);
      mbar_init(&S.aempty[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&S.pfull[i], 1);
      mbar_init(&S.pempty[i], 8);
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
          const int s = g % STAGES;
          const uint32_t r = (uint32_t)(g / STAGES);
          if (*abort_flag || !mbar_wait(&S.empty[s], (r & 1) ^ 1, &g_q8_err, 1)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          S.issued[s] = (int)r;
          mbar_expect_tx(&S.full[s], TILE_A + TILE_B);
          tma_load_2d(st, &map_a, &S.full[s], kg * KG, m0);
          tma_load_2d(st + TILE_A / 2, &map_a, &S.full[s], kg * KG + KG / 2, m0);
          tma_load_2d(st + TILE_A, &map_b, &S.full[s], kg * KG, n0);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % STAGES;
        const uint32_t r = (uint32_t)(g / STAGES);
        const int b = g & 1;
        const uint32_t u = (uint32_t)(g >> 1);
        const int ai = g % NACC;
        if (!ready(&S.full[s], r & 1, 2) || !ready(&S.afull[b], u & 1, 3) ||
            (g >= NACC && !ready(&S.pempty[ai], (uint32_t)(g / NACC - 1) & 1, 4))) {
          ok = false;
          break;
        }
        fence_after();
        const uint64_t dah = desc_k_sw128(smem_u32(smem + PLANES_AT + b * 2 * PLANE));
        const uint64_t dal = dah + (PLANE >> 4);
        const uint64_t db = desc_k_sw128(smem_u32(smem + s * STAGE_BYTES + TILE_A));
        issue_group(tmem + ai * 128, dah, dal, db, &S.empty[s], &S.aempty[b], &S.pfull[ai]);
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.done);  // also on abort: arrives once whatever was issued has completed
  } else if (warp < 6) {
    // ---- converters: thread = A row ----
    const int row = (warp - 2) * 32 + lane;
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % STAGES;
        const int b = g & 1;
        const uint32_t u = (uint32_t)(g >> 1);
        if (!ready(&S.full[s], (uint32_t)(g / STAGES) & 1, 5)) {
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
    if (!ok) *abort_flag = 1;
  } else {
    // ---- promotion and epilogue: thread = output row (its TMEM lane), 64 columns ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int cbase = (warp - 6) / 4 * EPI_COLS;
    const uint32_t lane_base = ((uint32_t)(quarter * 32) << 16) + (uint32_t)cbase;
    const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
      float acc[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) acc[j] = 0.f;
      for (int kg = 0; kg < ng; ++kg, ++g) {
        const int s = g % STAGES;
        const int ai = g % NACC;
        if (!ready(&S.pfull[ai], (uint32_t)(g / NACC) & 1, 7)) {
          ok = false;
          break;
        }
        fence_after();
        const float f = pow2f(-S.ex[g & 7][row]);
        // the group's scales of this warp's columns: the same for every lane (L1 broadcast)
        const float* scl = scales_t + (int64_t)kg * N + n0 + cbase;
#pragma unroll
        for (int c0 = 0; c0 < EPI_COLS; c0 += 32) {
          float pv[32];
          tmem_ld32(tmem + lane_base + ai * 128 + c0, pv);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 sv = __ldg(reinterpret_cast<const float4*>(scl + c0 + 4 * q));
            acc[c0 + 4 * q] = fmaf(pv[4 * q] * f, sv.x, acc[c0 + 4 * q]);
            acc[c0 + 4 * q + 1] = fmaf(pv[4 * q + 1] * f, sv.y, acc[c0 + 4 * q + 1]);
            acc[c0 + 4 * q + 2] = fmaf(pv[4 * q + 2] * f, sv.z, acc[c0 + 4 * q + 2]);
            acc[c0 + 4 * q + 3] = fmaf(pv[4 * q + 3] * f, sv.w, acc[c0 + 4 * q + 3]);
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.pempty[ai]);
      }
      if (!ok) break;
      const int grow = m0 + row;
      if (grow >= M) continue;
      float* crow = C + (int64_t)grow * ldc + n0 + cbase;
      const float* gate = ep.mode == 2 ? ep.gate + (ep.rows_per_group > 0 ? grow / ep.rows_per_group : 0) *
                                                     ep.gate_stride + n0 + cbase
                                       : nullptr;
      // chunks of 16 columns with every load (bias, gate, residual row) before the chunk's
      // stores: the residual is C itself
#pragma unroll
      for (int c0 = 0; c0 < EPI_COLS; c0 += 16) {
        float bv[16], gv[16], rv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          bv[j] = ep.bias ? __ldg(ep.bias + n0 + cbase + c0 + j) : 0.f;
          gv[j] = ep.mode == 2 ? __ldg(gate + c0 + j) : 0.f;
          rv[j] = 0.f;
        }
        if (ep.mode >= 2) {
          if (vec) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 t = *reinterpret_cast<const float4*>(crow + c0 + 4 * q);
              rv[4 * q] = t.x;
              rv[4 * q + 1] = t.y;
              rv[4 * q + 2] = t.z;
              rv[4 * q + 3] = t.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) rv[j] = crow[c0 + j];
          }
        }
        float o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = acc[c0 + j];
          if (ep.bias) y = __fadd_rn(y, bv[j]);
          if (ep.mode == 1) y = gelu_tanh(y);
          else if (ep.mode == 2) y = __fadd_rn(rv[j], __fmul_rn(gv[j], y));
          else if (ep.mode == 3) y = __fadd_rn(rv[j], y);
          o[j] = y;
        }
        if (vec) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4*>(crow + c0 + 4 * q) = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
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
        for (int s = 0; s < STAGES; ++s)
          if (S.issued[s] >= 0) mbar_wait(&S.full[s], (uint32_t)S.issued[s] & 1, &g_q8_err, 8);
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

extern "C" int cv3_tc_gemm_q8(const float* a, int64_t lda, const void* w16, const float* scales_t, float* c,
                              int64_t ldc, int64_t m, int64_t n, int64_t k, int mode, const float* bias,
                              const float* gate, int64_t rows_per_group, int64_t gate_stride, void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0 && mode >= 0 && mode <= 3, CV3_ERR_VALUE, "tc_gemm_q8: bad arguments");
  CV3_REQUIRE(mode != 2 || gate != nullptr, CV3_ERR_VALUE, "tc_gemm_q8: gated residual needs a gate");
  CV3_REQUIRE(n % BN == 0 && k % KG == 0, CV3_ERR_VALUE, "tc_gemm_q8: N a multiple of %d and K of %d", BN, KG);
  CV3_REQUIRE(lda >= k && ldc >= n && lda % 4 == 0, CV3_ERR_VALUE, "tc_gemm_q8: leading dimensions");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(k > 0 && m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_q8: sizes");
  CUtensorMap ma, mb;
  int rc = map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a, m, k, lda, KG / 2, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w16, n, k, k, KG, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  CV3_REQUIRE(((uintptr_t)scales_t & 15) == 0, CV3_ERR_VALUE, "tc_gemm_q8: 16-byte aligned scales");
  rc = cv3::allow_smem((const void*)tc_gemm_q8_kernel, SMEM_BYTES);
  if (rc) return rc;
  const int64_t ntiles = (n / BN) * ((m + BM - 1) / BM);
  CV3_REQUIRE(ntiles < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_q8: too many tiles");
  const int grid = (int)std::min<int64_t>(ntiles, cv3::sm_count());
  Epi ep{mode, bias, gate, rows_per_group, gate_stride};
  tc_gemm_q8_kernel<<<grid, THREADS, SMEM_BYTES, cv3::as_stream(stream)>>>(ma, mb, scales_t, (int)m, (int)n, (int)k,
                                                                          c, ldc, ep);
  return cv3::check_launch("tc_gemm_q8");
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

// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   C[M][N] = epilogue(A[M][K] . B[N][K]^T)      A, B, C fp32, row-major, K-major operands
//
// Precision: 3xTF32.  Each operand element x is split into hi = x with its low
// 13 mantissa bits cleared (exactly a tf32 value) and lo = x - hi (exact in
// fp32, <= 13 significant bits), and the product is accumulated in fp32 in
// TMEM as hi*hi + hi*lo + lo*hi; the dropped lo*lo term and the truncation of
// lo to tf32 leave ~2^-21 relative error per product, fp32-SGEMM territory.
// This is how the DiT's fp32 linears (cv3cpu/ops.py:121 -> BLAS sgemm) run on
// tensor cores without leaving the reference's 1e-5 tolerance.
//
// CTA = 6 warps, one 128x128 output tile, K in 32-element (128 B) blocks:
//   warp 0   TMA producer: A and B tiles (SWIZZLE_128B) into a 3-stage ring;
//   warp 1   MMA issuer (one thread): 4 K-steps x 3 tcgen05.mma kind::tf32 per
//            stage, tcgen05.commit frees the stage / signals the accumulator;
//   warps 2-5 split each landed stage in place (hi) and into the lo buffers,
//            then run the epilogue: tcgen05.ld 32 lanes x 32 columns at a
//            time, bias / GELU-tanh / gated residual, fp32 stores.
// The split buffers share the TMA tile's swizzled layout element for element,
// so the converters never need to know the swizzle.
//
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel records
// an error code (read with cv3_tc_gemm_status), skips its remaining work, waits
// (bounded) for its own MMAs, frees TMEM and exits.
#include <algorithm>

#include "tc_common.cuh"

namespace {

using namespace cv3tc;

constexpr int BM = 128, BN = 128, BK = 32;  // BK fp32 = 128 bytes = one swizzle row
constexpr int STAGES = 3;
constexpr int TILE_A = BM * BK * 4;  // 16 KB
constexpr int TILE_B = BN * BK * 4;  // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_B;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;  // up to 4 accumulators of BN fp32 columns

__device__ int g_tc_err = 0;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  return cv3tc::mbar_wait(bar, parity, &g_tc_err, code);
}

// kind::tf32 instruction descriptor: D f32, A/B tf32, K-major, M = 128, N = BN.
constexpr uint32_t IDESC = idesc_tf32(BM, BN);

__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) { return desc_k_sw128(addr); }

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  mma_ss(d_tmem, a, b, IDESC, accumulate);
}

struct Epi {
  int k_chunks;          // 1, 2 or 4 accumulators, each summing a contiguous K range
  int split_cross;       // 1: hi*lo + lo*hi accumulate apart from hi*hi (k_chunks <= 2)
  int mode;              // 0: +bias; 1: gelu_tanh(+bias); 2: h += gate * (+bias); 3: h += (+bias)
  const float* bias;     // [N] or null
  const float* gate;     // mode 2: gate + (row / rows_per_group) * gate_stride
  int64_t rows_per_group, gate_stride;
};

__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  const float inner = x + 0.044715f * x * x * x;
  return 0.5f * x * (1.0f + tanhf(c * inner));
}

__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int N,
               int K, float* __restrict__ C, int64_t ldc, Epi ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* accb = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued = abort_flag + 1;  // [STAGES]: last round loaded into each stage, -1 if none

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);  // one arrival per converter warp
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) issued[s] = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        if (*(volatile int*)abort_flag || !mbar_wait(&empty[s], (round & 1) ^ 1, 1)) {
          *(volatile int*)abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        issued[s] = (int)round;
        mbar_expect_tx(&full[s], TILE_A + TILE_B);
        tma_load_2d(st, &map_a, &full[s], kb * BK, m0);
        tma_load_2d(st + 2 * TILE_A, &map_b, &full[s], kb * BK, n0);
      }
    }
  } else if (warp == 1) {
    // the whole warp runs the MMA loop (operands warp-uniform), one elected lane issues
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      const uint32_t round = kb / STAGES;
      bool go = !*(volatile int*)abort_flag && mbar_wait(&conv[s], round & 1, 2);
      if (!__all_sync(0xffffffffu, go)) {
        if (lane == 0) *(volatile int*)abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a_hi = smem_u32(smem + s * STAGE_BYTES);
      const uint32_t a_lo = a_hi + TILE_A;
      const uint32_t b_hi = a_hi + 2 * TILE_A;
      const uint32_t b_lo = b_hi + TILE_B;
      // accumulator of this K block: K range chunk, cross terms optionally apart
      const int chunk = kb * ep.k_chunks / nk;
      const int first_kb = (chunk * nk + ep.k_chunks - 1) / ep.k_chunks;  // first kb of this chunk
      const uint32_t d_main = tmem + (uint32_t)(chunk * BN);
      const uint32_t d_cross = ep.split_cross ? tmem + (uint32_t)((ep.k_chunks + chunk) * BN) : d_main;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along the swizzled row
        const bool start = (kb == first_kb && kk == 0);
        mma_tf32(d_cross, umma_desc(a_lo + off), umma_desc(b_hi + off), start ? 0u : 1u);
        mma_tf32(d_cross, umma_desc(a_hi + off), umma_desc(b_lo + off), 1u);
        mma_tf32(d_main, umma_desc(a_hi + off), umma_desc(b_hi + off), (start && ep.split_cross) ? 0u : 1u);
      }
      mma_commit(&empty[s]);
    }
    // the accumulator barrier is committed even on abort so waiters are released
    // once whatever was issued has completed
    mma_commit(accb);
  } else {
    // converters, then the epilogue
    const int ctid = threadIdx.x - 64;  // 0..127
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      const uint32_t round = kb / STAGES;
      bool go = !*(volatile int*)abort_flag && mbar_wait(&full[s], round & 1, 3);
      go = __all_sync(0xffffffffu, go);  // warp-uniform, the loop body syncs the warp
      if (!go) {
        *(volatile int*)abort_flag = 1;
        break;
      }
      float* st = reinterpret_cast<float*>(smem + s * STAGE_BYTES);
      split_tile(st, st + TILE_A / 4, TILE_A, ctid, 128);
      split_tile(st + 2 * TILE_A / 4, st + (2 * TILE_A + TILE_B) / 4, TILE_B, ctid, 128);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
    bool ok = mbar_wait(accb, 0, 4) && !*(volatile int*)abort_flag;
    ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      const int quarter = warp & 3;  // TMEM lanes this warp may read
      const int row = m0 + quarter * 32 + lane;
      const int nacc = ep.k_chunks * (ep.split_cross ? 2 : 1);
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        // small (cross-term) accumulators first, then the main ones, in fp32
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((nacc - 1) * BN + c0), v);
        for (int a = nacc - 2; a >= 0; --a) {
          float w[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * BN + c0), w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += w[j];
        }
        if (row < M) {
          float* crow = C + (int64_t)row * ldc + n0 + c0;
          const float* gate = ep.mode == 2 ? ep.gate + (ep.rows_per_group > 0 ? row / ep.rows_per_group : 0) *
                                                           ep.gate_stride + n0 + c0
                                           : nullptr;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = n0 + c0 + j;
            if (col < N) {
              float y = v[j];
              if (ep.bias) y = __fadd_rn(y, ep.bias[col]);
              if (ep.mode == 1) {
                y = gelu_tanh(y);
              } else if (ep.mode == 2) {
                y = __fadd_rn(crow[j], __fmul_rn(gate[j], y));
              } else if (ep.mode == 3) {
                y = __fadd_rn(crow[j], y);
              }
              crow[j] = y;
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    if (*(volatile int*)abort_flag) {
      // on abort: let every issued TMA copy land and every issued MMA finish
      // (bounded) before the shared memory and the accumulator are released
      if (lane == 0)
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] >= 0) mbar_wait(&full[s], (uint32_t)issued[s] & 1, 6);
      mbar_wait(accb, 0, 5);
    }
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

int make_map(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  CV3_REQUIRE(encode != nullptr, CV3_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled is unavailable");
  CV3_REQUIRE(((uintptr_t)ptr & 15) == 0, CV3_ERR_VALUE, "tc_gemm: operand base must be 16-byte aligned");
  CV3_REQUIRE((ld * 4) % 16 == 0, CV3_ERR_VALUE, "tc_gemm: row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)ptr, dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CV3_REQUIRE(r == CUDA_SUCCESS, CV3_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CV3_OK;
}


// ---------------------------------------------------------------------------
// Pre-split variant (the DiT's linears).  B comes with its tf32 remainder
// b_lo = b - tf32(b) (made once per weight matrix by cv3_tf32_lo); the raw B
// is the hi operand, since kind::tf32 reads only the top 19 bits of each
// fp32.  A, B and B lo arrive by TMA in one 4-stage ring; the four converter
// warps read their A row (one row per thread = its TMEM lane) from the
// swizzled stage, split it and write hi/lo into TMEM, and the MMAs take A
// from TMEM, so shared memory carries A once each way and B to the tensor
// core.  A stage is free again when its A has been read (converters) and its
// B consumed (MMA commit).
// TMEM: two K-range accumulators for hi*hi, one for the cross terms (the
// tensor core truncates when it accumulates, so long sums lose bits; this
// layout measured 1.7e-6 / 2.9e-6 of max at K = 1024 / 2048 vs fp64) and two
// A stages of 32 hi + 32 lo columns.
// ---------------------------------------------------------------------------
namespace split {

// Pre-split GEMM: B comes with its tf32 remainder (cv3_tf32_lo, once per weight);
// A's remainder is made on the fly.  The tensor core truncates its fp32 inputs to
// tf32, so the raw TMA tiles serve as the hi operands.  (Splitting B on the fly
// too halves the TMA bytes of B but doubles the converters' work per K block;
// measured 8% slower.)
//
// MMA cost model (measured on B200, M = 128, K = 8 tf32 per instruction): an
// MMA into an accumulator that the previous one also wrote waits ~130 cycles;
// independent accumulators interleaved round-robin bring it to ~77 cycles with
// four of them, for N = 64 and 128 alike.  So the twelve MMAs of a K block go to
// four accumulators in turn: hi*hi of even K blocks, hi*hi of odd K blocks, lo*hi,
// hi*lo.  Splitting hi*hi over two accumulators also halves the sum each one
// holds, which bounds the tensor core's truncating adds (the reason the split was
// introduced; the epilogue adds the four in fp32).  All four live in TMEM (512
// columns), so A's remainder goes to shared memory and every MMA is the SS form.
//
// Persistent CTAs (one per SM) walk 128 x 128 output tiles; 14 warps:
//   warp 0     TMA: A, B, B lo tiles into a 4-stage ring, tile after tile;
//   warp 1     MMA issuer (converged warp, one elected thread, one asm block per
//              K block);
//   warps 2-5  converters: A lo = A - tf32(A) of each landed stage into a
//              2-buffer ring in the same swizzled layout;
//   warps 6-13 epilogue, two per TMEM lane quarter (64 columns each): as soon
//              as a tile's MMAs finish, fold its four accumulators into fp32
//              registers and hand TMEM back, then run bias / GELU / gated
//              residual and the stores while the MMA warp already works on the
//              next tile.
constexpr int BM = 128, BN = 128, BK = 32, STAGES = 4;
constexpr int TILE_A = BM * BK * 4;               // 16 KB
constexpr int TILE_B = BN * BK * 4;               // 16 KB
constexpr int STAGE_BYTES = TILE_A + 2 * TILE_B;  // A | B | B lo
constexpr int LO_AT = STAGES * STAGE_BYTES;       // A lo ring (2 x 16 KB)
constexpr int LO_BYTES = TILE_A;
constexpr int THREADS = 448;
constexpr int EPI_COLS = 64;  // columns per epilogue warp
constexpr uint32_t C_MAIN0 = 0, C_MAIN1 = 128, C_CROSS_A = 256, C_CROSS_B = 384;
constexpr uint32_t IDESC = idesc_tf32(BM, BN);

struct Bars {
  uint64_t full[STAGES], empty[STAGES], lofull[2], loempty[2], accfull, accempty, done;
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES];
};
constexpr int SMEM_BYTES = LO_AT + 2 * LO_BYTES + 1024 + (int)sizeof(Bars);

// One K block: k-steps kk = 0..3 (descriptor start + 2 kk), main (hi*hi) into m,
// then lo*hi and hi*lo into the two remainder accumulators, round-robin; then the
// commits that free the stage and the A lo buffer.  fm / fx: first use of the main
// / the remainder accumulators (they start from zero).
__device__ __forceinline__ void issue_kblock(uint32_t m, uint32_t xa, uint32_t xb, uint64_t a, uint64_t alo, uint64_t b,
                                             uint64_t blo, uint32_t fm, uint32_t fx, uint64_t* bar_stage,
                                             uint64_t* bar_lo) {
  asm volatile(
      "{\n\t.reg .pred e, pt, pm, px;\n\t"
      ".reg .b64 a1, a2, a3, l1, l2, l3, b1, b2, b3, c1, c2, c3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.eq.b32 pt, %7, %7;\n\tsetp.eq.b32 pm, %7, 0;\n\tsetp.eq.b32 px, %8, 0;\n\t"
      "add.s64 a1, %3, 2;\n\tadd.s64 a2, %3, 4;\n\tadd.s64 a3, %3, 6;\n\t"
      "add.s64 l1, %4, 2;\n\tadd.s64 l2, %4, 4;\n\tadd.s64 l3, %4, 6;\n\t"
      "add.s64 b1, %5, 2;\n\tadd.s64 b2, %5, 4;\n\tadd.s64 b3, %5, 6;\n\t"
      "add.s64 c1, %6, 2;\n\tadd.s64 c2, %6, 4;\n\tadd.s64 c3, %6, 6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %3, %5, %9, pm;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], %4, %5, %9, px;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%2], %3, %6, %9, px;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], a1, b1, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l1, b1, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%2], a1, c1, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], a2, b2, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l2, b2, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%2], a2, c2, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], a3, b3, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l3, b3, %9, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%2], a3, c3, %9, pt;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%10];\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%11];\n\t}" ::"r"(m),
      "r"(xa), "r"(xb), "l"(a), "l"(alo), "l"(b), "l"(blo), "r"(fm), "r"(fx), "r"(IDESC), "r"(smem_u32(bar_stage)),
      "r"(smem_u32(bar_lo))
      : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_split_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_blo, int M, int N, int K, float* __restrict__ C,
                     int64_t ldc, Epi ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& S = *reinterpret_cast<Bars*>(smem + LO_AT + 2 * LO_BYTES);
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (K + BK - 1) / BK;
  const int tiles_n = (N + BN - 1) / BN;
  const int ntiles = tiles_n * ((M + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 5);  // MMA commit + four converter warps
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.lofull[i], 4);
      mbar_init(&S.loempty[i], 1);
    }
    mbar_init(&S.accfull, 1);
    mbar_init(&S.accempty, 8);
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
    const bool ok = !*abort_flag && mbar_wait(bar, parity, code);
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // K blocks loaded so far (all tiles)
      bool go = true;
      for (int tile = blockIdx.x; go && tile < ntiles; tile += gridDim.x) {
        const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t r = (uint32_t)(g / STAGES);
          if (*abort_flag || !mbar_wait(&S.empty[s], (r & 1) ^ 1, 21)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          S.issued[s] = (int)r;
          mbar_expect_tx(&S.full[s], STAGE_BYTES);
          tma_load_2d(st, &map_a, &S.full[s], kb * BK, m0);
          tma_load_2d(st + TILE_A, &map_b, &S.full[s], kb * BK, n0);
          tma_load_2d(st + TILE_A + TILE_B, &map_blo, &S.full[s], kb * BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    bool ok = true;
    int g = 0, it = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      // the accumulators are free once the epilogue has folded the previous tile
      if (it >= 1 && !ready(&S.accempty, (uint32_t)(it - 1) & 1, 29)) {
        ok = false;
        break;
      }
      fence_after();
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int s = g % STAGES;
        const uint32_t r = (uint32_t)(g / STAGES);
        const int l = g & 1;
        if (!ready(&S.full[s], r & 1, 22) || !ready(&S.lofull[l], (uint32_t)(g >> 1) & 1, 23)) {
          ok = false;
          break;
        }
        fence_after();
        const uint64_t d_a = desc_k_sw128(smem_u32(smem + s * STAGE_BYTES));
        const uint64_t d_b = d_a + (TILE_A >> 4), d_blo = d_b + (TILE_B >> 4);
        const uint64_t d_alo = desc_k_sw128(smem_u32(smem + LO_AT + l * LO_BYTES));
        issue_kblock(tmem + ((kb & 1) ? C_MAIN1 : C_MAIN0), tmem + C_CROSS_A, tmem + C_CROSS_B, d_a, d_alo, d_b,
                     d_blo, kb < 2 ? 1u : 0u, kb == 0 ? 1u : 0u, &S.empty[s], &S.loempty[l]);
      }
      if (ok) mma_commit(&S.accfull);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.done);  // also on abort: arrives once whatever was issued has completed
  } else if (warp < 6) {
    // ---- converters: A lo of each stage.  Elementwise, so each 16-byte chunk goes to the
    // same physical place in the lo tile as in the A tile (no need to know the swizzle);
    // lanes visit the chunks in the order j ^ (row % 8) so a quarter-warp's eight rows hit
    // eight bank groups ----
    const int row = (warp & 3) * 32 + lane;
    bool ok = true;
    int g = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int s = g % STAGES;
        const int l = g & 1;
        if (!ready(&S.full[s], (uint32_t)(g / STAGES) & 1, 24)) {
          ok = false;
          break;
        }
        const uint8_t* arow = smem + s * STAGE_BYTES + row * 128;
        float4 lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 x = *reinterpret_cast<const float4*>(arow + ((j ^ (row & 7)) << 4));
          lo[j] = make_float4(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y), x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);  // this warp's rows of the stage are read
        if (!ready(&S.loempty[l], ((uint32_t)(g >> 1) & 1) ^ 1, 25)) {
          ok = false;
          break;
        }
        uint8_t* lrow = smem + LO_AT + l * LO_BYTES + row * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<float4*>(lrow + ((j ^ (row & 7)) << 4)) = lo[j];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.lofull[l]);
      }
    }
    if (!ok) *abort_flag = 1;
  } else {
    // ---- epilogue: thread = output row (its TMEM lane), columns [cbase, cbase + 64) ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int cbase = (warp - 6) / 4 * EPI_COLS;
    const uint32_t lane_base = ((uint32_t)(quarter * 32) << 16) + (uint32_t)cbase;
    const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int n0 = (tile % tiles_n) * BN, m0 = (tile / tiles_n) * BM;
      if (!ready(&S.accfull, (uint32_t)it & 1, 26)) {
        ok = false;
        break;
      }
      fence_after();
      // fold (lo*hi + hi*lo) + hi*hi(odd K blocks) + hi*hi(even K blocks) in fp32
      float v[EPI_COLS];
#pragma unroll
      for (int c0 = 0; c0 < EPI_COLS; c0 += 32) {
        float w[32];
        tmem_ld32(tmem + lane_base + C_CROSS_A + c0, v + c0);
        tmem_ld32(tmem + lane_base + C_CROSS_B + c0, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[c0 + j] += w[j];
        if (nk >= 2) {
          tmem_ld32(tmem + lane_base + C_MAIN1 + c0, w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[c0 + j] += w[j];
        }
        tmem_ld32(tmem + lane_base + C_MAIN0 + c0, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[c0 + j] += w[j];
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.accempty);
      const int grow = m0 + row;
      if (grow >= M) continue;
      float* crow = C + (int64_t)grow * ldc + n0 + cbase;
      const float* gate = ep.mode == 2 ? ep.gate + (ep.rows_per_group > 0 ? grow / ep.rows_per_group : 0) *
                                                     ep.gate_stride + n0 + cbase
                                       : nullptr;
      const int ncol = min(EPI_COLS, N - n0 - cbase);
      if (ncol <= 0) continue;
      const bool full = vec && ncol == EPI_COLS;
      // chunks of 16 columns with every load (bias, gate, residual row) before the chunk's
      // stores: the residual is C itself, so loads after a store could not be hoisted
#pragma unroll
      for (int c0 = 0; c0 < EPI_COLS; c0 += 16) {
        float bv[16], gv[16], rv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool in = c0 + j < ncol;
          bv[j] = (ep.bias && in) ? __ldg(ep.bias + n0 + cbase + c0 + j) : 0.f;
          gv[j] = (ep.mode == 2 && in) ? __ldg(gate + c0 + j) : 0.f;
          rv[j] = 0.f;
        }
        if (ep.mode >= 2) {
          if (full) {
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
            for (int j = 0; j < 16; ++j) rv[j] = c0 + j < ncol ? crow[c0 + j] : 0.f;
          }
        }
        float o[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y = v[c0 + j];
          if (ep.bias) y = __fadd_rn(y, bv[j]);
          if (ep.mode == 1) y = gelu_tanh(y);
          else if (ep.mode == 2) y = __fadd_rn(rv[j], __fmul_rn(gv[j], y));
          else if (ep.mode == 3) y = __fadd_rn(rv[j], y);
          o[j] = y;
        }
        if (full) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4*>(crow + c0 + 4 * q) = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < ncol) crow[c0 + j] = o[j];
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
          if (S.issued[s] >= 0) mbar_wait(&S.full[s], (uint32_t)S.issued[s] & 1, 27);
      mbar_wait(&S.done, 0, 28);  // every MMA (and its barrier arrivals) finished
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

__global__ void tf32_lo_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ lo) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    lo[i] = v - tf32_hi(v);
  }
}

}  // namespace split

}  // namespace

// cv3_tc_gemm with an explicit accumulator layout: k_chunks (1, 2, 4) TMEM
// accumulators each sum a contiguous K range; split_cross = 1 keeps the hi*lo +
// lo*hi terms in their own accumulators (at most 4 in all).
static int tc_gemm_layout(const float* a, int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc,
                               int64_t m, int64_t n, int64_t k, int mode, const float* bias, const float* gate,
                               int64_t rows_per_group, int64_t gate_stride, int k_chunks, int split_cross,
                               void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0 && mode >= 0 && mode <= 3, CV3_ERR_VALUE, "tc_gemm: bad arguments");
  CV3_REQUIRE((k_chunks == 1 || k_chunks == 2 || k_chunks == 4) && (split_cross == 0 || split_cross == 1) &&
                  k_chunks * (split_cross + 1) <= 4,
              CV3_ERR_VALUE, "tc_gemm: accumulator layout needs k_chunks in {1,2,4} and at most 4 accumulators");
  CV3_REQUIRE(mode != 2 || gate != nullptr, CV3_ERR_VALUE, "tc_gemm: gated residual needs a gate");
  CV3_REQUIRE(lda >= k && ldb >= k && ldc >= n, CV3_ERR_VALUE, "tc_gemm: leading dimension too small");
  CV3_REQUIRE(k % 4 == 0, CV3_ERR_VALUE, "tc_gemm: K must be a multiple of 4 (16-byte rows)");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(k > 0, CV3_ERR_VALUE, "tc_gemm: K must be positive");
  CV3_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CV3_ERR_VALUE, "tc_gemm: too large");
  CUtensorMap ma, mb;
  int rc = make_map(&ma, a, m, k, lda, BM);
  if (rc) return rc;
  rc = make_map(&mb, b, n, k, ldb, BN);
  if (rc) return rc;
  rc = cv3::allow_smem((const void*)tc_gemm_kernel, SMEM_BYTES);
  if (rc) return rc;
  dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
  CV3_REQUIRE(grid.y <= 65535, CV3_ERR_VALUE, "tc_gemm: too many row tiles");
  const int nk = (int)((k + BK - 1) / BK);
  if (k_chunks > nk) k_chunks = nk >= 4 ? 4 : (nk >= 2 ? 2 : 1);
  Epi ep{k_chunks, split_cross, mode, bias, gate, rows_per_group, gate_stride};
  tc_gemm_kernel<<<grid, THREADS, SMEM_BYTES, cv3::as_stream(stream)>>>(ma, mb, (int)m, (int)n, (int)k, c, ldc, ep);
  return cv3::check_launch("tc_gemm");
}

extern "C" int cv3_tc_gemm(const float* a, int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc, int64_t m,
                           int64_t n, int64_t k, int mode, const float* bias, const float* gate,
                           int64_t rows_per_group, int64_t gate_stride, void* stream) {
  // Two K-range accumulators for the hi*hi products and two for the hi*lo +
  // lo*hi terms (all 512 TMEM columns): measured against fp64 this keeps the
  // error of K = 1024 / 2048 reductions at 1.7e-6 / 3.1e-6, where a single
  // accumulator gives 1.0e-5 / 1.7e-5 -- small addends lose bits when the
  // tensor core adds them into a large accumulator.  Same speed.
  return tc_gemm_layout(a, lda, b, ldb, c, ldc, m, n, k, mode, bias, gate, rows_per_group, gate_stride, 2, 1,
                        stream);
}

extern "C" int cv3_tc_gemm_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_tc_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

extern "C" int cv3_tf32_lo(const float* x, int64_t n, float* lo, void* stream) {
  CV3_REQUIRE(n >= 0, CV3_ERR_VALUE, "tf32_lo: negative size");
  if (n == 0) return CV3_OK;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  split::tf32_lo_kernel<<<(unsigned)blocks, 256, 0, cv3::as_stream(stream)>>>(x, n, lo);
  return cv3::check_launch("tf32_lo");
}

extern "C" int cv3_tc_gemm_split(const float* a, int64_t lda, const float* b, const float* b_lo, int64_t ldb,
                                 float* c, int64_t ldc, int64_t m, int64_t n, int64_t k, int mode, const float* bias,
                                 const float* gate, int64_t rows_per_group, int64_t gate_stride, void* stream) {
  CV3_REQUIRE(m >= 0 && n >= 0 && k >= 0 && mode >= 0 && mode <= 3, CV3_ERR_VALUE, "tc_gemm_split: bad arguments");
  CV3_REQUIRE(mode != 2 || gate != nullptr, CV3_ERR_VALUE, "tc_gemm_split: gated residual needs a gate");
  CV3_REQUIRE(lda >= k && ldb >= k && ldc >= n, CV3_ERR_VALUE, "tc_gemm_split: leading dimension too small");
  CV3_REQUIRE(k % 4 == 0, CV3_ERR_VALUE, "tc_gemm_split: K must be a multiple of 4 (16-byte rows)");
  if (m == 0 || n == 0) return CV3_OK;
  CV3_REQUIRE(k > 0 && b_lo != nullptr, CV3_ERR_VALUE, "tc_gemm_split: K must be positive and b_lo given");
  CV3_REQUIRE(m < (1LL << 31) && n < (1LL << 31) && k < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_split: too large");
  CUtensorMap ma, mb, mbl;
  int rc = make_map(&ma, a, m, k, lda, split::BM);
  if (rc) return rc;
  rc = make_map(&mb, b, n, k, ldb, split::BN);
  if (rc) return rc;
  rc = make_map(&mbl, b_lo, n, k, ldb, split::BN);
  if (rc) return rc;
  rc = cv3::allow_smem((const void*)split::tc_gemm_split_kernel, split::SMEM_BYTES);
  if (rc) return rc;
  const int64_t ntiles = ((n + split::BN - 1) / split::BN) * ((m + split::BM - 1) / split::BM);
  CV3_REQUIRE(ntiles < (1LL << 31), CV3_ERR_VALUE, "tc_gemm_split: too many tiles");
  const int grid = (int)std::min<int64_t>(ntiles, cv3::sm_count());  // persistent: one CTA per SM
  Epi ep{1, 1, mode, bias, gate, rows_per_group, gate_stride};
  split::tc_gemm_split_kernel<<<grid, split::THREADS, split::SMEM_BYTES, cv3::as_stream(stream)>>>(
      ma, mb, mbl, (int)m, (int)n, (int)k, c, ldc, ep);
  return cv3::check_launch("tc_gemm_split");
}

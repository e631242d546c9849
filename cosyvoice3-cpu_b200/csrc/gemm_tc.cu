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

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 4;
constexpr int TILE_A = BM * BK * 4;               // 16 KB
constexpr int TILE_B = BN * BK * 4;               // 16 KB
constexpr int STAGE_BYTES = TILE_A + 2 * TILE_B;  // A | raw B | B lo
constexpr int THREADS = 192;
constexpr uint32_t C_MAIN0 = 0, C_MAIN1 = 128, C_CROSS = 256, C_A = 384;
constexpr uint32_t IDESC = idesc_tf32(BM, BN);

struct Bars {
  uint64_t full[STAGES], empty[STAGES], afull[2], aempty[2], acc;
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES];
};
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + (int)sizeof(Bars);

__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_split_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_blo, int M, int N, int K, float* __restrict__ C,
                     int64_t ldc, Epi ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& S = *reinterpret_cast<Bars*>(smem + STAGES * STAGE_BYTES);
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int nk = (K + BK - 1) / BK;
  const int half = (nk + 1) / 2;  // first K block of the second hi*hi accumulator (used when nk >= 2)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 5);  // MMA commit + four converter warps
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.afull[i], 4);
      mbar_init(&S.aempty[i], 1);
    }
    mbar_init(&S.acc, 1);
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
  auto ready = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    const bool ok = !*abort_flag && mbar_wait(bar, parity, code);
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (*abort_flag || !mbar_wait(&S.empty[s], (r & 1) ^ 1, 21)) {
          *abort_flag = 1;
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
  } else if (warp == 1) {
    bool ok = true;
    for (int kb = 0; ok && kb < nk; ++kb) {
      const int s = kb % STAGES;
      const uint32_t r = (uint32_t)(kb / STAGES);
      const int a = kb & 1;
      if (!ready(&S.full[s], r & 1, 22) || !ready(&S.afull[a], (uint32_t)(kb >> 1) & 1, 23)) {
        ok = false;
        break;
      }
      fence_after();
      const int chunk = (nk >= 2 && kb >= half) ? 1 : 0;
      const int chunk_first = chunk ? half : 0;
      const uint32_t d_main = tmem + (chunk ? C_MAIN1 : C_MAIN0), d_cross = tmem + C_CROSS;
      const uint32_t b_raw = smem_u32(smem + s * STAGE_BYTES + TILE_A), b_lo = b_raw + TILE_B;
      const uint32_t a_hi = tmem + C_A + 64u * a, a_lo = a_hi + 32;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;
        mma_ts(d_cross, a_lo + 8 * kk, desc_k_sw128(b_raw + off), IDESC, (kb == 0 && kk == 0) ? 0u : 1u);
        mma_ts(d_cross, a_hi + 8 * kk, desc_k_sw128(b_lo + off), IDESC, 1u);
        mma_ts(d_main, a_hi + 8 * kk, desc_k_sw128(b_raw + off), IDESC, (kb == chunk_first && kk == 0) ? 0u : 1u);
      }
      mma_commit(&S.empty[s]);
      mma_commit(&S.aempty[a]);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.acc);  // also on abort: arrives once whatever was issued has completed
  } else {
    // ---- A rows into TMEM (one row per thread = its TMEM lane), then the epilogue ----
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int grow = m0 + row;
    const bool live = grow < M;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      const int a = kb & 1;
      if (!ready(&S.full[s], (uint32_t)(kb / STAGES) & 1, 24)) {
        ok = false;
        break;
      }
      // this thread's row of the swizzled A tile: 16-byte chunk j sits at chunk j ^ (row % 8);
      // a quarter-warp reads eight rows' chunks from eight distinct bank groups
      const uint8_t* arow = smem + s * STAGE_BYTES + row * 128;
      float hi[32], lo[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = *reinterpret_cast<const float4*>(arow + ((j ^ (row & 7)) << 4));
        const float e4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[4 * j + e] = tf32_hi(e4[e]);
          lo[4 * j + e] = e4[e] - hi[4 * j + e];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);  // this warp's rows of the stage are read
      if (!ready(&S.aempty[a], ((uint32_t)(kb >> 1) & 1) ^ 1, 25)) {
        ok = false;
        break;
      }
      fence_after();
      tmem_st32(tmem + lane_base + C_A + 64u * a, hi);
      tmem_st32(tmem + lane_base + C_A + 64u * a + 32, lo);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.afull[a]);
    }
    if (!ok) *abort_flag = 1;
    ok = ok && ready(&S.acc, 0, 26);
    fence_after();
    if (ok) {
      const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32], w[32];
        tmem_ld32(tmem + lane_base + C_CROSS + c0, v);
        if (nk >= 2) {
          tmem_ld32(tmem + lane_base + C_MAIN1 + c0, w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += w[j];
        }
        tmem_ld32(tmem + lane_base + C_MAIN0 + c0, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += w[j];
        if (!live) continue;
        float* crow = C + (int64_t)grow * ldc + n0 + c0;
        const float* gate = ep.mode == 2 ? ep.gate + (ep.rows_per_group > 0 ? grow / ep.rows_per_group : 0) *
                                                       ep.gate_stride + n0 + c0
                                         : nullptr;
        const int ncol = min(32, N - (n0 + c0));
        if (ncol <= 0) continue;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float res[4] = {0.f, 0.f, 0.f, 0.f};
          const bool full4 = vec && 4 * j4 + 3 < ncol;
          if (ep.mode >= 2) {
            if (full4) {
              const float4 t = *reinterpret_cast<const float4*>(crow + 4 * j4);
              res[0] = t.x; res[1] = t.y; res[2] = t.z; res[3] = t.w;
            } else {
              for (int e = 0; e < 4; ++e)
                if (4 * j4 + e < ncol) res[e] = crow[4 * j4 + e];
            }
          }
          float out[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * j4 + e;
            float y = v[j];
            if (j < ncol) {
              if (ep.bias) y = __fadd_rn(y, ep.bias[n0 + c0 + j]);
              if (ep.mode == 1) y = gelu_tanh(y);
              else if (ep.mode == 2) y = __fadd_rn(res[e], __fmul_rn(gate[j], y));
              else if (ep.mode == 3) y = __fadd_rn(res[e], y);
            }
            out[e] = y;
          }
          if (full4) {
            *reinterpret_cast<float4*>(crow + 4 * j4) = make_float4(out[0], out[1], out[2], out[3]);
          } else {
            for (int e = 0; e < 4; ++e)
              if (4 * j4 + e < ncol) crow[4 * j4 + e] = out[e];
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      if (*abort_flag)
        for (int s = 0; s < STAGES; ++s)
          if (S.issued[s] >= 0) mbar_wait(&S.full[s], (uint32_t)S.issued[s] & 1, 27);
      mbar_wait(&S.acc, 0, 28);  // every MMA (and its barrier arrivals) finished
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

extern "C" int cv3_tc_gemm_cfg(const float* a, int64_t lda, const float* b, int64_t ldb, float* c, int64_t ldc,
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
  return cv3_tc_gemm_cfg(a, lda, b, ldb, c, ldc, m, n, k, mode, bias, gate, rows_per_group, gate_stride, 2, 1,
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
  dim3 grid((unsigned)((n + split::BN - 1) / split::BN), (unsigned)((m + split::BM - 1) / split::BM));
  CV3_REQUIRE(grid.y <= 65535, CV3_ERR_VALUE, "tc_gemm_split: too many row tiles");
  Epi ep{1, 1, mode, bias, gate, rows_per_group, gate_stride};
  split::tc_gemm_split_kernel<<<grid, split::THREADS, split::SMEM_BYTES, cv3::as_stream(stream)>>>(
      ma, mb, mbl, (int)m, (int)n, (int)k, c, ldc, ep);
  return cv3::check_launch("tc_gemm_split");
}

// ---------------------------------------------------------------------------
// Tensor-pipe peak probe: every SM issues back-to-back kind::tf32 MMAs
// (M = 128, N = 256, K = 8, operands from shared memory, one accumulator) and
// the rate is reported in TFLOP/s -- the denominator the 3xTF32 kernels'
// tensor-pipe utilisation is quoted against.
// ---------------------------------------------------------------------------
namespace {

__global__ void __launch_bounds__(64, 1) tf32_peak_kernel(int reps, int* err) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 48 * 1024 / 4; i += blockDim.x) reinterpret_cast<float*>(sm)[i] = 0.0f;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&slot)), "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = slot;
  constexpr uint32_t ID = idesc_tf32(128, 256);
  const uint32_t a = smem_u32(sm), b = a + 16384;
  if (warp == 1) {
    for (int i = 0; i < reps; ++i)
      mma_ss(tmem, desc_k_sw128(a + (i & 3) * 32), desc_k_sw128(b + (i & 3) * 32), ID, i > 0 ? 1u : 0u);
    mma_commit(&bar);
    if ((threadIdx.x & 31) == 0) cv3tc::mbar_wait(&bar, 0, err, 1);
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
}

__device__ int g_probe_err = 0;

}  // namespace

extern "C" int cv3_tc_tf32_peak(double* tflops, void* stream) {
  CV3_REQUIRE(tflops != nullptr, CV3_ERR_VALUE, "tc_tf32_peak: no output");
  const int smem = 50 * 1024;
  int rc = cv3::allow_smem((const void*)tf32_peak_kernel, smem);
  if (rc) return rc;
  int* err = nullptr;
  CV3_CUDA(cudaGetSymbolAddress((void**)&err, g_probe_err));
  cudaStream_t st = cv3::as_stream(stream);
  const int grid = cv3::sm_count(), reps = 8192;
  tf32_peak_kernel<<<grid, 64, smem, st>>>(256, err);  // warm-up
  rc = cv3::check_launch("tc_tf32_peak");
  if (rc) return rc;
  cudaEvent_t e0, e1;
  CV3_CUDA(cudaEventCreate(&e0));
  CV3_CUDA(cudaEventCreate(&e1));
  CV3_CUDA(cudaEventRecord(e0, st));
  tf32_peak_kernel<<<grid, 64, smem, st>>>(reps, err);
  rc = cv3::check_launch("tc_tf32_peak");
  CV3_CUDA(cudaEventRecord(e1, st));
  CV3_CUDA(cudaEventSynchronize(e1));
  float ms = 0.f;
  CV3_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  *tflops = 2.0 * 128 * 256 * 8 * (double)reps * grid / (ms * 1e-3) / 1e12;
  return CV3_OK;
}

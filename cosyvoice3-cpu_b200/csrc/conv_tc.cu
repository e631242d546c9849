// 1-D convolution as an implicit GEMM on the tcgen05 tensor cores.
//
//   y[b][co][t] = snake(act(bias[co] + sum_{j < k, ci < C_in/g} W[co][ci][j] *
//                             x[b][g*C_in/g + ci][t*stride + j*dil - pad_l]))  (+ res[b][co][t])
//
// with the activation and the per-channel snake optional, so a conv and the
// elementwise op after it (and a residual add) are one kernel.
//
// (cv3cpu/ops.py:165-219; zero padding implicit: inputs outside [0, T_in) read
// as zero, so t_out fixes the right pad.)  GEMM view per (batch, group):
// rows = output frames (M), columns = output channels (N), reduction =
// (input channel, tap) pairs, channel-block major: K block kb = cb * k + j covers
// input channels [32 cb, 32 cb + 32) of tap j.  The weights are rearranged once
// (cv3_conv_weight_tc) into Wt[co][cb][j][32], the K-major B operand, with an
// optional tf32 remainder (weights stored as fp16 -- the vocoder's -- are exact
// tf32 values and need none: two products per element instead of three).
//
// Two kernels share that layout and the epilogue.
//
// Window kernel (stride 1: the vocoder's and the DiT's convs).  Persistent CTAs
// walk 128-frame x 64-channel tiles.  For each channel block, the input window
// -- 32 channels x the 128 + (k-1) dil frames all k taps of the tile touch -- is
// staged ONCE in shared memory as a K-major, 128 B-swizzled [frames][32] tile
// (and its tf32 remainder beside it); tap j's A operand is then the same tile
// shifted down by j*dil rows: a shared-memory descriptor whose start moves by
// j*dil*128 bytes.  So the k taps of a channel block cost k x 4 tcgen05.mma per
// product and no per-tap data movement.  12 warps:
//   warp 0     TMA: Wt (and Wt lo) tiles into a 4-stage ring;
//   warp 1     MMA issuer (converged warp, elect.sync): A and B from shared memory;
//   warp 2     TMA: token-major input windows, straight into the swizzled A tile
//              (one 3-D box per channel block);
//   warps 4-7  builders: load a channel-major window from global memory
//              (lanes on consecutive frames, coalesced; issued before the wait for
//              a free A tile so the latency hides behind it) and transpose it into
//              the A tile; write the remainder tile (x - tf32(x)) for both layouts;
//   warps 8-11 drainers: fold each K block's TMEM accumulator into fp32
//              registers (round-to-nearest adds; the tensor core's own adds
//              truncate), then the tile's epilogue -- while the MMA warp already
//              runs the next tile into the other accumulator sets.
// TMEM: six main accumulator sets (one per K block in flight) and two remainder
// accumulators (one per tile parity), 64 columns each.
//
// Gather kernel (any stride and layout): A from TMEM; warps 2-5 load each
// thread's 32 inputs of a K block straight from global memory, split them into
// tf32 hi/lo and store them to TMEM.
//
// Every wait is bounded (error word: cv3_tc_conv_status).
#include <algorithm>
#include <cstring>

#include "snake.cuh"
#include "tc_common.cuh"

namespace {

using namespace cv3tc;

constexpr int BM = 128, BN = 64, BK = 32;
constexpr int TILE_B = BN * BK * 4;      // one 64 x 32 weight tile
constexpr int STAGE_BYTES = 2 * TILE_B;  // W | W lo
constexpr uint32_t IDESC = idesc_tf32(BM, BN);
constexpr int SMEM_MAX = 232448;  // opt-in shared memory per block

__device__ int g_conv_err = 0;

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, int code) {
  return cv3tc::mbar_wait(bar, parity, &g_conv_err, code);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

struct ConvArgs {
  const float* x;
  int64_t xsb, xsc, xst;  // element (b, c, t) of x at b*xsb + c*xsc + t*xst
  float* y;
  int64_t ysb, ysc, yst;
  const float* bias;   // [C_out] or null
  const float* alpha;  // snake alpha per output channel, or null
  const float* res;    // residual with y's strides (may alias y) or null
  int act;             // CV3_ACT_* applied after the bias, -1 none
  float act_p;
  int cin_g, t_in, cout_g, t_out;
  int k, stride, dil, pad_l, groups;
  int cblocks;  // ceil(cin_g / 32): channel blocks
  int has_lo;
};

// bias and activation of one accumulator value (channel parameters passed in)
template <int ACT>
__device__ __forceinline__ float pre_snake(const ConvArgs& a, float acc, float bias) {
  float o = acc;
  if (a.bias) o = __fadd_rn(o, bias);
  if (ACT >= 0) o = act_apply(ACT, a.act_p, o);
  return o;
}

// ... then the snake (cv3cpu/ops.py:77-81), whose squared sine is the branch-free form
// (FAST) or the one valid for any argument
template <int ACT, bool SNAKE, bool FAST>
__device__ __forceinline__ float epilogue_value(const ConvArgs& a, float acc, float bias, float alpha) {
  const float o = pre_snake<ACT>(a, acc, bias);
  if (!SNAKE) return o;
  const float z = __fmul_rn(alpha, o);
  return cv3snake::snake_combine(o, cv3snake::inv_alpha(alpha), FAST ? cv3snake::sin_sq_fast(z) : cv3snake::sin_sq(z));
}

// Epilogue of one output frame t (this thread's row): NC channels from co0 of group g,
// in chunks of CH channels whose bias / alpha / residual loads are all issued before the
// chunk's stores (y may alias the residual, so a load placed after a store could not be
// hoisted and every channel would pay a full load latency).  A chunk first checks its
// snake arguments against the branch-free sine's range, so that its values are one
// straight line of independent arithmetic that interleaves (sinf's range branch
// serialised them); the values replace acc in place.
template <int ACT, bool SNAKE, int CH = 16, int NC = BN>
__device__ __forceinline__ void store_row(const ConvArgs& a, float (&acc)[NC], int b, int g, int co0, int t) {
  const bool yvec = a.ysc == 1 && a.yst % 4 == 0 && ((reinterpret_cast<uintptr_t>(a.y) & 15) == 0) &&
                    (a.ysb % 4 == 0) && (a.cout_g % 4 == 0) &&
                    (!a.res || (reinterpret_cast<uintptr_t>(a.res) & 15) == 0);
  const int ch0 = g * a.cout_g + co0;  // first output channel (global index)
  const int64_t ybase = (int64_t)b * a.ysb + (int64_t)ch0 * a.ysc + (int64_t)t * a.yst;
  const int nco = min(NC, a.cout_g - co0);
#pragma unroll
  for (int c0 = 0; c0 < NC; c0 += CH) {
    float bv[CH], av[CH], rv[CH];
#pragma unroll
    for (int e = 0; e < CH; ++e) {
      const bool in = c0 + e < nco;
      bv[e] = (a.bias && in) ? __ldg(a.bias + ch0 + c0 + e) : 0.f;
      av[e] = (SNAKE && in) ? __ldg(a.alpha + ch0 + c0 + e) : 0.f;
    }
    bool big = false;
    if (SNAKE) {
#pragma unroll
      for (int e = 0; e < CH; ++e)
        big |= !(fabsf(__fmul_rn(av[e], pre_snake<ACT>(a, acc[c0 + e], bv[e]))) <= cv3snake::FAST_MAX);
    }
    if (SNAKE && big) {
#pragma unroll
      for (int e = 0; e < CH; ++e) acc[c0 + e] = epilogue_value<ACT, SNAKE, false>(a, acc[c0 + e], bv[e], av[e]);
    } else {
#pragma unroll
      for (int e = 0; e < CH; ++e) acc[c0 + e] = epilogue_value<ACT, SNAKE, true>(a, acc[c0 + e], bv[e], av[e]);
    }
    if (yvec && nco == NC) {
      // token-major y: this thread's channels are contiguous
      if (a.res) {
#pragma unroll
        for (int q = 0; q < CH / 4; ++q) {
          const float4 r4 = *reinterpret_cast<const float4*>(a.res + ybase + c0 + 4 * q);
          rv[4 * q] = r4.x;
          rv[4 * q + 1] = r4.y;
          rv[4 * q + 2] = r4.z;
          rv[4 * q + 3] = r4.w;
        }
      }
#pragma unroll
      for (int q = 0; q < CH / 4; ++q) {
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o[e] = acc[c0 + 4 * q + e];
          if (a.res) o[e] = __fadd_rn(o[e], rv[4 * q + e]);
        }
        *reinterpret_cast<float4*>(a.y + ybase + c0 + 4 * q) = make_float4(o[0], o[1], o[2], o[3]);
      }
    } else {
      // channel-major y: lanes write consecutive frames of each channel
      if (a.res) {
#pragma unroll
        for (int e = 0; e < CH; ++e) rv[e] = c0 + e < nco ? a.res[ybase + (int64_t)(c0 + e) * a.ysc] : 0.f;
      }
#pragma unroll
      for (int e = 0; e < CH; ++e) {
        if (c0 + e < nco) {
          float o = acc[c0 + e];
          if (a.res) o = __fadd_rn(o, rv[e]);
          a.y[ybase + (int64_t)(c0 + e) * a.ysc] = o;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Gather kernel
// ---------------------------------------------------------------------------------
namespace gk {

constexpr int STAGES = 4, THREADS = 192;
constexpr uint32_t C_A = 384;
// main (hi*W) accumulator of K block kb at 64 (kb & 1); the remainder products
// (2^-11 of the main terms, so their own truncation is harmless) accumulate over
// the whole reduction in one accumulator at 128
constexpr uint32_t C_CROSS = 128;
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;

struct Bars {
  uint64_t full[STAGES], empty[STAGES], afull[2], aempty[2], accfull[2], drained[2], done;
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES];
};
static_assert(sizeof(Bars) <= 256, "gather kernel barriers");

// the 32 inputs of K block kb for output frame t (zero outside the signal / channels).
// Channel-major x: lane-consecutive frames, one coalesced row per channel.  Token-major
// x (vec): the thread's 32 channels are contiguous, read as float4.
// (offsets inside one (batch, group) slab fit 31 bits; the host checks)
__device__ __forceinline__ void gather(float (&v)[32], const ConvArgs& a, const float* xg, int t, int kb, bool vec) {
  const int cb = kb / a.k, j = kb - cb * a.k;
  const int ci0 = cb * 32;
  const int ti = t * a.stride + j * a.dil - a.pad_l;
  const bool ok = t < a.t_out && ti >= 0 && ti < a.t_in;
  const int xsc = (int)a.xsc;
  const float* p = xg + (ok ? ti * (int)a.xst + ci0 * xsc : 0);
  if (!vec && ok && ci0 + 32 <= a.cin_g) {
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = __ldg(p + c * xsc);
    return;
  }
  if (vec) {
#pragma unroll
    for (int c4 = 0; c4 < 8; ++c4) {
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok && ci0 + 4 * c4 < a.cin_g) q = __ldg(reinterpret_cast<const float4*>(p + 4 * c4));
      v[4 * c4] = q.x;
      v[4 * c4 + 1] = q.y;
      v[4 * c4 + 2] = q.z;
      v[4 * c4 + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = (ok && ci0 + c < a.cin_g) ? __ldg(p + c * xsc) : 0.f;
  }
}

// Accuracy: the tensor core truncates when it adds into an fp32 accumulator, so
// a sum over thousands of products drifts (~K/8 truncations).  Here every main
// accumulator sums one K block; two alternate, and the converter warps drain
// each finished one into fp32 registers (round-to-nearest adds) while the tensor
// core fills the other.
template <int ACT, bool SNAKE>
__global__ void __launch_bounds__(THREADS, 1)
conv_gather_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_wlo, ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  Bars& S = *reinterpret_cast<Bars*>(smem + STAGES * STAGE_BYTES);
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * BM;
  const int co0 = blockIdx.y * BN;  // inside the group
  const int b = blockIdx.z / a.groups, g = blockIdx.z - b * a.groups;
  const int wrow0 = g * a.cout_g + co0;  // first row of Wt
  const int nk = a.k * a.cblocks;
  const uint32_t tx_bytes = (uint32_t)(a.has_lo ? STAGE_BYTES : TILE_B);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.afull[i], 4);
      mbar_init(&S.aempty[i], 1);
      mbar_init(&S.accfull[i], 1);
      mbar_init(&S.drained[i], 4);
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
  auto ready = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    const bool ok = !*abort_flag && bwait(bar, parity, code);
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t r = (uint32_t)(kb / STAGES);
        if (*abort_flag || !bwait(&S.empty[s], (r & 1) ^ 1, 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        S.issued[s] = (int)r;
        mbar_expect_tx(&S.full[s], tx_bytes);
        tma_load_2d(st, &map_w, &S.full[s], kb * BK, wrow0);
        if (a.has_lo) tma_load_2d(st + TILE_B, &map_wlo, &S.full[s], kb * BK, wrow0);
      }
    }
  } else if (warp == 1) {
    bool ok = true;
    for (int kb = 0; ok && kb < nk; ++kb) {
      const int s = kb % STAGES;
      const uint32_t r = (uint32_t)(kb / STAGES);
      const int as = kb & 1;
      // an accumulator is reused once its previous K block has been drained
      if (kb >= 2 && !ready(&S.drained[as], ((uint32_t)(kb >> 1) & 1) ^ 1, 8)) {
        ok = false;
        break;
      }
      if (!ready(&S.full[s], r & 1, 2) || !ready(&S.afull[as], (uint32_t)(kb >> 1) & 1, 3)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t d_main = tmem + 64u * as, d_cross = tmem + C_CROSS;
      const uint32_t w_raw = smem_u32(smem + s * STAGE_BYTES), w_lo = w_raw + TILE_B;
      const uint32_t a_hi = tmem + C_A + 64u * as, a_lo = a_hi + 32;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;
        mma_ts(d_cross, a_lo + 8 * kk, desc_k_sw128(w_raw + off), IDESC, (kb == 0 && kk == 0) ? 0u : 1u);
        if (a.has_lo) mma_ts(d_cross, a_hi + 8 * kk, desc_k_sw128(w_lo + off), IDESC, 1u);
        mma_ts(d_main, a_hi + 8 * kk, desc_k_sw128(w_raw + off), IDESC, kk == 0 ? 0u : 1u);
      }
      mma_commit(&S.empty[s]);
      mma_commit(&S.aempty[as]);
      mma_commit(&S.accfull[as]);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.done);  // also on abort: arrives once whatever was issued has completed
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int t = t0 + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float* xg = a.x + (int64_t)b * a.xsb + (int64_t)g * a.cin_g * a.xsc;
    const bool vec = a.xsc == 1 && a.xst % 4 == 0 && a.cin_g % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(xg) & 15) == 0);
    bool ok = true;
    float acc[BN];
#pragma unroll
    for (int c = 0; c < BN; ++c) acc[c] = 0.f;
    // fold K block q's accumulator into acc and hand it back to the MMA warp
    auto drain = [&](int q) -> bool {
      const int set = q & 1;
      if (!ready(&S.accfull[set], (uint32_t)(q >> 1) & 1, 5)) return false;
      fence_after();
      float m[BN];
      tmem_ld64(tmem + lane_base + 64u * set, m);
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = __fadd_rn(acc[j], m[j]);
      if (q == nk - 1) {  // the last block's MMAs are the last ones: the remainder sum is final
        tmem_ld64(tmem + lane_base + C_CROSS, m);
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = __fadd_rn(acc[j], m[j]);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.drained[set]);
      return true;
    };
    float cur[32], nxt[32];
    if (nk > 0) gather(cur, a, xg, t, 0, vec);
    int drained = 0;  // K blocks folded so far
    for (int kb = 0; kb < nk; ++kb) {
      if (kb + 1 < nk) gather(nxt, a, xg, t, kb + 1, vec);  // in flight while this block is stored
      const int as = kb & 1;
      float hi[32], lo[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        hi[c] = tf32_hi(cur[c]);
        lo[c] = cur[c] - hi[c];
      }
      if (!ready(&S.aempty[as], ((uint32_t)(kb >> 1) & 1) ^ 1, 4)) {
        ok = false;
        break;
      }
      fence_after();
      tmem_st32(tmem + lane_base + C_A + 64u * as, hi);
      tmem_st32(tmem + lane_base + C_A + 64u * as + 32, lo);
      tmem_st_wait();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.afull[as]);
      // once block kb's A is stored, block kb - 1 is (or soon is) complete
      if (kb >= 1) {
        if (!drain(drained)) {
          ok = false;
          break;
        }
        ++drained;
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) cur[c] = nxt[c];
    }
    while (ok && drained < nk) {
      if (!drain(drained)) ok = false;
      ++drained;
    }
    if (!ok) *abort_flag = 1;
    if (ok && t < a.t_out) store_row<ACT, SNAKE>(a, acc, b, g, co0, t);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      if (*abort_flag)
        for (int s = 0; s < STAGES; ++s)
          if (S.issued[s] >= 0) bwait(&S.full[s], (uint32_t)S.issued[s] & 1, 6);
      bwait(&S.done, 0, 7);
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace gk

// ---------------------------------------------------------------------------------
// Window kernel
// ---------------------------------------------------------------------------------
namespace wk {

constexpr int MAX_STAGES = 8;            // weight ring (as many stages as shared memory leaves, >= 2)
constexpr int NSET_MAX = 6;
constexpr int FMAX = 256;                // window rows (TMA box limit)

// Tile width: 64 output channels, or 128 where a group has that many (one MMA then does
// twice the work: at these widths the tensor pipe is paced by the reduction length, not
// by N).  TMEM holds NSET main accumulators (K blocks in flight between MMA and drain)
// and two remainder accumulators (even / odd tiles), BNW columns each.  Eight drain warps,
// two per TMEM lane quarter, fold BNW / 2 channels each: two warps per SM sub-partition
// hide each other's TMEM-load and barrier latencies.
template <int BNW>
struct Wide {
  static constexpr int THREADS = 512;
  static constexpr int NSET = BNW == 64 ? 6 : 2;
  static constexpr int NDRAIN = 8;         // drain warps
  static constexpr int DW = BNW / 2;       // channels per drain warp
  static constexpr uint32_t C_CROSS = NSET * BNW;
  static constexpr int TILE = BNW * BK * 4;  // one BNW x 32 weight tile
  static constexpr uint32_t IDESC = idesc_tf32(BM, BNW);
};

struct Bars {
  uint64_t full[MAX_STAGES], empty[MAX_STAGES];
  uint64_t afull[2], aempty[2];      // A tile pair nb: built / free again
  uint64_t winfull[2];               // token-major window nb landed in A tile nb
  uint64_t accfull[NSET_MAX], drained[NSET_MAX];
  uint64_t crossdrained[2];
  uint64_t done;
  uint32_t tmem;
  int abort_flag;
  int issued[MAX_STAGES];
  int issued_win[2];
};

struct WinArgs {
  ConvArgs c;
  int frames;   // window rows F = 128 + (k - 1) dil
  int abytes;   // bytes of one A tile (F x 128 B, rounded up to the 1024 B swizzle period)
  int nx, ny, ntiles;
  int nstages;      // weight ring depth
  int stage_bytes;  // 8 KB (W) or 16 KB (W | W lo)
};

// smem: [W ring | A hi 0 | A hi 1 | A lo 0 | A lo 1 | Bars]
__host__ __device__ inline int bars_at(int abytes, int nstages, int stage_bytes) {
  return nstages * stage_bytes + 4 * abytes;
}

// The A operands are descriptors of the window tiles advanced by whole 128 B rows.
// The 128 B swizzle is a function of the absolute shared-memory address (chunk bits
// 4-6 XOR row bits 7-9), the same rule TMA and the builders write with, so such a
// start needs no base-offset field (measured: filling that field with the row phase
// scrambles the products).

// byte offset of (frame f, channels 4q..4q+3) in a [frames][32] tile with the 128 B swizzle
__device__ __forceinline__ int sw_off(int f, int q) { return f * 128 + ((q ^ (f & 7)) << 4); }

// One K block of the window kernel from one elected thread: for k-steps kk = 0..3
// (descriptor start + 2 kk), main += A hi x W (fresh at kk = 0) and remainder +=
// A lo x W (+ A hi x W lo with LO), then the two commits (weight slot free, K block's
// accumulator complete).  One asm block: a single elect and no per-MMA bookkeeping
// between the eight (twelve) issues.
template <bool LO>
__device__ __forceinline__ void issue_kblock(uint32_t d_main, uint32_t d_cross, uint64_t a_hi, uint64_t a_lo,
                                             uint64_t w, uint64_t w_lo, uint32_t cross_acc, uint64_t* bar_empty,
                                             uint64_t* bar_acc, uint32_t idesc) {
  if (LO) {
    asm volatile(
        "{\n\t.reg .pred e, pf, pt, pc;\n\t.reg .b64 h1, h2, h3, l1, l2, l3, w1, w2, w3, v0, v1, v2, v3;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 pf, %4, %4;\n\tsetp.eq.b32 pt, %4, %4;\n\tsetp.ne.b32 pc, %4, 0;\n\t"
        "add.s64 h1, %5, 2;\n\tadd.s64 h2, %5, 4;\n\tadd.s64 h3, %5, 6;\n\t"
        "add.s64 l1, %6, 2;\n\tadd.s64 l2, %6, 4;\n\tadd.s64 l3, %6, 6;\n\t"
        "add.s64 w1, %7, 2;\n\tadd.s64 w2, %7, 4;\n\tadd.s64 w3, %7, 6;\n\t"
        "mov.b64 v0, %8;\n\tadd.s64 v1, %8, 2;\n\tadd.s64 v2, %8, 4;\n\tadd.s64 v3, %8, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %5, %7, %2, pf;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], %6, %7, %2, pc;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], %5, v0, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h1, w1, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l1, w1, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], h1, v1, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h2, w2, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l2, w2, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], h2, v2, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h3, w3, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l3, w3, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], h3, v3, %2, pt;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%3];\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%9];\n\t}" ::"r"(d_main),
        "r"(d_cross), "r"(idesc), "r"(smem_u32(bar_empty)), "r"(cross_acc), "l"(a_hi), "l"(a_lo), "l"(w), "l"(w_lo),
        "r"(smem_u32(bar_acc))
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e, pf, pt, pc;\n\t.reg .b64 h1, h2, h3, l1, l2, l3, w1, w2, w3;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 pf, %4, %4;\n\tsetp.eq.b32 pt, %4, %4;\n\tsetp.ne.b32 pc, %4, 0;\n\t"
        "add.s64 h1, %5, 2;\n\tadd.s64 h2, %5, 4;\n\tadd.s64 h3, %5, 6;\n\t"
        "add.s64 l1, %6, 2;\n\tadd.s64 l2, %6, 4;\n\tadd.s64 l3, %6, 6;\n\t"
        "add.s64 w1, %7, 2;\n\tadd.s64 w2, %7, 4;\n\tadd.s64 w3, %7, 6;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %5, %7, %2, pf;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], %6, %7, %2, pc;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h1, w1, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l1, w1, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h2, w2, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l2, w2, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], h3, w3, %2, pt;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%1], l3, w3, %2, pt;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%3];\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%8];\n\t}" ::"r"(d_main),
        "r"(d_cross), "r"(idesc), "r"(smem_u32(bar_empty)), "r"(cross_acc), "l"(a_hi), "l"(a_lo), "l"(w),
        "r"(smem_u32(bar_acc))
        : "memory");
  }
}

__device__ __forceinline__ float4 split_lo(float4 h) {
  return make_float4(h.x - tf32_hi(h.x), h.y - tf32_hi(h.y), h.z - tf32_hi(h.z), h.w - tf32_hi(h.w));
}

// acc[j] += TMEM row columns j (NC of them), rounded to nearest, in loads of 32 columns
template <int NC>
__device__ __forceinline__ void fold_cols(uint32_t taddr, float (&acc)[NC]) {
#pragma unroll
  for (int h = 0; h < NC / 32; ++h) {
    float m[32];
    tmem_ld32(taddr + 32 * h, m);
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[32 * h + j] = __fadd_rn(acc[32 * h + j], m[j]);
  }
}

// LAYOUT 1: channel-major x (frames contiguous); 2: token-major x (channels contiguous)
template <int ACT, bool SNAKE, int LAYOUT, int BNW>
__global__ void __launch_bounds__(Wide<BNW>::THREADS, 1)
conv_window_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_wlo,
                   const __grid_constant__ CUtensorMap map_x, WinArgs p) {
  const ConvArgs& a = p.c;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* const abase = smem + p.nstages * p.stage_bytes;  // A hi 0, A hi 1, A lo 0, A lo 1
  Bars& S = *reinterpret_cast<Bars*>(smem + bars_at(p.abytes, p.nstages, p.stage_bytes));
  const int ns = p.nstages;
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = a.k * a.cblocks;
  using C = Wide<BNW>;
  const uint32_t tx_bytes = (uint32_t)(a.has_lo ? 2 * C::TILE : C::TILE);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
      S.issued[s] = -1;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.afull[i], 4);
      mbar_init(&S.aempty[i], 1);
      mbar_init(&S.winfull[i], 1);
      mbar_init(&S.crossdrained[i], C::NDRAIN);
      S.issued_win[i] = -1;
    }
    for (int i = 0; i < C::NSET; ++i) {
      mbar_init(&S.accfull[i], 1);
      mbar_init(&S.drained[i], C::NDRAIN);
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
    const bool ok = !*abort_flag && bwait(bar, parity, code);
    return __all_sync(0xffffffffu, ok);
  };
  // tile -> first frame, first channel (in the group), batch, group; consecutive tiles
  // run along time, so CTAs working at the same time share weight tiles in L2
  auto tile_of = [&](int tile, int& t0, int& co0, int& b, int& g) {
    const int tx = tile % p.nx, rest = tile / p.nx;
    const int ty = rest % p.ny, z = rest / p.ny;
    t0 = tx * BM;
    co0 = ty * BNW;
    b = z / a.groups;
    g = z - b * a.groups;
  };

  if (warp == 0) {
    // weight tiles, K block by K block, tile after tile
    if (lane == 0) {
      int s = 0, r = 0;  // ring slot, and how many times the ring has wrapped
      bool go = true;
      for (int tile = blockIdx.x; go && tile < p.ntiles; tile += gridDim.x) {
        int t0, co0, b, g;
        tile_of(tile, t0, co0, b, g);
        const int wrow0 = g * a.cout_g + co0;
        for (int kb = 0; kb < nk; ++kb) {
          if (*abort_flag || !bwait(&S.empty[s], (uint32_t)(r & 1) ^ 1, 1)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          uint8_t* st = smem + s * p.stage_bytes;
          S.issued[s] = r;
          mbar_expect_tx(&S.full[s], tx_bytes);
          tma_load_2d(st, &map_w, &S.full[s], kb * BK, wrow0);
          if (a.has_lo) tma_load_2d(st + C::TILE, &map_wlo, &S.full[s], kb * BK, wrow0);
          if (++s == ns) s = 0, ++r;
        }
      }
    }
  } else if (warp == 1) {
    bool ok = true;
    const bool has_lo = a.has_lo != 0;
    int gkb = 0, gcb = 0, it = 0, s = 0, r = 0;
    for (int tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x, ++it) {
      const int cp = it & 1;
      // this tile's remainder accumulator was last used two tiles ago: drained by now?
      if (it >= 2 && !ready(&S.crossdrained[cp], ((uint32_t)(it >> 1) & 1) ^ 1, 12)) {
        ok = false;
        break;
      }
      const uint32_t d_cross = tmem + C::C_CROSS + (uint32_t)BNW * cp;
      for (int cb = 0; ok && cb < a.cblocks; ++cb, ++gcb) {
        const int nb = gcb & 1;
        if (!ready(&S.afull[nb], (uint32_t)(gcb >> 1) & 1, 3)) {
          ok = false;
          break;
        }
        // descriptors advance in 16 B units of their start-address field: + 8 per window
        // row (tap shift), + 2 per k-step of 8 tf32 (the field cannot carry: smem < 256 KB)
        const uint64_t d_ahi = desc_k_sw128(smem_u32(abase + nb * p.abytes));
        const uint64_t d_alo = desc_k_sw128(smem_u32(abase + (2 + nb) * p.abytes));
        for (int j = 0; j < a.k; ++j, ++gkb) {
          const int set = gkb % C::NSET;
          if (gkb >= C::NSET && !ready(&S.drained[set], ((uint32_t)(gkb / C::NSET) & 1) ^ 1, 8)) {
            ok = false;
            break;
          }
          if (!ready(&S.full[s], (uint32_t)r & 1, 2)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t d_main = tmem + (uint32_t)BNW * set;
          const uint64_t d_w = desc_k_sw128(smem_u32(smem + s * p.stage_bytes)), d_wlo = d_w + (C::TILE >> 4);
          const uint64_t shift = (uint64_t)(j * a.dil) * 8;  // tap j reads the window shifted by j*dil frames
          const uint32_t first = (cb == 0 && j == 0) ? 0u : 1u;
          if (has_lo)
            issue_kblock<true>(d_main, d_cross, d_ahi + shift, d_alo + shift, d_w, d_wlo, first, &S.empty[s],
                               &S.accfull[set], C::IDESC);
          else
            issue_kblock<false>(d_main, d_cross, d_ahi + shift, d_alo + shift, d_w, d_wlo, first, &S.empty[s],
                                &S.accfull[set], C::IDESC);
          if (++s == ns) s = 0, ++r;
        }
        if (!ok) break;
        mma_commit(&S.aempty[nb]);
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;
    mma_commit(&S.done);  // also on abort: arrives once whatever was issued has completed
  } else if (warp == 2) {
    // token-major input windows
    if (LAYOUT == 2 && lane == 0) {
      int gcb = 0;
      bool go = true;
      for (int tile = blockIdx.x; go && tile < p.ntiles; tile += gridDim.x) {
        int t0, co0, b, g;
        tile_of(tile, t0, co0, b, g);
        const int wstart = t0 - a.pad_l;  // window row 0 = input frame of output t0, tap 0
        const int ch0 = g * a.cin_g;
        for (int cb = 0; cb < a.cblocks; ++cb, ++gcb) {
          const int nb = gcb & 1;
          if (*abort_flag || !bwait(&S.aempty[nb], ((uint32_t)(gcb >> 1) & 1) ^ 1, 9)) {
            *abort_flag = 1;
            go = false;
            break;
          }
          S.issued_win[nb] = gcb >> 1;
          mbar_expect_tx(&S.winfull[nb], (uint32_t)(p.frames * 128));
          tma_load_3d(abase + nb * p.abytes, &map_x, &S.winfull[nb], ch0 + 32 * cb, wstart, b);
        }
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // builders: window frames tid and tid + 128
    const int tid = threadIdx.x - 128;
    int gcb = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x) {
      int t0, co0, b, g;
      tile_of(tile, t0, co0, b, g);
      const int wstart = t0 - a.pad_l;
      const int ch0 = g * a.cin_g;
      for (int cb = 0; cb < a.cblocks; ++cb, ++gcb) {
        const int nb = gcb & 1;
        const int nval = a.cin_g - 32 * cb;  // channels of this block inside the group (>= 32: all)
        uint8_t* hb = abase + nb * p.abytes;
        uint8_t* lb = abase + (2 + nb) * p.abytes;
        if (LAYOUT == 1) {
          // the block's inputs for frames tid and tid + 128, in flight during the wait below
          const float* xc = a.x + (int64_t)b * a.xsb + (int64_t)(ch0 + 32 * cb) * a.xsc;
          float v0[32], v1[32];
          const int f1 = tid + 128;
          const bool has1 = f1 < p.frames;
          const int t0f = wstart + tid, t1f = wstart + f1;
          const bool in0 = t0f >= 0 && t0f < a.t_in, in1 = has1 && t1f >= 0 && t1f < a.t_in;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float* pc = xc + (int64_t)c * a.xsc;
            v0[c] = (in0 && c < nval) ? __ldg(pc + t0f) : 0.f;
            v1[c] = (in1 && c < nval) ? __ldg(pc + t1f) : 0.f;
          }
          if (!ready(&S.aempty[nb], ((uint32_t)(gcb >> 1) & 1) ^ 1, 4)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 h = make_float4(v0[4 * q], v0[4 * q + 1], v0[4 * q + 2], v0[4 * q + 3]);
            *reinterpret_cast<float4*>(hb + sw_off(tid, q)) = h;
            *reinterpret_cast<float4*>(lb + sw_off(tid, q)) = split_lo(h);
          }
          if (has1) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 h = make_float4(v1[4 * q], v1[4 * q + 1], v1[4 * q + 2], v1[4 * q + 3]);
              *reinterpret_cast<float4*>(hb + sw_off(f1, q)) = h;
              *reinterpret_cast<float4*>(lb + sw_off(f1, q)) = split_lo(h);
            }
          }
        } else {
          if (!ready(&S.aempty[nb], ((uint32_t)(gcb >> 1) & 1) ^ 1, 4) ||
              !ready(&S.winfull[nb], (uint32_t)(gcb >> 1) & 1, 10)) {
            ok = false;
            break;
          }
          for (int f = tid; f < p.frames; f += 128) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 h = *reinterpret_cast<const float4*>(hb + sw_off(f, q));
              if (4 * q >= nval) {  // the next group's channels (or nothing): zero
                h = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(hb + sw_off(f, q)) = h;
              }
              *reinterpret_cast<float4*>(lb + sw_off(f, q)) = split_lo(h);
            }
          }
        }
        // order these generic-proxy writes before the tensor core's reads
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.afull[nb]);
      }
    }
    if (!ok) *abort_flag = 1;
  } else if (warp >= 8) {
    // drainers + epilogue: thread = output frame t0 + row (its TMEM lane), channels
    // DW half .. DW half + DW - 1 of the tile
    const int quarter = warp & 3, half = (warp - 8) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = ((uint32_t)(quarter * 32) << 16) + (uint32_t)(C::DW * half);
    int gkb = 0, it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x, ++it) {
      int t0, co0, b, g;
      tile_of(tile, t0, co0, b, g);
      const int cp = it & 1;
      float acc[C::DW];
#pragma unroll
      for (int c = 0; c < C::DW; ++c) acc[c] = 0.f;
      for (int kb = 0; kb < nk; ++kb, ++gkb) {
        const int set = gkb % C::NSET;
        if (!ready(&S.accfull[set], (uint32_t)(gkb / C::NSET) & 1, 5)) {
          ok = false;
          break;
        }
        fence_after();
        fold_cols<C::DW>(tmem + lane_base + (uint32_t)BNW * set, acc);
        const bool last = kb == nk - 1;  // its MMAs are the tile's last: the remainder sum is final
        if (last) {
          fold_cols<C::DW>(tmem + lane_base + C::C_CROSS + (uint32_t)BNW * cp, acc);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&S.drained[set]);
          if (last) mbar_arrive(&S.crossdrained[cp]);
        }
      }
      if (!ok) break;
      const int t = t0 + row;
      if (t < a.t_out) store_row<ACT, SNAKE, BNW == 64 ? 16 : 8, C::DW>(a, acc, b, g, co0 + C::DW * half, t);
    }
    if (!ok) *abort_flag = 1;
  }
  fence_before();
  __syncthreads();
  if (LAYOUT == 2 && warp == 2 && lane == 0 && *abort_flag) {  // window loads still in flight land first
    for (int i = 0; i < 2; ++i)
      if (S.issued_win[i] >= 0) bwait(&S.winfull[i], (uint32_t)S.issued_win[i] & 1, 11);
  }
  if (warp == 0) {
    if (lane == 0) {
      if (*abort_flag)
        for (int s = 0; s < ns; ++s)
          if (S.issued[s] >= 0) bwait(&S.full[s], (uint32_t)S.issued[s] & 1, 6);
      bwait(&S.done, 0, 7);
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace wk

int make_w_map(CUtensorMap* map, const float* ptr, int64_t rows, int64_t kp, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  CV3_REQUIRE(encode != nullptr, CV3_ERR_CUDA, "conv1d_tc: cuTensorMapEncodeTiled is unavailable");
  CV3_REQUIRE(((uintptr_t)ptr & 15) == 0, CV3_ERR_VALUE, "conv1d_tc: weight base must be 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(kp * 4)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)ptr, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CV3_REQUIRE(r == CUDA_SUCCESS, CV3_ERR_CUDA, "conv1d_tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CV3_OK;
}

// Token-major x as (channels, frames, batch) with boxes of 32 channels x `frames`,
// 128 B-swizzled: the window lands as the kernel's A tile.  False when the strides
// are not 16-byte multiples.
bool make_x_map_tokens(CUtensorMap* map, const float* x, int64_t xsb, int64_t xst, int64_t batch, int64_t cin,
                       int64_t t_in, int frames) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (!encode || ((uintptr_t)x & 15)) return false;
  const int64_t sb = batch > 1 ? xsb : xst * t_in;
  if (xst % 4 || sb % 4 || xst <= 0 || sb <= 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cin, (cuuint64_t)t_in, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(xst * 4), (cuuint64_t)(sb * 4)};
  cuuint32_t box[3] = {32, (cuuint32_t)frames, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)x, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int g_window_enabled = 1;
int g_last_path = -1;  // kernel of the last launch: 0 gather, 1 / 2 window (channel- / token-major)

__global__ void conv_weight_kernel(const float* __restrict__ w, int cout, int cin_g, int k, int ci_pad,
                                   float* __restrict__ wt, float* __restrict__ wt_lo) {
  const int64_t total = (int64_t)cout * k * ci_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    // Wt[co][cb][j][32]
    const int ci = (int)((i / (32 * k)) % (ci_pad / 32)) * 32 + (int)(i % 32);
    const int j = (int)((i / 32) % k);
    const int co = (int)(i / ((int64_t)ci_pad * k));
    const float v = ci < cin_g ? w[((int64_t)co * cin_g + ci) * k + j] : 0.f;
    wt[i] = v;
    if (wt_lo) wt_lo[i] = v - tf32_hi(v);
  }
}

using GatherFn = void (*)(const CUtensorMap, const CUtensorMap, ConvArgs);
using WindowFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, wk::WinArgs);

template <int ACT>
GatherFn gather_fn(bool sn) {
  return sn ? gk::conv_gather_kernel<ACT, true> : gk::conv_gather_kernel<ACT, false>;
}

// token-major inputs come from the DiT (no snake): that layout is built without one
template <int ACT, int BNW>
WindowFn window_fn_w(bool sn, int layout) {
  if (layout == 1)
    return sn ? wk::conv_window_kernel<ACT, true, 1, BNW> : wk::conv_window_kernel<ACT, false, 1, BNW>;
  return sn ? nullptr : wk::conv_window_kernel<ACT, false, 2, BNW>;
}

template <int ACT>
WindowFn window_fn(bool sn, int layout, bool wide) {
  return wide ? window_fn_w<ACT, 128>(sn, layout) : window_fn_w<ACT, 64>(sn, layout);
}

}  // namespace

extern "C" int cv3_conv_weight_tc(const float* w, int64_t cout, int64_t cin_g, int64_t k, int64_t ci_pad, float* wt,
                                  float* wt_lo, void* stream) {
  CV3_REQUIRE(cout > 0 && cin_g > 0 && k > 0 && ci_pad >= cin_g && ci_pad % 32 == 0, CV3_ERR_VALUE,
              "conv_weight_tc: bad geometry (ci_pad must be a multiple of 32 covering C_in/groups)");
  CV3_REQUIRE(cout * k * ci_pad < (1LL << 40), CV3_ERR_VALUE, "conv_weight_tc: too large");
  const int64_t total = cout * k * ci_pad;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  conv_weight_kernel<<<(unsigned)blocks, 256, 0, cv3::as_stream(stream)>>>(w, (int)cout, (int)cin_g, (int)k,
                                                                          (int)ci_pad, wt, wt_lo);
  return cv3::check_launch("conv_weight_tc");
}

extern "C" int cv3_conv1d_tc(const float* x, int64_t xsb, int64_t xsc, int64_t xst, int64_t batch, int64_t cin,
                             int64_t t_in, const float* wt, const float* wt_lo, int64_t ci_pad, int64_t cout,
                             int64_t k, int64_t stride, int64_t dilation, int64_t groups, int64_t pad_left,
                             const float* bias, int act, float act_param, const float* snake_alpha,
                             const float* residual, float* y, int64_t ysb, int64_t ysc, int64_t yst, int64_t t_out,
                             void* stream) {
  CV3_REQUIRE(batch >= 0 && cin > 0 && cout > 0 && k > 0 && stride > 0 && dilation > 0 && groups > 0 &&
                  pad_left >= 0 && t_in >= 0 && t_out >= 0,
              CV3_ERR_VALUE, "conv1d_tc: bad geometry");
  CV3_REQUIRE(cin % groups == 0 && cout % groups == 0, CV3_ERR_VALUE, "conv1d_tc: channels not divisible by groups");
  const int64_t cin_g = cin / groups, cout_g = cout / groups;
  CV3_REQUIRE(ci_pad % 32 == 0 && ci_pad >= cin_g && ci_pad < cin_g + 32, CV3_ERR_VALUE,
              "conv1d_tc: ci_pad must be C_in/groups rounded up to 32");
  if (batch == 0 || t_out == 0) return CV3_OK;
  CV3_REQUIRE(t_in < (1LL << 30) && t_out < (1LL << 30) && k * ci_pad < (1LL << 30), CV3_ERR_VALUE,
              "conv1d_tc: too large");
  CV3_REQUIRE(act == -1 || act == CV3_ACT_MISH || act == CV3_ACT_ELU || act == CV3_ACT_LEAKY_RELU,
              CV3_ERR_UNSUPPORTED, "conv1d_tc: activation %d not built into the conv epilogue", act);
  const int64_t nx = (t_out + BM - 1) / BM, ny = (cout_g + BN - 1) / BN, nz = batch * groups;
  CV3_REQUIRE(ny <= 65535 && nz <= 65535, CV3_ERR_VALUE, "conv1d_tc: grid too large");
  CV3_REQUIRE(cin_g * xsc < (1LL << 31) && t_in * xst + cin * xsc < (1LL << 31), CV3_ERR_VALUE,
              "conv1d_tc: one (batch, group) slab of x must span < 2^31 elements");
  CUtensorMap mw, mwl;
  int rc = make_w_map(&mw, wt, cout, k * ci_pad, BN);
  if (rc) return rc;
  rc = make_w_map(&mwl, wt_lo ? wt_lo : wt, cout, k * ci_pad, BN);
  if (rc) return rc;
  const ConvArgs a{x, xsb, xsc, xst, y, ysb, ysc, yst, bias, snake_alpha, residual, act, act_param,
                   (int)cin_g, (int)t_in, (int)cout_g, (int)t_out,
                   (int)k, (int)stride, (int)dilation, (int)pad_left, (int)groups, (int)(ci_pad / 32), wt_lo ? 1 : 0};
  const bool sn = snake_alpha != nullptr;

  // window kernel: stride 1 and a window of <= 256 rows; tiles 128 channels wide where a
  // group has that many
  const int64_t frames = BM + (k - 1) * dilation;
  const bool wide = cout_g >= 128;
  const int bnw = wide ? 128 : BN;
  const int64_t nyw = (cout_g + bnw - 1) / bnw;
  const int64_t ntiles = nx * nyw * nz;
  if (g_window_enabled && stride == 1 && ntiles < (1LL << 31)) {
    wk::WinArgs p{};
    CUtensorMap mx;
    std::memset(&mx, 0, sizeof(mx));
    int layout = 0;
    if (xst == 1 && frames <= wk::FMAX) {
      layout = 1;
    } else if (xsc == 1 && frames <= wk::FMAX && cin_g % 4 == 0 &&
               make_x_map_tokens(&mx, x, xsb, xst, batch, cin, t_in, (int)frames)) {
      layout = 2;
    }
    WindowFn fn = nullptr;
    if (layout) {
      switch (act) {
        case -1: fn = window_fn<-1>(sn, layout, wide); break;
        case CV3_ACT_MISH: fn = window_fn<CV3_ACT_MISH>(sn, layout, wide); break;
        case CV3_ACT_ELU: fn = window_fn<CV3_ACT_ELU>(sn, layout, wide); break;
        default: fn = window_fn<CV3_ACT_LEAKY_RELU>(sn, layout, wide); break;
      }
    }
    CUtensorMap mww = mw, mwlw = mwl;  // weight tiles of the window kernel: bnw rows
    if (fn && wide) {
      rc = make_w_map(&mww, wt, cout, k * ci_pad, bnw);
      if (rc) return rc;
      rc = make_w_map(&mwlw, wt_lo ? wt_lo : wt, cout, k * ci_pad, bnw);
      if (rc) return rc;
    }
    p.c = a;
    p.frames = (int)frames;
    p.abytes = (int)((frames * 128 + 1023) / 1024 * 1024);
    p.nx = (int)nx;
    p.ny = (int)nyw;
    p.ntiles = (int)ntiles;
    // the weight ring takes what the windows leave: deep rings hide the L2 latency of
    // one 8 / 16 KB (x2 with the remainder) tile per K block
    const int tile_w = bnw * BK * 4;
    p.stage_bytes = wt_lo ? 2 * tile_w : tile_w;
    const int fixed = wk::bars_at(p.abytes, 0, 0) + (int)sizeof(wk::Bars) + 1024;
    p.nstages = std::min(wk::MAX_STAGES, (SMEM_MAX - fixed) / p.stage_bytes);
    const int smem = fixed + p.nstages * p.stage_bytes;
    if (fn && p.nstages >= 2) {
      rc = cv3::allow_smem((const void*)fn, smem);
      if (rc) return rc;
      const int grid = (int)std::min<int64_t>(ntiles, cv3::sm_count());
      g_last_path = layout;
      fn<<<grid, wide ? wk::Wide<128>::THREADS : wk::Wide<64>::THREADS, smem, cv3::as_stream(stream)>>>(mww, mwlw, mx,
                                                                                                   p);
      return cv3::check_launch("conv1d_tc");
    }
  }

  GatherFn fn;
  switch (act) {
    case -1: fn = gather_fn<-1>(sn); break;
    case CV3_ACT_MISH: fn = gather_fn<CV3_ACT_MISH>(sn); break;
    case CV3_ACT_ELU: fn = gather_fn<CV3_ACT_ELU>(sn); break;
    default: fn = gather_fn<CV3_ACT_LEAKY_RELU>(sn); break;
  }
  rc = cv3::allow_smem((const void*)fn, gk::SMEM);
  if (rc) return rc;
  g_last_path = 0;
  dim3 grid((unsigned)nx, (unsigned)ny, (unsigned)nz);
  fn<<<grid, gk::THREADS, gk::SMEM, cv3::as_stream(stream)>>>(mw, mwl, a);
  return cv3::check_launch("conv1d_tc");
}

extern "C" int cv3_conv_tc_set_window(int enable) {
  g_window_enabled = enable ? 1 : 0;
  return CV3_OK;
}

extern "C" int cv3_conv_tc_last_path(int* path) {
  if (path) *path = g_last_path;
  return CV3_OK;
}

extern "C" int cv3_tc_conv_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_conv_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_conv_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

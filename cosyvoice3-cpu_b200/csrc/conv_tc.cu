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
// (tap, input channel) pairs, tap-major: K block kb covers 32 input channels of
// one tap.  The weights are rearranged once (cv3_conv_weight_tc) into
// Wt[co][j][ci_pad], the K-major B operand, with an optional tf32 remainder
// (weights stored as fp16 -- the vocoder's -- are exact tf32 values and need
// none: two products per element instead of three).
//
// CTA = 128 output frames x 64 channels, 6 warps:
//   warp 0     TMA: Wt (and Wt lo) tiles into a 4-stage ring;
//   warp 1     MMA issuer (converged warp, elect.sync): A from TMEM, B from smem;
//   warps 2-5  one output frame per thread (= its TMEM lane): gather the 32
//              (tap, channel) inputs of each K block straight from global memory
//              (channel-major x: lanes read consecutive frames, coalesced), the
//              next block in flight while the current one is split into tf32
//              hi/lo and stored to TMEM; they also fold the finished TMEM
//              accumulators into fp32 registers, then run the epilogue.
// TMEM: two main accumulator sets and one remainder accumulator (64 columns
// each), two A stages (32 hi + 32 lo columns each).  Every wait is bounded (error
// word: cv3_tc_conv_status).
#include <algorithm>

#include "tc_common.cuh"

namespace {

using namespace cv3tc;

constexpr int BM = 128, BK = 32, STAGES = 4, THREADS = 192;
constexpr uint32_t C_A = 384;

__device__ int g_conv_err = 0;

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, int code) {
  return cv3tc::mbar_wait(bar, parity, &g_conv_err, code);
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
  int cblocks;  // ceil(cin_g / 32): K blocks per tap
  int has_lo;
};

struct Bars {
  uint64_t full[STAGES], empty[STAGES], afull[2], aempty[2], accfull[2], drained[2], done;
  uint32_t tmem;
  int abort_flag;
  int issued[STAGES];
};

// 128 frames x 64 channels per CTA (TS MMAs with N = 64 run at the full tensor rate)
constexpr int BN = 64;
constexpr int TILE_B = BN * BK * 4;
constexpr int STAGE_BYTES = 2 * TILE_B;  // W | W lo
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + (int)sizeof(Bars);
#ifndef CV3_CONV_GROUP
#define CV3_CONV_GROUP 1
#endif
constexpr int GROUP = CV3_CONV_GROUP;  // K blocks summed in one TMEM accumulator before it is drained
constexpr uint32_t IDESC = idesc_tf32(BM, BN);
// main (hi*W) accumulator set q at 64q; the remainder products (2^-11 of the
// main terms, so their own truncation is harmless) accumulate over the whole
// reduction in one accumulator at 128
__device__ __forceinline__ uint32_t c_main(int set) { return (uint32_t)(64 * set); }
constexpr uint32_t C_CROSS = 128;

// the 32 inputs of K block kb for output frame t (zero outside the signal / channels).
// Channel-major x: lane-consecutive frames, one coalesced row per channel.  Token-major
// x (vec): the thread's 32 channels are contiguous, read as float4.
// (offsets inside one (batch, group) slab fit 31 bits; the host checks)
__device__ __forceinline__ void gather(float (&v)[32], const ConvArgs& a, const float* xg, int t, int kb, bool vec) {
  const int j = kb / a.cblocks;
  const int ci0 = (kb - j * a.cblocks) * 32;
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

template <int ACT, bool SNAKE>
__device__ __forceinline__ float epilogue_value(const ConvArgs& a, int ch, float acc) {
  float o = acc;
  if (a.bias) o = __fadd_rn(o, a.bias[ch]);
  if (ACT >= 0) o = act_apply(ACT, a.act_p, o);
  if (SNAKE) {  // snake (cv3cpu/models/hift.py: x + 1/(alpha + 1e-9) * sin(alpha x)^2)
    const float al = a.alpha[ch];
    const float sn = sinf(al * o);
    o = o + (1.0f / (al + 1e-9f)) * (sn * sn);
  }
  return o;
}

// Accuracy: the tensor core truncates when it adds into an fp32 accumulator, so
// a sum over thousands of products drifts (~K/8 truncations).  Here every
// accumulator sums only GROUP K blocks; two sets alternate, and the converter
// warps drain each finished set into fp32 registers (round-to-nearest adds)
// while the tensor core fills the other.  Measured on the full f32 vocoder
// (dozens of chained convs, then exp() in the iSTFT) against the oracle:
// GROUP 4 / 2 / 1 -> 1.2e-5 / 8.9e-6 / 8.1e-6 of max (fp32 CUDA-core convs:
// 7.6e-6), for a 5% time difference; 1 is the default.
// ACT: the activation (CV3_ACT_*, -1 none) and SNAKE compiled in, so each
// instantiation carries only its own epilogue
template <int ACT, bool SNAKE>
__global__ void __launch_bounds__(THREADS, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_wlo, ConvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars& S = *reinterpret_cast<Bars*>(smem + STAGES * STAGE_BYTES);
  volatile int* abort_flag = &S.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * BM;
  const int co0 = blockIdx.y * BN;  // inside the group
  const int b = blockIdx.z / a.groups, g = blockIdx.z - b * a.groups;
  const int wrow0 = g * a.cout_g + co0;  // first row of Wt
  const int nk = a.k * a.cblocks;
  const int ngroups = (nk + GROUP - 1) / GROUP;
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
      const int q = kb / GROUP, set = q & 1;
      const bool first = kb == q * GROUP, last = kb == nk - 1 || kb == (q + 1) * GROUP - 1;
      // a set is reused once its previous group has been drained
      if (first && q >= 2 && !ready(&S.drained[set], ((uint32_t)(q >> 1) & 1) ^ 1, 8)) {
        ok = false;
        break;
      }
      if (!ready(&S.full[s], r & 1, 2) || !ready(&S.afull[as], (uint32_t)(kb >> 1) & 1, 3)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t d_main = tmem + c_main(set), d_cross = tmem + C_CROSS;
      const uint32_t w_raw = smem_u32(smem + s * STAGE_BYTES), w_lo = w_raw + TILE_B;
      const uint32_t a_hi = tmem + C_A + 64u * as, a_lo = a_hi + 32;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint32_t off = kk * 32;
        const uint32_t acc = (first && kk == 0) ? 0u : 1u;
        mma_ts(d_cross, a_lo + 8 * kk, desc_k_sw128(w_raw + off), IDESC, (kb == 0 && kk == 0) ? 0u : 1u);
        if (a.has_lo) mma_ts(d_cross, a_hi + 8 * kk, desc_k_sw128(w_lo + off), IDESC, 1u);
        mma_ts(d_main, a_hi + 8 * kk, desc_k_sw128(w_raw + off), IDESC, acc);
      }
      mma_commit(&S.empty[s]);
      mma_commit(&S.aempty[as]);
      if (last) mma_commit(&S.accfull[set]);
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
    // fold accumulator set q into acc and hand it back to the MMA warp
    auto drain = [&](int q) -> bool {
      const int set = q & 1;
      if (!ready(&S.accfull[set], (uint32_t)(q >> 1) & 1, 5)) return false;
      fence_after();
      float m[BN];
      tmem_ld64(tmem + lane_base + c_main(set), m);
#pragma unroll
      for (int j = 0; j < BN; ++j) acc[j] = __fadd_rn(acc[j], m[j]);
      if (q == ngroups - 1) {  // the last group's MMAs are the last ones: the remainder sum is final
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
    int drained = 0;  // groups folded so far
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
      // once the A of group q is all stored, group q - 1 is (or soon is) complete
      if ((kb == nk - 1 || (kb + 1) % GROUP == 0) && kb / GROUP >= 1) {
        if (!drain(drained)) {
          ok = false;
          break;
        }
        ++drained;
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) cur[c] = nxt[c];
    }
    while (ok && drained < ngroups) {
      if (!drain(drained)) ok = false;
      ++drained;
    }
    if (!ok) *abort_flag = 1;
    if (ok && t < a.t_out) {
      const bool yvec = a.ysc == 1 && a.yst % 4 == 0 && ((reinterpret_cast<uintptr_t>(a.y) & 15) == 0) &&
                        (a.ysb % 4 == 0) && (a.cout_g % 4 == 0) &&
                        (!a.res || (reinterpret_cast<uintptr_t>(a.res) & 15) == 0);
      const int64_t ybase = (int64_t)b * a.ysb + (int64_t)(g * a.cout_g) * a.ysc + (int64_t)t * a.yst;
      if (yvec && co0 + BN <= a.cout_g) {
        // token-major y: this thread's channels are contiguous
        float* yp = a.y + ybase + co0;
        const float* rp = a.res ? a.res + ybase + co0 : nullptr;
#pragma unroll
        for (int j4 = 0; j4 < BN / 4; ++j4) {
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o[e] = epilogue_value<ACT, SNAKE>(a, g * a.cout_g + co0 + 4 * j4 + e, acc[4 * j4 + e]);
          if (rp) {
            const float4 r4 = *reinterpret_cast<const float4*>(rp + 4 * j4);
            o[0] = __fadd_rn(o[0], r4.x);
            o[1] = __fadd_rn(o[1], r4.y);
            o[2] = __fadd_rn(o[2], r4.z);
            o[3] = __fadd_rn(o[3], r4.w);
          }
          *reinterpret_cast<float4*>(yp + 4 * j4) = make_float4(o[0], o[1], o[2], o[3]);
        }
      } else {
        // channel-major y: lanes write consecutive frames of each channel
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          const int co = co0 + j;
          if (co < a.cout_g) {
            float o = epilogue_value<ACT, SNAKE>(a, g * a.cout_g + co, acc[j]);
            const int64_t idx = ybase + (int64_t)co * a.ysc;
            if (a.res) o = __fadd_rn(o, a.res[idx]);
            a.y[idx] = o;
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
          if (S.issued[s] >= 0) bwait(&S.full[s], (uint32_t)S.issued[s] & 1, 6);
      bwait(&S.done, 0, 7);
    }
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

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

__global__ void conv_weight_kernel(const float* __restrict__ w, int cout, int cin_g, int k, int ci_pad,
                                   float* __restrict__ wt, float* __restrict__ wt_lo) {
  const int64_t total = (int64_t)cout * k * ci_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int ci = (int)(i % ci_pad);
    const int j = (int)((i / ci_pad) % k);
    const int co = (int)(i / ((int64_t)ci_pad * k));
    const float v = ci < cin_g ? w[((int64_t)co * cin_g + ci) * k + j] : 0.f;
    wt[i] = v;
    if (wt_lo) wt_lo[i] = v - tf32_hi(v);
  }
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
  CUtensorMap mw, mwl;
  int rc = make_w_map(&mw, wt, cout, k * ci_pad, BN);
  if (rc) return rc;
  rc = make_w_map(&mwl, wt_lo ? wt_lo : wt, cout, k * ci_pad, BN);
  if (rc) return rc;
  CV3_REQUIRE(act >= -1 && act <= CV3_ACT_EXP, CV3_ERR_VALUE, "conv1d_tc: unknown activation %d", act);
  ConvArgs a{x, xsb, xsc, xst, y, ysb, ysc, yst, bias, snake_alpha, residual, act, act_param,
             (int)cin_g, (int)t_in, (int)cout_g, (int)t_out,
             (int)k, (int)stride, (int)dilation, (int)pad_left, (int)groups, (int)(ci_pad / 32), wt_lo ? 1 : 0};
  dim3 grid((unsigned)((t_out + BM - 1) / BM), (unsigned)((cout_g + BN - 1) / BN), (unsigned)(batch * groups));
  CV3_REQUIRE(grid.y <= 65535 && grid.z <= 65535, CV3_ERR_VALUE, "conv1d_tc: grid too large");
  CV3_REQUIRE(cin_g * xsc < (1LL << 31) && t_in * xst + cin * xsc < (1LL << 31), CV3_ERR_VALUE,
              "conv1d_tc: one (batch, group) slab of x must span < 2^31 elements");
  using Fn = void (*)(const CUtensorMap, const CUtensorMap, ConvArgs);
  Fn fn = nullptr;
  const bool sn = snake_alpha != nullptr;
  switch (act) {
    case -1: fn = sn ? conv_tc_kernel<-1, true> : conv_tc_kernel<-1, false>; break;
    case CV3_ACT_MISH: fn = sn ? conv_tc_kernel<CV3_ACT_MISH, true> : conv_tc_kernel<CV3_ACT_MISH, false>; break;
    case CV3_ACT_ELU: fn = sn ? conv_tc_kernel<CV3_ACT_ELU, true> : conv_tc_kernel<CV3_ACT_ELU, false>; break;
    case CV3_ACT_LEAKY_RELU:
      fn = sn ? conv_tc_kernel<CV3_ACT_LEAKY_RELU, true> : conv_tc_kernel<CV3_ACT_LEAKY_RELU, false>;
      break;
    default: break;
  }
  CV3_REQUIRE(fn != nullptr, CV3_ERR_UNSUPPORTED, "conv1d_tc: activation %d not built into the conv epilogue", act);
  rc = cv3::allow_smem((const void*)fn, SMEM);
  if (rc) return rc;
  fn<<<grid, THREADS, SMEM, cv3::as_stream(stream)>>>(mw, mwl, a);
  return cv3::check_launch("conv1d_tc");
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

// Decode GEMV for q8 weights on the tensor cores (the LM's per-token linears,
// up to 32 activation rows):  y[m][row] = epilogue( sum_k xn[m][k] * q[row][k] * s[row][k/64] ).
//
// Why tensor cores for a GEMV: with 8 sequences every weight byte needs 8
// multiply-adds, which on CUDA cores makes the kernel instruction-bound well
// below HBM speed.  Here a warp-level MMA (m16n8k16, bf16 in, fp32 out) does
// them: A = 16 weight rows x 16 k (int8 values are exact in bf16), B = 16 k x
// 8 sequences of the activations split exactly into three bf16 parts
// (x = hi + mid + lo to fp32 precision), so each product is exact and the
// per-64-group fp16 scale is applied to the group's partial sum in fp32.
//
// K order inside a 64-wide scale group is permuted (the same way for both
// operands, so the dot product is unchanged) so that lane (g, c) of a warp --
// g = lane / 4, c = lane % 4 -- needs bytes 16c .. 16c+15 of weight rows g and
// g+8 and activations 16c .. 16c+15 of sequence g: one 16-byte load per row per
// group, straight into the MMA fragments.
//
// Up to 32 rows: the sequences form NB blocks of 8 (one n8 MMA column block each);
// every weight fragment is widened once per row tile and multiplied into all NB
// blocks, so the weights are streamed once per step whatever the batch.  A
// sequence's result does not depend on NB (its column block sees the same MMAs in
// the same order), so a sequence decodes the same ids in a batch of 32 as alone.
//
// CTA = 16 x RT weight rows x all of K, 8 warps (warp w takes every 8th scale
// group, for all RT row tiles); all of a warp's weight loads are issued
// first, with the epilogue's bias and the RMSNorm weight (constants); after
// the dependency wait the residual is read at once and the activations are
// copied to shared memory by one bulk copy per row (few large L2 requests: every
// CTA reads the same rows), completing on an mbarrier.  A fused RMSNorm
// (qwen2.py:145-150: (x * r) * w) is folded: the MMAs take x * w, each warp adds
// up x^2 for the groups it multiplies, and the row factor r multiplies the
// finished dot product -- no separate pass over x; the results differ from
// normalising first by fp32 rounding only.  The warps' partial sums are added in
// a fixed order in shared memory (deterministic).  Epilogues: bias, residual add
// (y may alias it), SwiGLU of interleaved gate/up rows (cv3cpu/models/qwen2.py:
// 155-177, llm.py:74-78).
#include "tc_common.cuh"

__device__ int g_gemv_err = 0;  // 1: an activation copy did not land in time (cv3_decode_gemv_status)

namespace {

using cv3tc::bulk_load;
using cv3tc::mbar_expect_tx;
using cv3tc::mbar_init;
using cv3tc::mbar_wait;

constexpr int NWARP = 8, MAXB = 8, MAXSEQ = 32;  // MAXB: sequences per n8 column block

struct MmaArgs {
  const float* x;
  int64_t ldx;
  int m, k;
  const int8_t* q;
  const uint16_t* sc;
  int n;
  const float* bias;
  const float* residual;
  float* y;
  int64_t ldy;
  const float* norm_w;
  float eps;
  int swiglu;
  int gsplit;        // scale groups per K split (all of them when not split)
  float* partial;    // [splits][n][8 NB] when split
  int* counter;      // [row tiles], zero on entry and left zero
  int cluster;       // 1: the K splits of a row tile form one thread-block cluster
};

// the 4 int8 values of one 32-bit word of a weight fragment as floats (exact)
__device__ __forceinline__ void widen4(uint32_t word, float f[4]) {
  const uint32_t u = word ^ 0x80808080u;
#pragma unroll
  for (int b = 0; b < 4; ++b) f[b] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7440u | b)) - 8388736.0f;
}

__device__ __forceinline__ uint32_t word_of(const int4& v, int j) {
  return (uint32_t)(j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w)));
}

// two floats that are exact bf16 values (low 16 bits zero) as one bf16x2
// register, `lo` in the low half (the lower k index): their top halves
__device__ __forceinline__ uint32_t pack(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

__device__ __forceinline__ float bf16_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFF0000u); }

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The 16 activations of one lane for one scale group (x * w with the folded RMSNorm,
// whose sum of squares of x goes to `ssq`), split exactly into three bf16 parts:
// hi = x truncated to bf16, mid = the remainder truncated, lo = what is left (<= 8
// significant bits, itself a bf16 value); packed as the MMA's B fragments.
__device__ __forceinline__ void split_activations(const float* xrow, const float* wrow, float& ssq,
                                                  uint32_t (&bp)[3][4][2]) {
  float xv[16];
  const float4* xp = reinterpret_cast<const float4*>(xrow);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const float4 t = xp[v];
    xv[4 * v] = t.x;
    xv[4 * v + 1] = t.y;
    xv[4 * v + 2] = t.z;
    xv[4 * v + 3] = t.w;
  }
  if (wrow) {
    const float4* wp = reinterpret_cast<const float4*>(wrow);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const float4 w4 = wp[v];
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ssq = fmaf(xv[4 * v + e], xv[4 * v + e], ssq);
        xv[4 * v + e] *= wv[e];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float pv[3][2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float x = xv[4 * j + 2 * h + u];
        const float hi = bf16_trunc(x);
        const float r1v = x - hi;
        const float mid = bf16_trunc(r1v);
        pv[0][u] = hi;
        pv[1][u] = mid;
        pv[2][u] = bf16_trunc(r1v - mid);
      }
#pragma unroll
      for (int pp = 0; pp < 3; ++pp) bp[pp][j][h] = pack(pv[pp][0], pv[pp][1]);
    }
}

// A fragments of the four k-steps of one 16-row tile and scale group (int8 exact in bf16)
__device__ __forceinline__ void weight_fragments(const int4& w0, const int4& w1, uint32_t (&A)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f0[4], f1[4];
    widen4(word_of(w0, j), f0);
    widen4(word_of(w1, j), f1);
    A[j][0] = pack(f0[0], f0[1]);  // row g,     k 2c, 2c+1
    A[j][1] = pack(f1[0], f1[1]);  // row g + 8, k 2c, 2c+1
    A[j][2] = pack(f0[2], f0[3]);  // row g,     k 2c+8, 2c+9
    A[j][3] = pack(f1[2], f1[3]);  // row g + 8, k 2c+8, 2c+9
  }
}

// one scale group of one row tile and one 8-sequence block: a chain of four MMAs per
// activation part, the parts added small first, times the rows' scales into acc
__device__ __forceinline__ void mma_group(const uint32_t (&A)[4][4], const uint32_t (&bp)[3][4][2], float s0,
                                          float s1, float (&acc)[4]) {
  float d[3][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int pp = 0; pp < 3; ++pp) mma_bf16(d[pp], A[j][0], A[j][1], A[j][2], A[j][3], bp[pp][j][0], bp[pp][j][1]);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float v = (d[2][e] + d[1][e]) + d[0][e];
    acc[e] = fmaf(v, e < 2 ? s0 : s1, acc[e]);
  }
}

// RT: 16-row tiles per CTA, every warp multiplying its scale groups into all of them
// (the activation split is done once per group and CTA); GMAX: most scale groups one
// warp takes (K <= 64 * NWARP * GMAX); NB: blocks of 8 sequences (8 NB rows at most)
template <int RT, int GMAX, int NB>
__global__ void __launch_bounds__(NWARP * 32, (GMAX <= 4 && NB == 1) ? 3 : 1)  // short K: 3 CTAs per SM (9728 rows in one wave)
q8_gemv_mma_kernel(MmaArgs a) {
  constexpr int ROWS = 16 * RT;
  constexpr int SEQ = MAXB * NB;                          // staged sequences
  constexpr int EPI = (ROWS * SEQ + NWARP * 32 - 1) / (NWARP * 32);  // epilogue outputs per thread
  extern __shared__ float xs[];  // [SEQ][k] staged activations, rows >= m zero
  __shared__ float red[NWARP][ROWS][SEQ];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int ks = a.k >> 6;
  // this CTA's K split: scale groups [g0, g0 + ng); x columns [64 g0, 64 (g0 + ng))
  const int g0 = blockIdx.y * a.gsplit;
  const int ng = min(a.gsplit, ks - g0);
  const int kw = 64 * ng;  // staged row width

  // -- weights first: they do not depend on x --------------------------------------------
  int4 w0[GMAX][RT], w1[GMAX][RT];
  float s0[GMAX][RT], s1[GMAX][RT];
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    const int G = warp + NWARP * i;
    const bool in = G < ng;
#pragma unroll
    for (int t = 0; t < RT; ++t) {
      const int r0 = min(blockIdx.x * ROWS + 16 * t + g, a.n - 1), r1 = min(blockIdx.x * ROWS + 16 * t + g + 8, a.n - 1);
      w0[i][t] = in ? ld_stream16(a.q + (int64_t)r0 * a.k + 64 * (g0 + G) + 16 * c) : make_int4(0, 0, 0, 0);
      w1[i][t] = in ? ld_stream16(a.q + (int64_t)r1 * a.k + 64 * (g0 + G) + 16 * c) : make_int4(0, 0, 0, 0);
      s0[i][t] = in ? h2f(a.sc[(int64_t)r0 * ks + g0 + G]) : 0.f;
      s1[i][t] = in ? h2f(a.sc[(int64_t)r1 * ks + g0 + G]) : 0.f;
    }
  }

  // constants of the epilogue and the RMSNorm weight (staged behind x) do not depend on
  // the previous kernels either
  const int k4 = kw >> 2;
  float* nws = xs + SEQ * kw;  // [kw] RMSNorm weight of this CTA's K range (only with norm_w)
  if (a.norm_w)
    for (int i = tid; i < k4; i += NWARP * 32)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(nws + 4 * i)),
                   "l"(a.norm_w + 64 * g0 + 4 * i)
                   : "memory");
  // epilogue outputs of this thread: index tid + 256 e -> (row inside the CTA, sequence)
  float bias_v[EPI], bias_u[EPI];
#pragma unroll
  for (int e = 0; e < EPI; ++e) {
    const int idx = tid + NWARP * 32 * e, rt = idx / SEQ, bb = idx - rt * SEQ;
    const int row = blockIdx.x * ROWS + rt;
    const bool epi = idx < ROWS * SEQ && row < a.n && bb < a.m;
    bias_v[e] = (epi && a.bias) ? a.bias[row] : 0.f;
    bias_u[e] = (epi && a.bias && a.swiglu && row + 1 < a.n) ? a.bias[row + 1] : 0.f;
  }

  // rows >= m read as zeros; the barrier of the activation copies
  __shared__ __align__(8) uint64_t xbar;
  for (int i = tid; i < (SEQ - a.m) * k4; i += NWARP * 32)
    reinterpret_cast<float4*>(xs + a.m * kw)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid == 0) {
    mbar_init(&xbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");  // the RMSNorm weight
  __syncthreads();

  // everything below reads what the previous kernels wrote
  dep_wait();
  dep_release();
  if (tid == 0) {
    mbar_expect_tx(&xbar, (uint32_t)(a.m * kw * 4));
    for (int mr = 0; mr < a.m; ++mr)
      bulk_load(xs + mr * kw, a.x + (int64_t)mr * a.ldx + 64 * g0, (uint32_t)(kw * 4), &xbar);
  }
  // the residual row is read now, so that its latency hides behind the copies and math
  // (y may alias it: each element is read and written by this same thread only)
  float res_v[EPI];
#pragma unroll
  for (int e = 0; e < EPI; ++e) {
    const int idx = tid + NWARP * 32 * e, rt = idx / SEQ, bb = idx - rt * SEQ;
    const int row = blockIdx.x * ROWS + rt;
    const bool epi = idx < ROWS * SEQ && row < a.n && bb < a.m;
    res_v[e] = (epi && !a.swiglu && a.residual) ? a.residual[(int64_t)bb * a.ldy + row] : 0.f;
  }
  const bool landed = mbar_wait(&xbar, 0, &g_gemv_err, 1);
  if (!__syncthreads_and(landed)) {
    // a copy that never lands: once more (bounded) before the CTA's shared memory goes
    if (tid == 0 && !landed) mbar_wait(&xbar, 0, &g_gemv_err, 1);
    return;
  }

  // -- per scale group: 4 k-steps x 3 activation parts x RT tiles x NB blocks MMAs, * scale --
  float acc[NB][RT][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int t = 0; t < RT; ++t) acc[nb][t][0] = acc[nb][t][1] = acc[nb][t][2] = acc[nb][t][3] = 0.f;
  float ssq[NB];  // sum of x^2 of sequence 8 nb + g over this lane's columns (RMSNorm)
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) ssq[nb] = 0.f;
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    const int G = warp + NWARP * i;
    if (G < ng) {
      if constexpr (NB == 1) {
        // one block: the activations split once, then every row tile
        uint32_t bp[3][4][2];
        split_activations(xs + g * kw + 64 * G + 16 * c, a.norm_w ? nws + 64 * G + 16 * c : nullptr, ssq[0], bp);
#pragma unroll
        for (int t = 0; t < RT; ++t) {
          uint32_t A[4][4];
          weight_fragments(w0[i][t], w1[i][t], A);
          mma_group(A, bp, s0[i][t], s1[i][t], acc[0][t]);
        }
      } else {
        // several blocks: every row tile's weights widened once, then each block's
        // activations split once and multiplied into all row tiles
        uint32_t A[RT][4][4];
#pragma unroll
        for (int t = 0; t < RT; ++t) weight_fragments(w0[i][t], w1[i][t], A[t]);
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          uint32_t bp[3][4][2];
          split_activations(xs + (MAXB * nb + g) * kw + 64 * G + 16 * c, a.norm_w ? nws + 64 * G + 16 * c : nullptr,
                            ssq[nb], bp);
#pragma unroll
          for (int t = 0; t < RT; ++t) mma_group(A[t], bp, s0[i][t], s1[i][t], acc[nb][t]);
        }
      }
    }
  }
  // every column is in exactly one warp: the warps' sums of squares
  __shared__ float sq[NWARP][SEQ];
  if (a.norm_w) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      float v = ssq[nb];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (c == 0) sq[warp][MAXB * nb + g] = v;
    }
  }
  // D fragments: rows 16t + g / 16t + g + 8, sequences 8 nb + 2c, 8 nb + 2c + 1
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int t = 0; t < RT; ++t) {
      red[warp][16 * t + g][MAXB * nb + 2 * c] = acc[nb][t][0];
      red[warp][16 * t + g][MAXB * nb + 2 * c + 1] = acc[nb][t][1];
      red[warp][16 * t + g + 8][MAXB * nb + 2 * c] = acc[nb][t][2];
      red[warp][16 * t + g + 8][MAXB * nb + 2 * c + 1] = acc[nb][t][3];
    }
  __syncthreads();

  // -- reduce the warps in a fixed order, then the K splits -----------------------------------
  __shared__ float tot[ROWS][SEQ];
  __shared__ float rnorm[SEQ];
  __shared__ int last_cta;
  for (int idx = tid; idx < ROWS * SEQ; idx += NWARP * 32) {
    const int rt = idx / SEQ, bb = idx - rt * SEQ;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) v += red[w][rt][bb];
    tot[rt][bb] = v;
  }
  // this CTA's sum of squares per sequence (its K range); with K splits split 0 adds the
  // others' in split order below, before the row factor is formed
  __shared__ float sqt[SEQ];
  if (a.norm_w && tid < SEQ) {
    float q = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) q += sq[w][tid];
    sqt[tid] = q;
    if (gridDim.y == 1) rnorm[tid] = 1.0f / sqrtf(q / (float)a.k + a.eps);
  }
  if (gridDim.y > 1 && a.cluster) {
    // the K splits of this row tile are one cluster: split 0 adds the others' sums from
    // their shared memory in split order (deterministic), the rest wait until it has read
    // them and leave; no global round trip
    float v[EPI];
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (a.norm_w && blockIdx.y == 0 && tid < SEQ) {
      float q = sqt[tid];
      const uint32_t local = (uint32_t)__cvta_generic_to_shared(&sqt[tid]);
      for (int sp = 1; sp < (int)gridDim.y; ++sp) {
        uint32_t remote;
        float pv;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(sp));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(remote) : "memory");
        q += pv;
      }
      rnorm[tid] = 1.0f / sqrtf(q / (float)a.k + a.eps);
    }
#pragma unroll
    for (int e = 0; e < EPI; ++e) {
      const int idx = tid + NWARP * 32 * e, rt = idx / SEQ, bb = idx - rt * SEQ;
      v[e] = 0.f;
      if (blockIdx.y == 0 && idx < ROWS * SEQ) {
        v[e] = tot[rt][bb];
        const uint32_t local = (uint32_t)__cvta_generic_to_shared(&tot[rt][bb]);
        for (int sp = 1; sp < (int)gridDim.y; ++sp) {
          uint32_t remote;
          float pv;
          asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(sp));
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(remote) : "memory");
          v[e] += pv;
        }
      }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (blockIdx.y != 0) return;
#pragma unroll
    for (int e = 0; e < EPI; ++e) {
      const int idx = tid + NWARP * 32 * e, rt = idx / SEQ, bb = idx - rt * SEQ;
      if (idx < ROWS * SEQ) tot[rt][bb] = v[e];
    }
  } else if (gridDim.y > 1) {
    // deterministic split reduction: every split parks its sums, the last CTA of
    // the row tile to arrive adds them in split order and runs the epilogue
    for (int idx = tid; idx < ROWS * SEQ; idx += NWARP * 32) {
      const int rt = idx / SEQ, bb = idx - rt * SEQ, row = blockIdx.x * ROWS + rt;
      if (row < a.n) __stcg(a.partial + ((int64_t)blockIdx.y * a.n + row) * SEQ + bb, tot[rt][bb]);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_cta = atomicAdd(&a.counter[blockIdx.x], 1) == (int)gridDim.y - 1;
    __syncthreads();
    if (!last_cta) return;
    __threadfence();
    for (int idx = tid; idx < ROWS * SEQ; idx += NWARP * 32) {
      const int rt = idx / SEQ, bb = idx - rt * SEQ, row = blockIdx.x * ROWS + rt;
      if (row < a.n) {
        float v = 0.f;
        for (int sp = 0; sp < (int)gridDim.y; ++sp) v += __ldcg(a.partial + ((int64_t)sp * a.n + row) * SEQ + bb);
        tot[rt][bb] = v;
      }
    }
    if (tid == 0) a.counter[blockIdx.x] = 0;  // ready for the next launch
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < EPI; ++e) {
    const int idx = tid + NWARP * 32 * e, rt = idx / SEQ, bb = idx - rt * SEQ;
    const int row = blockIdx.x * ROWS + rt;
    if (idx < ROWS * SEQ && row < a.n && bb < a.m) {
      const int rr = rt % 16;
      const float rn = a.norm_w ? rnorm[bb] : 1.f;
      float v = tot[rt][bb] * rn;
      if (a.bias) v += bias_v[e];
      if (a.swiglu) {
        if ((rr & 1) == 0) {  // rows 2i (gate) and 2i+1 (up)
          float up = tot[rt + 1][bb] * rn;
          if (a.bias) up += bias_u[e];
          a.y[(int64_t)bb * a.ldy + row / 2] = (v / (1.0f + expf(-v))) * up;
        }
      } else {
        if (a.residual) v = v + res_v[e];
        a.y[(int64_t)bb * a.ldy + row] = v;
      }
    }
  }
}

}  // namespace

extern "C" int cv3_decode_gemv_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_gemv_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_gemv_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return 0;
}

extern "C" int cv3_q8_decode_gemv_mma(const float* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q,
                                      const uint16_t* scales, int64_t n, int64_t kp, const float* bias,
                                      const float* residual, const float* norm_w, float eps, int swiglu, float* y,
                                      int64_t ldy, int64_t splits, float* workspace, int64_t workspace_floats,
                                      int* counters, void* stream) {
  CV3_REQUIRE(m >= 1 && m <= MAXSEQ, CV3_ERR_VALUE, "q8_decode_gemv_mma: 1..32 rows per call (got %lld)", (long long)m);
  const int nb = m <= MAXB ? 1 : (m <= 2 * MAXB ? 2 : 4);  // 8-sequence column blocks
  const int seq = MAXB * nb;
  CV3_REQUIRE(n > 0 && k > 0 && k % 64 == 0 && kp == k, CV3_ERR_VALUE,
              "q8_decode_gemv_mma: K must be a multiple of 64 with no padding (K %lld, padded %lld)", (long long)k,
              (long long)kp);
  CV3_REQUIRE(k <= 64 * NWARP * 10 && n < (1LL << 30), CV3_ERR_VALUE, "q8_decode_gemv_mma: K up to 5120");
  CV3_REQUIRE(ldx >= k && ldx % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)q & 15) == 0, CV3_ERR_VALUE,
              "q8_decode_gemv_mma: x rows and the payload must be 16-byte aligned");
  CV3_REQUIRE(swiglu ? (n % 2 == 0 && ldy >= n / 2 && !residual) : ldy >= n, CV3_ERR_VALUE,
              "q8_decode_gemv_mma: bad output layout");
  CV3_REQUIRE(!norm_w || ((uintptr_t)norm_w & 15) == 0, CV3_ERR_VALUE, "q8_decode_gemv_mma: norm weight alignment");
  CV3_REQUIRE(splits >= 1 && splits <= 16, CV3_ERR_VALUE, "q8_decode_gemv_mma: 1..16 K splits");
  const int ngroups = (int)(k / 64);
  const int gsplit = (ngroups + (int)splits - 1) / (int)splits;
  const int nsplit = (ngroups + gsplit - 1) / gsplit;
  // big matrices with K <= 1024: 32-row CTAs (one wave on 148 SMs for 9728 rows); else 16
  const bool wide = n >= 4096 && (ngroups + (int)splits - 1) / (int)splits <= NWARP * 2;
  const int rows = wide ? 32 : 16;
  const int tiles = (int)((n + rows - 1) / rows);
  const bool cluster = nsplit > 1 && nsplit <= 8;  // portable cluster size
  CV3_REQUIRE(!norm_w || nsplit == 1 || cluster, CV3_ERR_VALUE,
              "q8_decode_gemv_mma: a fused RMSNorm takes at most 8 K splits (one cluster)");
  if (nsplit > 1 && !cluster) {
    CV3_REQUIRE(workspace && counters && workspace_floats >= (int64_t)nsplit * n * seq, CV3_ERR_VALUE,
                "q8_decode_gemv_mma: more than 8 K splits need a workspace of splits*n*8*ceil(m/8) floats "
                "(m > 16: 32) and zeroed counters (one per %d-row tile)", rows);
  }
  MmaArgs a{x, ldx, (int)m, (int)k, q, scales, (int)n, bias, residual, y, ldy, norm_w, eps, swiglu,
            gsplit, workspace, counters, cluster ? 1 : 0};
  const int smem = (seq + (norm_w ? 1 : 0)) * 64 * gsplit * 4;
  // the kernel's static shared memory: warp partials and totals per (row, sequence), sums of squares
  const int static_smem = (NWARP + 1) * rows * seq * 4 + NWARP * seq * 4 + 2 * seq * 4 + 64;
  CV3_REQUIRE(smem + static_smem <= 226 * 1024 && (nb == 1 || gsplit <= NWARP * 4), CV3_ERR_VALUE,
              "q8_decode_gemv_mma: %lld rows x %d columns per CTA do not fit in shared memory: split K", (long long)m,
              64 * gsplit);
  dim3 grid((unsigned)tiles, (unsigned)nsplit);
  cudaStream_t st = cv3::as_stream(stream);
  void (*fn)(MmaArgs);
  const bool short_k = gsplit <= NWARP * 2;
  if (nb == 1) fn = wide ? q8_gemv_mma_kernel<2, 2, 1> : (short_k ? q8_gemv_mma_kernel<1, 2, 1> : q8_gemv_mma_kernel<1, 10, 1>);
  else if (nb == 2) fn = wide ? q8_gemv_mma_kernel<2, 2, 2> : (short_k ? q8_gemv_mma_kernel<1, 2, 2> : q8_gemv_mma_kernel<1, 4, 2>);
  else fn = wide ? q8_gemv_mma_kernel<2, 2, 4> : (short_k ? q8_gemv_mma_kernel<1, 2, 4> : q8_gemv_mma_kernel<1, 4, 4>);
  if (smem > 48 * 1024) {
    int rc = cv3::allow_smem((const void*)fn, smem);
    if (rc) return rc;
  }
  if (!cluster)
    return cv3::check_launch("q8_decode_gemv_mma", cv3::launch_dep(fn, grid, dim3(NWARP * 32), (size_t)smem, st, a));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NWARP * 32);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cv3::dependent_launch_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)nsplit;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cv3::check_launch("q8_decode_gemv_mma", cudaLaunchKernelEx(&cfg, fn, a));
}

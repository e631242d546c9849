// Device sampler of the speech LM: one decode step's token choice per sequence,
// with the reference's semantics and its random stream.
//
// Per sequence b (one CTA), as cv3cpu/models/llm.py does per step
// (generate :107-123, _sample :125-149, nucleus_sampling :37-49):
//   logp   = log_softmax(logits)                     (ops.py:90-93)
//   scores = logp, stop ids masked while fewer than min_len tokens were made
//            (only speech_token_size, or all 200 with strict_min_len)
//   probs  = softmax(scores)                          (ops.py:84-87)
//   order  = stable argsort of -probs; take entries while their running
//            float64 sum is < top_p, at most top_k;  p = those, float64,
//            p /= p.sum();  top = order[rng.choice(n, p=p)]
//   if top occurs >= win_size * tau_r times among the last win_size tokens:
//            scores[top] = -inf; p = softmax(scores) as float64, p /= p.sum();
//            top = rng.choice(len(p), p=p)
//   a stop id ends the sequence (not recorded); so does reaching max_len.
//
// The random stream is numpy's Generator(PCG64) bit for bit: the 128-bit
// state and increment live on the device ([b][4] uint64: state hi, lo, inc
// hi, lo, as numpy's bit_generator.state holds them), each draw steps the LCG
// and outputs XSL-RR, random() = (draw >> 11) * 2^-53, and choice(n, p) is
// cdf = cumsum(p) (sequential), cdf /= cdf[-1], searchsorted(cdf, random(),
// 'right').  float32 and float64 sums follow numpy's pairwise summation (eight
// accumulators per block of <= 128, halving above), sequential cumulative
// sums stay sequential, so every value that does not pass through exp is
// computed in the reference's order; exp itself is CUDA's (numpy's float32
// exp rounds differently in the last place), so probabilities can differ from
// the reference's by an ulp.
#include "common.cuh"

namespace {

constexpr int ST = 1024, SW = ST / 32;
constexpr int KMAX = 32;  // largest top_k

struct SampleArgs {
  const float* logits;
  int vocab, sts;  // sts: speech_token_size, first of the 200 stop ids
  const int* min_len;
  const int* max_len;
  int strict;
  double top_p, tau_r;
  int top_k, win;
  uint64_t* rng;  // [batch][4]
  int64_t* next_ids;
  int* pos;
  int* lens;
  int64_t* history;
  int64_t hist_stride;
  int* count;
  int* done;
  float* logp_out;
};

__device__ __forceinline__ uint64_t rotr64(uint64_t x, unsigned r) { return (x >> r) | (x << ((64u - r) & 63u)); }

// numpy PCG64: step the 128-bit LCG, then XSL-RR output; random() keeps the top 53 bits
__device__ double pcg_next_double(unsigned __int128& state, unsigned __int128 inc) {
  const unsigned __int128 mult = ((unsigned __int128)0x2360ED051FC65DA4ull << 64) | 0x4385DF649FCCF645ull;
  state = state * mult + inc;
  const uint64_t hi = (uint64_t)(state >> 64), lo = (uint64_t)state;
  const uint64_t out = rotr64(hi ^ lo, (unsigned)(state >> 122));
  return (double)(out >> 11) * (1.0 / 9007199254740992.0);
}

// numpy's pairwise summation (one thread): < 8 terms in order; <= 128 terms with eight
// interleaved accumulators ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) then the tail in order;
// above that the two halves (split at a multiple of 8) summed separately and added.
// numpy recurses; this walks the same tree with an explicit stack (device recursion would
// need more than the default per-thread stack).
template <typename T>
__device__ T np_pairwise_leaf(const T* a, int n) {
  if (n < 8) {
    T r = (T)0;
    for (int i = 0; i < n; ++i) r += a[i];
    return r;
  }
  T r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = a[j];
  int i = 8;
  for (; i < n - (n % 8); i += 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] += a[i + j];
  T res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; ++i) res += a[i];
  return res;
}

__device__ __forceinline__ int np_half(int m) { return m / 2 - (m / 2) % 8; }

template <typename T>
__device__ T np_pairwise(const T* a, int n) {
  constexpr int DEPTH = 16;  // halvings to reach <= 128 terms: 7 for n <= 10240 (the launcher's limit)
  int off[DEPTH], len[DEPTH], stage[DEPTH];
  T left[DEPTH];
  int sp = 0;
  off[0] = 0;
  len[0] = n;
  stage[0] = 0;
  while (true) {
    const int o = off[sp], m = len[sp];
    if (m <= 128 || sp == DEPTH - 1) {
      T v = np_pairwise_leaf(a + o, m);
      while (true) {  // hand the value up until a left half completes
        if (sp == 0) return v;
        --sp;
        if (stage[sp] == 0) {
          left[sp] = v;
          stage[sp] = 1;
          const int m2 = np_half(len[sp]);
          off[sp + 1] = off[sp] + m2;
          len[sp + 1] = len[sp] - m2;
          stage[sp + 1] = 0;
          ++sp;
          break;
        }
        v = left[sp] + v;
      }
    } else {
      stage[sp] = 0;
      off[sp + 1] = o;
      len[sp + 1] = np_half(m);
      stage[sp + 1] = 0;
      ++sp;
    }
  }
}

constexpr int MAX_LEAVES = 256;  // n <= 10240 (the launcher's limit): leaves of > 64 terms, <= 160

// numpy's pairwise sum of a[0..n) by the whole block, bit-identical to np_pairwise:
// thread 0 lists the tree's leaves (blocks of <= 128 terms) left to right, the block
// sums them in parallel with the eight-accumulator rule, and thread 0 adds the leaf
// sums up the same tree.  Returns the sum to every thread.
template <typename T>
__device__ T np_pairwise_block(const T* a, int n, T* leafsum, int* leafoff, int* leaflen, int* nleaves, T* out) {
  constexpr int DEPTH = 16;  // n <= 10240: at most 9 levels
  if (threadIdx.x == 0) {
    int off[DEPTH], len[DEPTH], sp = 0, nl = 0;
    off[0] = 0;
    len[0] = n;
    while (sp >= 0) {  // pre-order with the right half pushed first: leaves in order
      const int o = off[sp], m = len[sp];
      --sp;
      if (m <= 128) {
        leafoff[nl] = o;
        leaflen[nl] = m;
        ++nl;
      } else {
        const int m2 = np_half(m);
        off[++sp] = o + m2;
        len[sp] = m - m2;
        off[++sp] = o;
        len[sp] = m2;
      }
    }
    *nleaves = nl;
  }
  __syncthreads();
  const int nl = *nleaves;
  for (int l = threadIdx.x; l < nl; l += blockDim.x) leafsum[l] = np_pairwise_leaf(a + leafoff[l], leaflen[l]);
  __syncthreads();
  if (threadIdx.x == 0) {
    // post-order walk of the same tree, a leaf's sum taken from leafsum in order
    int len[DEPTH], stage[DEPTH];
    T left[DEPTH];
    int sp = 0, leaf = 0;
    len[0] = n;
    stage[0] = 0;
    bool done = false;
    while (!done) {
      const int m = len[sp];
      if (m <= 128) {
        T v = leafsum[leaf++];
        while (true) {  // hand the value up until a left half completes
          if (sp == 0) {
            *out = v;
            done = true;
            break;
          }
          --sp;
          if (stage[sp] == 0) {
            left[sp] = v;
            stage[sp] = 1;
            len[sp + 1] = len[sp] - np_half(len[sp]);
            stage[sp + 1] = 0;
            ++sp;
            break;
          }
          v = left[sp] + v;
        }
      } else {
        stage[sp] = 0;
        len[sp + 1] = np_half(m);
        stage[sp + 1] = 0;
        ++sp;
      }
    }
  }
  __syncthreads();
  return *out;
}

// first index whose cumulative share exceeds u: searchsorted(cdf / cdf[-1], u, 'right')
__device__ int search_right(const double* cdf, int n, double u) {
  const double last = cdf[n - 1];
  int lo = 0, hi = n;  // answer in [lo, hi]
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (cdf[mid] / last > u) hi = mid;
    else lo = mid + 1;
  }
  return min(lo, n - 1);
}

__device__ __forceinline__ bool before(float v, int i, float w, int j) { return v > w || (v == w && i < j); }

struct SumScratch {  // shared memory of np_pairwise_block
  float leaf_f[MAX_LEAVES];
  double leaf_d[MAX_LEAVES];
  int off[MAX_LEAVES], len[MAX_LEAVES];
  int nleaves;
  float out_f;
  double out_d;
};

// softmax of src into dst (max, exp(x - max), numpy-order float32 sum, divide)
__device__ void softmax_block(const float* src, float* dst, int V, float* red, SumScratch& ss) {
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += ST) m = fmaxf(m, src[i]);
  m = block_max(m, red);
  for (int i = threadIdx.x; i < V; i += ST) dst[i] = expf(src[i] - m);
  __syncthreads();
  const float s = np_pairwise_block(dst, V, ss.leaf_f, ss.off, ss.len, &ss.nleaves, &ss.out_f);
  for (int i = threadIdx.x; i < V; i += ST) dst[i] = dst[i] / s;
  __syncthreads();
}

__global__ void __launch_bounds__(ST) sample_select_kernel(SampleArgs a) {
  extern __shared__ double smd[];
  const int V = a.vocab;
  double* cdf = smd;                                 // [V] float64 (top-k: float working copy)
  float* lp = reinterpret_cast<float*>(smd + V);     // [V] log-probabilities, then the scores
  float* pr = lp + V;                                // [V] probabilities
  float* work = reinterpret_cast<float*>(cdf);
  __shared__ float red[32];
  __shared__ SumScratch ss;
  __shared__ float candv[SW][KMAX];
  __shared__ int candi[SW][KMAX];
  __shared__ float topv[KMAX];
  __shared__ int topi[KMAX];
  __shared__ int s_top, s_rep;
  __shared__ double nuc[2][KMAX];  // thread 0's nucleus weights and cumulative sums
  dep_wait();
  dep_release();
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (a.done[b]) return;
  const int cnt = a.count[b];
  if (cnt >= a.max_len[b]) {  // the reference's loop has run max_len times
    if (tid == 0) a.done[b] = 1;
    return;
  }
  // -- log_softmax (ops.py:90-93): z = x - max; logp = z - log(sum(exp(z))) ------------------
  const float* x = a.logits + (int64_t)b * V;
  float m = -INFINITY;
  for (int i = tid; i < V; i += ST) m = fmaxf(m, x[i]);
  m = block_max(m, red);
  for (int i = tid; i < V; i += ST) {
    const float z = x[i] - m;
    lp[i] = z;
    pr[i] = expf(z);
  }
  __syncthreads();
  const float lse = logf(np_pairwise_block(pr, V, ss.leaf_f, ss.off, ss.len, &ss.nleaves, &ss.out_f));
  for (int i = tid; i < V; i += ST) {
    const float v = lp[i] - lse;
    lp[i] = v;
    if (a.logp_out) a.logp_out[(int64_t)b * V + i] = v;
  }
  __syncthreads();
  // -- stop ids masked below min_len, probabilities ---------------------------------------------
  if (cnt < a.min_len[b]) {
    if (a.strict) {
      for (int i = a.sts + tid; i < min(a.sts + 200, V); i += ST) lp[i] = -INFINITY;
    } else if (tid == 0 && a.sts < V) {
      lp[a.sts] = -INFINITY;
    }
  }
  __syncthreads();
  softmax_block(lp, pr, V, red, ss);
  // -- top-k by (probability desc, index asc): each warp its chunk, then a 32-way merge -------
  const int K = min(a.top_k, V);
  for (int i = tid; i < V; i += ST) work[i] = pr[i];
  __syncthreads();
  {
    const int chunk = (V + SW - 1) / SW;
    const int c0 = warp * chunk, c1 = min(V, c0 + chunk);
    for (int r = 0; r < K; ++r) {
      float bv = -2.f;
      int bi = 0x7FFFFFFF;
      for (int i = c0 + lane; i < c1; i += 32) {
        const float v = work[i];
        if (v >= 0.f && before(v, i, bv, bi)) {
          bv = v;
          bi = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (before(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        candv[warp][r] = bv;
        candi[warp][r] = bi;
        if (bv >= 0.f) work[bi] = -1.f;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  if (warp == 0) {
    int ptr = 0;
    for (int r = 0; r < K; ++r) {
      float bv = ptr < K ? candv[lane][ptr] : -2.f;
      int bi = ptr < K ? candi[lane][ptr] : 0x7FFFFFFF;
      if (bv < 0.f) {
        bv = -2.f;
        bi = 0x7FFFFFFF;
      }
      const int mine = lane;
      int owner = mine;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const int ow = __shfl_xor_sync(0xffffffffu, owner, o);
        if (before(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
          owner = ow;
        }
      }
      if (lane == owner) ++ptr;
      if (lane == 0) {
        topv[r] = bv;
        topi[r] = bi;
      }
    }
  }
  __syncthreads();
  // -- nucleus draw and the repetition test (thread 0) -----------------------------------------
  if (tid == 0) {
    uint64_t* rs = a.rng + 4 * (int64_t)b;
    unsigned __int128 state = ((unsigned __int128)rs[0] << 64) | rs[1];
    const unsigned __int128 inc = ((unsigned __int128)rs[2] << 64) | rs[3];
    double cum = 0.0;
    int n = 0;
    for (int i = 0; i < K; ++i) {
      if (cum >= a.top_p) break;
      cum += (double)topv[i];
      ++n;
    }
    n = max(n, 1);
    double* p = nuc[0];
    double* c = nuc[1];
    for (int i = 0; i < n; ++i) p[i] = (double)topv[i];
    const double s = np_pairwise(p, n);
    double acc = 0.0;
    for (int i = 0; i < n; ++i) {
      acc += p[i] / s;
      c[i] = acc;
    }
    const int j = search_right(c, n, pcg_next_double(state, inc));
    const int top = min(max(topi[j], 0), V - 1);  // (always in range for finite logits)
    int rep = 0;
    const int64_t* hist = a.history + (int64_t)b * a.hist_stride;
    for (int i = max(0, cnt - a.win); i < cnt; ++i) rep += hist[i] == top;
    s_top = top;
    s_rep = (double)rep >= (double)a.win * a.tau_r;
    rs[0] = (uint64_t)(state >> 64);
    rs[1] = (uint64_t)state;
  }
  __syncthreads();
  if (s_rep) {
    // resample from the whole distribution with the pick removed
    if (tid == 0) lp[s_top] = -INFINITY;
    __syncthreads();
    softmax_block(lp, pr, V, red, ss);
    for (int i = tid; i < V; i += ST) cdf[i] = (double)pr[i];
    __syncthreads();
    const double s = np_pairwise_block(cdf, V, ss.leaf_d, ss.off, ss.len, &ss.nleaves, &ss.out_d);
    for (int i = tid; i < V; i += ST) cdf[i] = cdf[i] / s;
    __syncthreads();
    if (tid == 0) {
      double acc = 0.0;  // cumsum: sequential by definition; loads run ahead of the chain
      for (int i = 0; i < V; i += 8) {
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = i + j < V ? cdf[i + j] : 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i + j < V) {
            acc += v[j];
            cdf[i + j] = acc;
          }
      }
      uint64_t* rs = a.rng + 4 * (int64_t)b;
      unsigned __int128 state = ((unsigned __int128)rs[0] << 64) | rs[1];
      const unsigned __int128 inc = ((unsigned __int128)rs[2] << 64) | rs[3];
      s_top = search_right(cdf, V, pcg_next_double(state, inc));
      rs[0] = (uint64_t)(state >> 64);
      rs[1] = (uint64_t)state;
    }
    __syncthreads();
  }
  // -- record the token, or end the sequence on a stop id ----------------------------------------
  if (tid == 0) {
    const int top = s_top;
    if (top >= a.sts && top < a.sts + 200) {
      a.done[b] = 1;
    } else {
      if (cnt < a.hist_stride) a.history[(int64_t)b * a.hist_stride + cnt] = top;
      a.count[b] = cnt + 1;
      a.next_ids[b] = top;
      a.pos[b] += 1;
      a.lens[b] += 1;
      if (cnt + 1 >= a.max_len[b] || cnt + 1 >= a.hist_stride) a.done[b] = 1;
    }
  }
}

}  // namespace

extern "C" int cv3_sample_select(const float* logits, int64_t batch, int64_t vocab, int64_t speech_token_size,
                                 const int* min_len, const int* max_len, int strict_min_len, double top_p,
                                 int64_t top_k, int64_t win_size, double tau_r, uint64_t* rng_state,
                                 int64_t* next_ids, int* pos, int* lens, int64_t* history, int64_t hist_stride,
                                 int* count, int* done, float* logp_out, void* stream) {
  CV3_REQUIRE(batch >= 0 && vocab > 0 && vocab <= 10240 && speech_token_size >= 0, CV3_ERR_VALUE,
              "sample_select: vocabulary of 1..10240 entries");
  CV3_REQUIRE(top_k >= 1 && top_k <= KMAX && top_p > 0.0 && win_size >= 0, CV3_ERR_VALUE,
              "sample_select: top_k in 1..%d, top_p > 0, win_size >= 0", KMAX);
  CV3_REQUIRE(min_len && max_len && rng_state && next_ids && pos && lens && history && count && done &&
                  hist_stride > 0,
              CV3_ERR_VALUE, "sample_select: state arrays required");
  if (batch == 0) return CV3_OK;
  const int smem = (int)(vocab * 8 + 2 * vocab * 4);
  int rc = cv3::allow_smem((const void*)sample_select_kernel, smem);
  if (rc) return rc;
  SampleArgs a{logits, (int)vocab, (int)speech_token_size, min_len, max_len, strict_min_len, top_p, tau_r,
               (int)top_k, (int)win_size, rng_state, next_ids, pos, lens, history, hist_stride, count, done,
               logp_out};
  return cv3::check_launch("sample_select", cv3::launch_dep(sample_select_kernel, dim3((unsigned)batch), dim3(ST),
                                                            (size_t)smem, cv3::as_stream(stream), a));
}

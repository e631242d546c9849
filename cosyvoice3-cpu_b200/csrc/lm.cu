// Qwen2 decode-step kernels (cv3cpu/models/qwen2.py:139-179, cv3cpu/models/llm.py:112-121).
//
// Positions, cache lengths and token ids live in device memory so a whole
// decode step -- every layer, the head and the next input's embedding -- is a
// fixed sequence of launches that a CUDA graph replays without the host.
//
// KV cache layout: k/v [seq][kv_head][cap][head_dim] fp32 (cv3cpu/models/qwen2.py:74-121
// keeps (kv_head, cap, head_dim) per layer; here all sequences of a batch are
// stacked and the capacity is reserved up front).
#include <algorithm>

#include "tc_common.cuh"

__device__ int g_attn_err = 0;  // 1: a staged key/value copy did not land in time (cv3_decode_attention_status)

namespace {

using cv3tc::bulk_load;
using cv3tc::mbar_expect_tx;
using cv3tc::mbar_init;
using cv3tc::mbar_wait;

// rows r of qkv [R][(H + 2Hk) * D]: sequence seq[r] at position pos[r].
// q -> qout[r][H][D] rotated; k rotated and v copied into the caches.
__global__ void rope_qkv_append_kernel(const float* __restrict__ qkv, int64_t ldq, const float* __restrict__ cosT,
                                       const float* __restrict__ sinT, const int* __restrict__ seq,
                                       const int* __restrict__ pos, int heads, int kv_heads, int d,
                                       float* __restrict__ qout, float* __restrict__ kc, float* __restrict__ vc,
                                       int64_t cap) {
  dep_wait();
  dep_release();
  const int r = blockIdx.x;
  const int slot = blockIdx.y;  // [0, H) q heads, [H, H+Hk) k heads, [H+Hk, H+2Hk) v heads
  const int e = threadIdx.x;
  if (e >= d) return;
  const int p = pos[r], s = seq[r];
  const bool in_cache = p >= 0 && p < cap;  // a position past the cache is not stored (the host checks first)
  const float* row = qkv + (int64_t)r * ldq;
  if (slot < heads + kv_heads) {
    const float* x = row + (int64_t)slot * d;
    const int half = d / 2;
    const float rot = e < half ? -x[e + half] : x[e - half];
    const int pt = in_cache ? p : 0;  // (tables cover the cache's positions)
    const float c = cosT[(int64_t)pt * d + e], sn = sinT[(int64_t)pt * d + e];
    const float v = __fadd_rn(__fmul_rn(x[e], c), __fmul_rn(rot, sn));  // x*cos + rotate_half(x)*sin
    if (slot < heads) {
      qout[((int64_t)r * heads + slot) * d + e] = v;
    } else if (in_cache) {
      const int hk = slot - heads;
      kc[(((int64_t)s * kv_heads + hk) * cap + p) * d + e] = v;
    }
  } else if (in_cache) {
    const int hk = slot - heads - kv_heads;
    vc[(((int64_t)s * kv_heads + hk) * cap + p) * d + e] = row[(int64_t)slot * d + e];
  }
}

constexpr int AT = 256;
constexpr int DM = 64;
constexpr int HPG = 8;       // most query heads sharing one kv head (Qwen2-0.5B: 7)
constexpr int PG = AT / 16;  // key groups of the V pass (16 lanes x float4 per group)

// One CTA per (sequence, kv head, HC query heads of that group): the query heads
// of a group are spread over hpg / HC CTAs, each reading the group's cached
// key/value rows (the repeats hit L2).  HC is the smallest of 1, 2, 4, 8 whose
// grid fits one CTA per SM (measured at 8 sequences: 1 head per CTA beats 2 and
// 7; at 32 sequences 1 head per CTA would need four waves).  A head's arithmetic
// does not depend on HC.  Scores: one key per
// thread (its 256-byte row as 16 independent float4 loads) against the CTA's
// heads.  Softmax: one warp per head.  V pass: 16 key groups x 16 lanes of
// float4 dims, eight keys' value loads in flight per group, per-group partial
// sums reduced in a fixed order.  Same arithmetic as ops.sdpa with no mask
// (cv3cpu/ops.py:284-300): scores of the scaled query, exp(s - max), sum, then
// P.V / sum.
// ROPE: q is the raw qkv projection (rows ldq apart); every CTA rotates its
// query heads and its kv head's key (half-split RoPE at pos[b], rounded as
// cv3_rope_qkv_append does) and takes that key and the value for position pos[b]
// from shared memory; the first CTA of the group also appends them to the cache.
// So RoPE, the cache append and attention are one launch, and no CTA reads a
// cache row another CTA of the launch writes.
// STAGING (ROPE only): the cached rows [0, pos[b]) were written at earlier steps
// and pos[b] three or more launches back, all complete before this launch's CTAs
// start (every kernel of the chain releases its successor only after its own
// dependency wait).  So before the wait, bulk copies bring up to `kmax` of those
// key and value rows into shared memory, overlapping the qkv projection; after
// the wait the position is read again and the staged rows are used only if it is
// unchanged (else every row is read from global memory).  Every key's dot product
// takes its float4 columns rotated by the row index (conflict-free banks for the
// staged rows), wherever the row is read from, so a score does not depend on how
// many rows were staged (the staging budget varies with the cache capacity and HC).
template <bool ROPE, int HC>
__global__ void __launch_bounds__(AT)
decode_attention_kernel(const float* __restrict__ q, int64_t ldq, const float* __restrict__ cosT,
                        const float* __restrict__ sinT, const int* __restrict__ pos, float* kc, float* vc,
                        const int* __restrict__ lens, int heads, int kv_heads, int64_t cap, float scale,
                        float* __restrict__ out, int kmax, int64_t kv_off) {
  extern __shared__ float sc[];  // [HC][cap] scores, then probabilities; staged K, V rows at kv_off
  __shared__ float4 qs[HC][DM / 4];
  __shared__ float4 knew[DM / 4], vnew[DM / 4];
  __shared__ float4 part[PG][HC][DM / 4];
  __shared__ float stat[HC];
  __shared__ __align__(8) uint64_t kvbar;
  const int g = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* kb = kc + ((int64_t)b * kv_heads + g) * cap * DM;
  const float* vb = vc + ((int64_t)b * kv_heads + g) * cap * DM;
  float4* sk = reinterpret_cast<float4*>(sc + kv_off);  // [kmax][DM / 4]
  float4* sv = sk + (int64_t)kmax * (DM / 4);
  int ns = 0, p_pre = -1;  // rows staged in shared memory; the position they were staged for
  if (ROPE && kmax > 0) {
    p_pre = *(const volatile int*)(pos + b);
    ns = (int)min((int64_t)min(max(p_pre, 0), kmax), cap);
    if (tid == 0) {
      mbar_init(&kvbar, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      if (ns > 0) {
        mbar_expect_tx(&kvbar, (uint32_t)(2 * ns * DM * 4));
        constexpr int CH = 64;  // rows per copy (16 KB)
        for (int r = 0; r < ns; r += CH) {
          const uint32_t bytes = (uint32_t)(min(CH, ns - r) * DM * 4);
          bulk_load(sk + (int64_t)r * (DM / 4), kb + (int64_t)r * DM, bytes, &kvbar);
          bulk_load(sv + (int64_t)r * (DM / 4), vb + (int64_t)r * DM, bytes, &kvbar);
        }
      }
    }
  }
  if (threadIdx.x == 0) {
    // Warm L2 with the cached rows that are not staged while the previous kernel still
    // runs.  Only a hint: L2 is coherent, so even a stale length (read before the wait)
    // cannot change what the loads below see; the range stays inside the cache rows of
    // this (sequence, kv head).
    const int64_t rows = min((int64_t)max(*(const volatile int*)(lens + b), 0), cap) - ns;
    const uint32_t bytes = rows > 0 ? (uint32_t)(rows * DM * 4) : 0u;
    if (bytes >= 16) {
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(kb + (int64_t)ns * DM), "r"(bytes) : "memory");
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vb + (int64_t)ns * DM), "r"(bytes) : "memory");
    }
  }
  dep_wait();
  dep_release();
  const int hpg = heads / kv_heads;
  const int h0 = blockIdx.z * HC;            // this CTA's first query head within the group
  const int nh = min(HC, hpg - h0);          // >= 1: the grid covers ceil(hpg / HC) pairs
  const int m = (int)min((int64_t)lens[b], cap);
  int pnew = -1;  // position whose key and value come from shared memory
  if (ROPE) {
    const int p = pos[b];
    if (p != p_pre) ns = 0;  // not the position staged for: every row from global memory
    const bool in_cache = p >= 0 && p < cap;  // a position past the cache is not stored
    const int pt = in_cache ? p : 0;
    const float* row = q + (int64_t)b * ldq;
    for (int i = tid; i < (nh + 2) * DM; i += AT) {
      const int hh = i / DM, e = i - hh * DM;  // hh < nh: query head; nh: key; nh + 1: value
      const int slot = hh < nh ? g * hpg + h0 + hh : (hh == nh ? heads + g : heads + kv_heads + g);
      const float* x = row + (int64_t)slot * DM;
      float v = x[e];
      if (hh <= nh) {
        const float rot = e < DM / 2 ? -x[e + DM / 2] : x[e - DM / 2];
        v = __fadd_rn(__fmul_rn(v, cosT[(int64_t)pt * DM + e]), __fmul_rn(rot, sinT[(int64_t)pt * DM + e]));
      }
      if (hh < nh) {
        reinterpret_cast<float*>(&qs[hh][0])[e] = v * scale;
      } else {
        reinterpret_cast<float*>(hh == nh ? knew : vnew)[e] = v;
        if (in_cache && blockIdx.z == 0) (hh == nh ? kc : vc)[(((int64_t)b * kv_heads + g) * cap + p) * DM + e] = v;
      }
    }
    pnew = in_cache ? p : -1;
  } else {
    for (int i = tid; i < nh * (DM / 4); i += AT) {
      const int h = i / (DM / 4), c = i - h * (DM / 4);
      float4 v = reinterpret_cast<const float4*>(q + ((int64_t)b * heads + g * hpg + h0 + h) * DM)[c];
      v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
      qs[h][c] = v;
    }
  }
  // the staged rows (a copy issued before the wait lands even when it is not used)
  bool landed = true;
  if (ROPE && kmax > 0 && p_pre > 0 && min((int64_t)min(p_pre, kmax), cap) > 0) landed = mbar_wait(&kvbar, 0, &g_attn_err, 1);
  if (!__syncthreads_and(landed)) {
    if (tid == 0 && !landed) mbar_wait(&kvbar, 0, &g_attn_err, 1);  // once more (bounded) before leaving
    return;
  }
  for (int j = tid; j < m; j += AT) {
    float4 kr[DM / 4];
    const int rot = j & (DM / 4 - 1);  // float4 column c of kr holds column (c + rot) % 16
    if (j < ns) {
#pragma unroll
      for (int c = 0; c < DM / 4; ++c) kr[c] = sk[(int64_t)j * (DM / 4) + ((c + rot) & (DM / 4 - 1))];
    } else if (j == pnew) {
#pragma unroll
      for (int c = 0; c < DM / 4; ++c) kr[c] = knew[(c + rot) & (DM / 4 - 1)];
    } else {
      const float4* src = reinterpret_cast<const float4*>(kb + (int64_t)j * DM);
#pragma unroll
      for (int c = 0; c < DM / 4; ++c) kr[c] = src[(c + rot) & (DM / 4 - 1)];
    }
#pragma unroll
    for (int h = 0; h < HC; ++h) {
      if (h < nh) {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < DM / 4; ++c) {
          const float4 qq = qs[h][(c + rot) & (DM / 4 - 1)];
          s = fmaf(qq.x, kr[c].x, s);
          s = fmaf(qq.y, kr[c].y, s);
          s = fmaf(qq.z, kr[c].z, s);
          s = fmaf(qq.w, kr[c].w, s);
        }
        sc[h * cap + j] = s;
      }
    }
  }
  __syncthreads();
  if (warp < nh) {
    float* row = sc + warp * cap;
    float mx = -INFINITY;
    for (int j = lane; j < m; j += 32) mx = fmaxf(mx, row[j]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < m; j += 32) {
      const float p = expf(row[j] - mx);
      row[j] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    if (lane == 0) stat[warp] = sum;
  }
  __syncthreads();
  const int grp = tid / (DM / 4), l = tid % (DM / 4);
  float4 acc[HC];
#pragma unroll
  for (int h = 0; h < HC; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int VU = 8;  // value rows in flight per key group: one L2 round trip per VU keys
  for (int j = grp; j < m; j += VU * PG) {
    float4 v[VU];
#pragma unroll
    for (int u = 0; u < VU; ++u) {
      const int jj = j + u * PG;
      v[u] = jj >= m ? make_float4(0.f, 0.f, 0.f, 0.f)
                     : (jj < ns ? sv[(int64_t)jj * (DM / 4) + l]
                                : (jj == pnew ? vnew[l] : reinterpret_cast<const float4*>(vb + (int64_t)jj * DM)[l]));
    }
#pragma unroll
    for (int u = 0; u < VU; ++u) {
      if (j + u * PG < m) {
#pragma unroll
        for (int h = 0; h < HC; ++h) {
          if (h < nh) {
            const float p = sc[h * cap + j + u * PG];
            acc[h].x = fmaf(p, v[u].x, acc[h].x);
            acc[h].y = fmaf(p, v[u].y, acc[h].y);
            acc[h].z = fmaf(p, v[u].z, acc[h].z);
            acc[h].w = fmaf(p, v[u].w, acc[h].w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < HC; ++h)
    if (h < nh) part[grp][h][l] = acc[h];
  __syncthreads();
  for (int i = tid; i < nh * DM; i += AT) {
    const int h = i / DM, e = i - h * DM;
    float o = 0.f;
    for (int p = 0; p < PG; ++p) o += reinterpret_cast<const float*>(&part[p][h][0])[e];
    out[(int64_t)b * heads * DM + (int64_t)(g * hpg + h0 + h) * DM + e] = o / stat[h];
  }
}

// y[r][i] = silu(gu[r][i]) * gu[r][inter + i]   (qwen2.py:175-177, ops.py:30-31)
__global__ void swiglu_kernel(const float* __restrict__ gu, int64_t rows, int64_t inter, float* __restrict__ y) {
  const int64_t total = rows * inter;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / inter, c = i - r * inter;
    const float g = gu[r * 2 * inter + c], u = gu[r * 2 * inter + inter + c];
    y[i] = (g / (1.0f + expf(-g))) * u;
  }
}

// Greedy head: logp = log_softmax(logits) over the whole vocabulary
// (llm.py:114); token = first argmax of logp[:select] (stop ids masked);
// records the token, feeds it as the next input id and advances the position.
__global__ void __launch_bounds__(1024)
head_select_kernel(const float* __restrict__ logits, int64_t vocab, int64_t select, float* logp_out,
                   int64_t* __restrict__ next_ids, int* __restrict__ pos, int* __restrict__ lens,
                   int64_t* __restrict__ history, int64_t hist_stride, const int* __restrict__ step) {
  __shared__ float red[32];
  __shared__ float bv[32];
  __shared__ int bi[32];
  dep_wait();
  dep_release();
  const int b = blockIdx.x;
  const float* x = logits + (int64_t)b * vocab;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, x[i]);
  m = block_max(m, red);
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) s += expf(x[i] - m);
  s = block_sum(s, red);
  const float lse = logf(s);
  float best = -INFINITY;
  int besti = 0x7FFFFFFF;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float lp = (x[i] - m) - lse;
    if (logp_out) logp_out[(int64_t)b * vocab + i] = lp;
    if (i < select && (lp > best || (lp == best && i < besti))) { best = lp; besti = (int)i; }
  }
  // warp argmax, lowest index on ties
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { bv[wid] = best; bi[wid] = besti; }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = (blockDim.x + 31) / 32;
    float B = bv[0];
    int I = bi[0];
    for (int w = 1; w < nw; ++w)
      if (bv[w] > B || (bv[w] == B && bi[w] < I)) { B = bv[w]; I = bi[w]; }
    next_ids[b] = I;
    const int sn = step ? *step : 0;
    if (history && sn >= 0 && sn < hist_stride) history[(int64_t)b * hist_stride + sn] = I;  // full history: not kept
    pos[b] += 1;
    lens[b] += 1;
  }
}

__global__ void step_increment_kernel(int* step) {
  dep_wait();
  dep_release();
  if (threadIdx.x == 0 && blockIdx.x == 0) *step += 1;
}

}  // namespace

extern "C" int cv3_rope_qkv_append(const float* qkv, int64_t rows, int64_t ldq, const float* cos_table,
                                   const float* sin_table, const int* seq, const int* pos, int64_t heads,
                                   int64_t kv_heads, int64_t head_dim, float* q_out, float* k_cache, float* v_cache,
                                   int64_t cap, void* stream) {
  CV3_REQUIRE(rows >= 0 && heads > 0 && kv_heads > 0 && head_dim > 0 && head_dim <= 1024 && head_dim % 2 == 0,
              CV3_ERR_VALUE, "rope_qkv_append: bad shape");
  CV3_REQUIRE(ldq >= (heads + 2 * kv_heads) * head_dim, CV3_ERR_VALUE, "rope_qkv_append: ldq too small");
  if (rows == 0) return CV3_OK;
  dim3 grid((unsigned)rows, (unsigned)(heads + 2 * kv_heads));
  const int threads = ((int)head_dim + 31) / 32 * 32;
  return cv3::check_launch(
      "rope_qkv_append", cv3::launch_dep(rope_qkv_append_kernel, grid, dim3(threads), 0, cv3::as_stream(stream), qkv,
                                         ldq, cos_table, sin_table, seq, pos, (int)heads, (int)kv_heads,
                                         (int)head_dim, q_out, k_cache, v_cache, cap));
}

namespace {

int launch_decode_attention(bool rope, const float* q, int64_t ldq, const float* cos_table, const float* sin_table,
                            const int* pos, float* k_cache, float* v_cache, const int* lens, int64_t batch,
                            int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cap, float scale, float* out,
                            void* stream) {
  CV3_REQUIRE(batch >= 0 && heads > 0 && kv_heads > 0 && heads % kv_heads == 0, CV3_ERR_VALUE,
              "%lld query heads is not a multiple of %lld kv heads", (long long)heads, (long long)kv_heads);
  CV3_REQUIRE(head_dim == DM, CV3_ERR_UNSUPPORTED, "decode_attention: head_dim %lld (built for %d)",
              (long long)head_dim, DM);
  CV3_REQUIRE(heads / kv_heads <= HPG, CV3_ERR_UNSUPPORTED, "decode_attention: more than %d heads per kv head", HPG);
  const int64_t hpg = heads / kv_heads;
  // query heads per CTA: the fewest that keep the grid within one CTA per SM
  int HC = 8;
  for (int hc : {1, 2, 4}) {
    if (batch * kv_heads * ((hpg + hc - 1) / hc) <= cv3::sm_count()) {
      HC = hc;
      break;
    }
  }
  CV3_REQUIRE(cap > 0 && cap * 4 <= 150 * 1024, CV3_ERR_UNSUPPORTED, "decode_attention: cap too large");
  while (HC > 1 && HC * cap * 4 > 150 * 1024) HC /= 2;  // long caches: fewer heads per CTA, more waves
  // staged key/value rows (RoPE launches): as many as fit next to the scores in 200 KB
  const int64_t kv_off = (HC * cap + 3) / 4 * 4;  // floats, 16-byte aligned
  const int64_t kmax = rope ? std::min<int64_t>(cap, (200 * 1024 - kv_off * 4) / (2 * DM * 4)) : 0;
  const int64_t smem = kv_off * 4 + kmax * 2 * DM * 4;
  CV3_REQUIRE(((uintptr_t)q & 15) == 0 && ((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0,
              CV3_ERR_VALUE, "decode_attention: 16-byte aligned tensors required");
  if (batch == 0) return CV3_OK;
  using Fn = void (*)(const float*, int64_t, const float*, const float*, const int*, float*, float*, const int*, int,
                      int, int64_t, float, float*, int, int64_t);
  Fn fn;
  switch (HC) {
    case 1: fn = rope ? decode_attention_kernel<true, 1> : decode_attention_kernel<false, 1>; break;
    case 2: fn = rope ? decode_attention_kernel<true, 2> : decode_attention_kernel<false, 2>; break;
    case 4: fn = rope ? decode_attention_kernel<true, 4> : decode_attention_kernel<false, 4>; break;
    default: fn = rope ? decode_attention_kernel<true, 8> : decode_attention_kernel<false, 8>; break;
  }
  int rc = cv3::allow_smem((const void*)fn, (int)smem);
  if (rc) return rc;
  dim3 grid((unsigned)kv_heads, (unsigned)batch, (unsigned)((hpg + HC - 1) / HC));
  return cv3::check_launch("decode_attention",
                           cv3::launch_dep(fn, grid, dim3(AT), (size_t)smem, cv3::as_stream(stream), q, ldq,
                                           cos_table, sin_table, pos, k_cache, v_cache, lens, (int)heads,
                                           (int)kv_heads, cap, scale, out, (int)kmax, kv_off));
}

}  // namespace

extern "C" int cv3_decode_attention_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_attn_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

extern "C" int cv3_decode_attention(const float* q, const float* k_cache, const float* v_cache, const int* lens,
                                    int64_t batch, int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t cap,
                                    float scale, float* out, void* stream) {
  return launch_decode_attention(false, q, 0, nullptr, nullptr, nullptr, const_cast<float*>(k_cache),
                                 const_cast<float*>(v_cache), lens, batch, heads, kv_heads, head_dim, cap, scale, out,
                                 stream);
}

extern "C" int cv3_decode_rope_attention(const float* qkv, int64_t ldq, const float* cos_table,
                                         const float* sin_table, const int* pos, float* k_cache, float* v_cache,
                                         const int* lens, int64_t batch, int64_t heads, int64_t kv_heads,
                                         int64_t head_dim, int64_t cap, float scale, float* out, void* stream) {
  CV3_REQUIRE(ldq >= (heads + 2 * kv_heads) * head_dim && ldq % 4 == 0 && cos_table && sin_table && pos,
              CV3_ERR_VALUE, "decode_rope_attention: qkv rows of (heads + 2 kv_heads) * head_dim, tables, positions");
  return launch_decode_attention(true, qkv, ldq, cos_table, sin_table, pos, k_cache, v_cache, lens, batch, heads,
                                 kv_heads, head_dim, cap, scale, out, stream);
}

extern "C" int cv3_swiglu(const float* gate_up, int64_t rows, int64_t inter, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && inter > 0, CV3_ERR_VALUE, "swiglu: bad shape");
  if (rows == 0) return CV3_OK;
  int64_t grid = (rows * inter + 255) / 256;
  if (grid > cv3::sm_count() * 16) grid = cv3::sm_count() * 16;
  swiglu_kernel<<<(unsigned)grid, 256, 0, cv3::as_stream(stream)>>>(gate_up, rows, inter, y);
  return cv3::check_launch("swiglu");
}

extern "C" int cv3_head_select(const float* logits, int64_t batch, int64_t vocab, int64_t select, float* logp_out,
                               int64_t* next_ids, int* pos, int* lens, int64_t* history, int64_t hist_stride,
                               int* step, void* stream) {
  CV3_REQUIRE(batch >= 0 && vocab > 0 && select > 0 && select <= vocab, CV3_ERR_VALUE, "head_select: bad shape");
  if (batch == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  int rc = cv3::check_launch("head_select", cv3::launch_dep(head_select_kernel, dim3((unsigned)batch), dim3(1024), 0,
                                                            st, logits, vocab, select, logp_out, next_ids, pos, lens,
                                                            history, hist_stride, step));
  if (rc || !step) return rc;
  return cv3::check_launch("step_increment", cv3::launch_dep(step_increment_kernel, dim3(1), dim3(32), 0, st, step));
}

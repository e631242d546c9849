// Persistent greedy decode of the Qwen2 speech LM: all decode steps of a batch
// of <= 8 sequences in one cooperative launch (one CTA per SM).
//
// Per token (cv3cpu/models/qwen2.py:139-179, llm.py:114-136) and layer, five
// phases separated by grid barriers:
//   A  qkv = RMSNorm(h, ln1) . Wqkv^T + b, RoPE on q/k, k/v appended to the
//      cache at pos  -- one CTA per 64-row head block, so RoPE (which pairs
//      dims d and d +- 32 of a head) needs nothing from other CTAs;
//   B  GQA attention over the cache -- one CTA per (sequence, kv head);
//   C  h += attn . Wo^T;
//   D  act = silu(gate) * up from the interleaved gate|up GEMV on RMSNorm(h, ln2);
//   E  h += act . Wdown^T.
// Then F: logits = RMSNorm(h, norm_f) . Whead^T and G: per sequence
// log_softmax, first argmax over the speech tokens, bookkeeping and the
// embedding of the chosen token into h for the next step.
//
// GEMV layout: a warp takes two weight rows at a time, lanes run along K in
// 16-byte pieces (each warp load is two contiguous 512-byte row segments),
// the activations of all sequences come from shared memory (staged, and
// RMS-normalised where the op says so), per-piece partial dots are scaled by
// the piece's fp16 group scale and the lanes are reduced with shuffles.  No
// split-K workspace, no atomics.  Data one CTA writes and another reads in a
// later phase goes through L2 (st.cg / ld.cg), never a possibly stale L1.
// The grid barrier is a counter + generation word with bounded waits; on
// expiry the kernel records an error (cv3_decode_status) and every CTA leaves.
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int NT = 256, NW = NT / 32;
constexpr int HD = 64;                 // head dim
constexpr int HPG = 8;                 // most query heads per kv head
constexpr int PG = 16;                 // key groups of the attention V pass
constexpr unsigned long long WAIT_NS = 2000000000ull;

__device__ int g_dec_err = 0;

struct Params {
  cv3_decode_params p;
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Grid-wide barrier over per-CTA flags: a CTA publishes how many barriers it
// has reached (after a fence, so its writes are visible first) and warp 0 of
// every CTA polls all flags -- no same-address atomics to serialise.  false
// (after recording an error) if the barrier could not complete in time.
__device__ __noinline__ bool grid_sync(uint32_t* flags, uint32_t& gen) {
  __shared__ int ok_s;
  __syncthreads();
  const uint32_t target = gen + 1;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    if (lane == 0) {
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(&flags[blockIdx.x]) = target;
    }
    const unsigned long long t0 = now_ns();
    int ok = 1;
    while (true) {
      bool all = true;
      for (int i = lane; i < (int)gridDim.x; i += 32)
        all &= (int)(*reinterpret_cast<volatile uint32_t*>(&flags[i]) - target) >= 0;
      if (__all_sync(0xffffffffu, all)) break;
      const bool stop = *reinterpret_cast<volatile int*>(&g_dec_err) != 0 || now_ns() - t0 > WAIT_NS;
      if (__any_sync(0xffffffffu, stop)) {
        if (lane == 0) atomicCAS(&g_dec_err, 0, 1);
        ok = 0;
        break;
      }
    }
    __threadfence();
    if (lane == 0) ok_s = ok;
  }
  __syncthreads();
  gen = target;
  return ok_s != 0;
}

__device__ __forceinline__ void widen16(const int4 w, float f[16]) {
  const uint32_t words[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u,
                             (uint32_t)w.z ^ 0x80808080u, (uint32_t)w.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int b = 0; b < 4; ++b) f[4 * i + b] = __int_as_float(__byte_perm(words[i], 0x4B000000u, 0x7440u | b)) - 8388736.0f;
}

// RB weight rows (row < 0: absent) against MB activation rows xs[m][0..K) in
// shared memory, U 16-byte pieces per lane and row (K <= U * 512).  All of the
// warp's weight loads are issued before any arithmetic (one memory round trip
// per batch), and each activation chunk is read once for all RB rows.  Every
// lane ends with the full sums y[r][m].
template <int MB, int RB, int U>
__device__ __forceinline__ void gemv_batch(const float* xs, int K, const int8_t* W, const uint16_t* S,
                                           const int (&rows)[RB], float (&y)[RB][MB]) {
  const int lane = threadIdx.x & 31;
  const int np = K >> 4, ks = K >> 6;
  int4 w[RB][U];
  float sc[RB][U];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = lane + 32 * u;
      const bool in = rows[r] >= 0 && p < np;
      w[r][u] = in ? ld_stream16(W + (int64_t)rows[r] * K + 16 * p) : make_int4(0, 0, 0, 0);
      sc[r][u] = in ? h2f(S[(int64_t)rows[r] * ks + (p >> 2)]) : 0.f;
    }
  float acc[RB][MB];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[r][m] = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int p = lane + 32 * u;
    if (p < np) {
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        const float4* xv = reinterpret_cast<const float4*>(xs + m * K + 16 * p);
        float x[16];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 t = xv[v];
          x[4 * v] = t.x;
          x[4 * v + 1] = t.y;
          x[4 * v + 2] = t.z;
          x[4 * v + 3] = t.w;
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          float f[16];
          widen16(w[r][u], f);
          float d = 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) d = fmaf(f[j], x[j], d);
          acc[r][m] = fmaf(d, sc[r][u], acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      y[r][m] = v;
    }
}

// L2 prefetch of rows [r0, r1) of a q8 matrix with K columns (payload + scales),
// issued by lane 0 of warp 0: the next phase's weights stream in while this one
// (and the barrier) runs.
__device__ __forceinline__ void prefetch_rows(const int8_t* W, const uint16_t* S, int r0, int r1, int K) {
  if (threadIdx.x != 0 || r0 >= r1) return;
  const char* a = reinterpret_cast<const char*>(W + (int64_t)r0 * K);
  int64_t n = (int64_t)(r1 - r0) * K;  // a multiple of 64 bytes
  while (n > 0) {
    const uint32_t c = (uint32_t)(n > (1 << 20) ? (1 << 20) : n);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(c) : "memory");
    a += c;
    n -= c;
  }
  const char* sa = reinterpret_cast<const char*>(S + (int64_t)r0 * (K >> 6));
  const uint32_t sn = (uint32_t)((int64_t)(r1 - r0) * (K >> 6) * 2);
  const uintptr_t lo = reinterpret_cast<uintptr_t>(sa) & ~uintptr_t(15);
  const uint32_t len = (uint32_t)(((reinterpret_cast<uintptr_t>(sa) + sn + 15) & ~uintptr_t(15)) - lo);
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"(len) : "memory");
}

// xs[m][0..K) = src rows (ld.cg), optionally RMS-normalised with weight w:
// (x * (1/sqrt(mean(x^2) + eps))) * w (the fused decode GEMV's order).
template <int MB>
__device__ void stage_rows(float* xs, float* rn, const float* src, int B, int K, const float* w, float eps) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int k4 = K >> 2;
  // eight independent 16-byte loads in flight per thread per round
  for (int i0 = tid; i0 < MB * k4; i0 += 8 * NT) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * NT;
      const int m = i / k4;
      v[u] = (i < MB * k4 && m < B) ? ldcg4(src + (int64_t)m * K + 4 * (i - m * k4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * NT < MB * k4) reinterpret_cast<float4*>(xs)[i0 + u * NT] = v[u];
  }
  __syncthreads();
  if (!w) return;
  for (int m = warp; m < MB; m += NW) {
    float s = 0.f;
    for (int c = lane; c < K; c += 32) {
      const float v = xs[m * K + c];
      s += v * v;
    }
    s = warp_sum(s);
    if (lane == 0) rn[m] = 1.0f / sqrtf(s / (float)K + eps);
  }
  __syncthreads();
  for (int i = tid; i < MB * k4; i += NT) {
    const int m = i / k4, c4 = i - m * k4;
    const float r = rn[m];
    const float4 w4 = reinterpret_cast<const float4*>(w)[c4];
    float4 v = reinterpret_cast<float4*>(xs)[i];
    v.x = (v.x * r) * w4.x;
    v.y = (v.y * r) * w4.y;
    v.z = (v.z * r) * w4.z;
    v.w = (v.w * r) * w4.w;
    reinterpret_cast<float4*>(xs)[i] = v;
  }
  __syncthreads();
}

struct Layer {
  const int8_t* qkv_q;
  const uint16_t* qkv_s;
  const float* qkv_b;
  const float* ln1;
  const int8_t* o_q;
  const uint16_t* o_s;
  const int8_t* gu_q;
  const uint16_t* gu_s;
  const float* ln2;
  const int8_t* dn_q;
  const uint16_t* dn_s;
  float* kc;
  float* vc;
};

__device__ __forceinline__ Layer layer_at(const cv3_decode_params& p, int i) {
  const void* const* t = p.layers + (int64_t)i * CV3_DECODE_LAYER_FIELDS;
  Layer L;
  L.qkv_q = (const int8_t*)t[0];
  L.qkv_s = (const uint16_t*)t[1];
  L.qkv_b = (const float*)t[2];
  L.ln1 = (const float*)t[3];
  L.o_q = (const int8_t*)t[4];
  L.o_s = (const uint16_t*)t[5];
  L.gu_q = (const int8_t*)t[6];
  L.gu_s = (const uint16_t*)t[7];
  L.ln2 = (const float*)t[8];
  L.dn_q = (const int8_t*)t[9];
  L.dn_s = (const uint16_t*)t[10];
  L.kc = (float*)t[11];
  L.vc = (float*)t[12];
  return L;
}

// rows [r0, r1) of a q8 matrix (K <= U * 512 columns) against the staged rows,
// round-robin over the warps, RB rows per warp batch; `emit(r, m, y)` gets every
// (row, sequence) result once (lane m of the warp that owns the row)
template <int MB, int RB, int U, typename Emit>
__device__ __forceinline__ void gemv_rows(const float* xs, int K, const int8_t* W, const uint16_t* S, int r0, int r1,
                                          int B, Emit emit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int base = r0 + warp; base < r1; base += NW * RB) {
    int rows[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) rows[r] = base + NW * r < r1 ? base + NW * r : -1;
    float y[RB][MB];
    gemv_batch<MB, RB, U>(xs, K, W, S, rows, y);
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
      for (int m = 0; m < MB; ++m)
        if (lane == m && m < B && rows[r] >= 0) emit(rows[r], m, y[r][m]);
  }
}

// contiguous row range of CTA `c` when `rows` rows are shared by G CTAs
__device__ __forceinline__ void share(int rows, int c, int G, int& r0, int& r1) {
  const int per = (rows + G - 1) / G;
  r0 = min(rows, c * per);
  r1 = min(rows, r0 + per);
}

template <int MB>
__global__ void __launch_bounds__(NT, 1) decode_steps_kernel(const Params P) {
  const cv3_decode_params& p = P.p;
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  __shared__ float rn[8];
  __shared__ float red[32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, hid = p.hidden, H = p.heads, Hk = p.kv_heads, inter = p.inter;
  const int hpg = H / Hk;
  uint32_t gen = 0;
  const int step0 = __ldcg(p.step);

  for (int s = 0; s < p.steps; ++s) {
    for (int li = 0; li < p.n_layers; ++li) {
      const Layer L = layer_at(p, li);
      // ---- A: qkv GEMV (+bias), RoPE, cache append: one CTA per head block --------
      {
        int c0, c1;
        share(hid, cta, G, c0, c1);
        prefetch_rows(L.o_q, L.o_s, c0, c1, H * HD);  // phase C's rows
      }
      if (cta < H + 2 * Hk) {
        const int u = cta;
        float* xs = sm;
        float* ys = sm + MB * hid;  // [MB][64]
        stage_rows<MB>(xs, rn, p.h, B, hid, L.ln1, p.eps);
        gemv_rows<MB, 8, 2>(xs, hid, L.qkv_q, L.qkv_s, u * HD, u * HD + HD, B, [&](int r, int m, float y) {
          ys[m * HD + (r - u * HD)] = y + L.qkv_b[r];
        });
        __syncthreads();
        for (int i = tid; i < B * HD; i += NT) {
          const int m = i / HD, e = i - m * HD;
          const int ps = __ldcg(p.pos + m);
          if (ps < 0 || ps >= p.cap) {  // past the cache: record, write nothing
            if (e == 0) atomicCAS(&g_dec_err, 0, 2);
            continue;
          }
          const float x = ys[m * HD + e];
          if (u < H + Hk) {
            const float rot = e < HD / 2 ? -ys[m * HD + e + HD / 2] : ys[m * HD + e - HD / 2];
            const float c = p.cos_table[(int64_t)ps * HD + e], sn = p.sin_table[(int64_t)ps * HD + e];
            const float v = __fadd_rn(__fmul_rn(x, c), __fmul_rn(rot, sn));
            if (u < H) __stcg(p.q + ((int64_t)m * H + u) * HD + e, v);
            else __stcg(L.kc + (((int64_t)m * Hk + (u - H)) * p.cap + ps) * HD + e, v);
          } else {
            __stcg(L.vc + (((int64_t)m * Hk + (u - H - Hk)) * p.cap + ps) * HD + e, x);
          }
        }
      }
      if (!grid_sync(p.barrier, gen)) return;

      // ---- B: attention, one CTA per (sequence, kv head) -----------------------------
      {
        int d0, d1;
        share(inter, cta, G, d0, d1);
        prefetch_rows(L.gu_q, L.gu_s, 2 * d0, 2 * d1, hid);  // phase D's rows
      }
      if (cta < B * Hk) {
        const int b = cta / Hk, g = cta - b * Hk;
        const int m = (int)min((int64_t)__ldcg(p.lens + b), p.cap);
        float4* qs = smem4;                                    // [HPG][16]
        float4* part = smem4 + HPG * (HD / 4);                 // [PG][HPG][16]
        float* stat = reinterpret_cast<float*>(part + PG * HPG * (HD / 4));  // [HPG]
        float* sc = stat + HPG;                                // [hpg][cap]
        for (int i = tid; i < hpg * (HD / 4); i += NT) {
          const int h = i / (HD / 4), c = i - h * (HD / 4);
          float4 v = ldcg4(p.q + ((int64_t)b * H + g * hpg + h) * HD + 4 * c);
          v.x *= p.scale; v.y *= p.scale; v.z *= p.scale; v.w *= p.scale;
          qs[h * (HD / 4) + c] = v;
        }
        __syncthreads();
        const float* kb = L.kc + ((int64_t)b * Hk + g) * p.cap * HD;
        const float* vb = L.vc + ((int64_t)b * Hk + g) * p.cap * HD;
        for (int j = tid; j < m; j += NT) {
          float4 kr[HD / 4];
#pragma unroll
          for (int c = 0; c < HD / 4; ++c) kr[c] = ldcg4(kb + (int64_t)j * HD + 4 * c);
          for (int h = 0; h < hpg; ++h) {
            float sv = 0.f;
#pragma unroll
            for (int c = 0; c < HD / 4; ++c) {
              const float4 qq = qs[h * (HD / 4) + c];
              sv = fmaf(qq.x, kr[c].x, sv);
              sv = fmaf(qq.y, kr[c].y, sv);
              sv = fmaf(qq.z, kr[c].z, sv);
              sv = fmaf(qq.w, kr[c].w, sv);
            }
            sc[h * p.cap + j] = sv;
          }
        }
        __syncthreads();
        if (warp < hpg) {
          float* row = sc + warp * p.cap;
          float mx = -INFINITY;
          for (int j = lane; j < m; j += 32) mx = fmaxf(mx, row[j]);
          mx = warp_max(mx);
          float sum = 0.f;
          for (int j = lane; j < m; j += 32) {
            const float e = expf(row[j] - mx);
            row[j] = e;
            sum += e;
          }
          sum = warp_sum(sum);
          if (lane == 0) stat[warp] = sum;
        }
        __syncthreads();
        const int grp = tid / (HD / 4), l = tid % (HD / 4);
        float4 acc[HPG];
#pragma unroll
        for (int h = 0; h < HPG; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = grp; j0 < m; j0 += 4 * PG) {
          float4 vv[4];  // four value rows in flight
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j0 + u * PG;
            vv[u] = j < m ? ldcg4(vb + (int64_t)j * HD + 4 * l) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j0 + u * PG;
            if (j < m) {
#pragma unroll
              for (int h = 0; h < HPG; ++h) {
                if (h < hpg) {
                  const float pr = sc[h * p.cap + j];
                  acc[h].x = fmaf(pr, vv[u].x, acc[h].x);
                  acc[h].y = fmaf(pr, vv[u].y, acc[h].y);
                  acc[h].z = fmaf(pr, vv[u].z, acc[h].z);
                  acc[h].w = fmaf(pr, vv[u].w, acc[h].w);
                }
              }
            }
          }
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h)
          if (h < hpg) part[(grp * HPG + h) * (HD / 4) + l] = acc[h];
        __syncthreads();
        for (int i = tid; i < hpg * HD; i += NT) {
          const int h = i / HD, e = i - h * HD;
          float o = 0.f;
          for (int q = 0; q < PG; ++q) o += reinterpret_cast<const float*>(&part[(q * HPG + h) * (HD / 4)])[e];
          __stcg(p.attn + (int64_t)b * H * HD + (int64_t)(g * hpg + h) * HD + e, o / stat[h]);
        }
      }
      if (!grid_sync(p.barrier, gen)) return;

      // ---- C: h += attn . Wo^T ----------------------------------------------------------
      {
        int e0, e1;
        share(hid, cta, G, e0, e1);
        prefetch_rows(L.dn_q, L.dn_s, e0, e1, inter);  // phase E's rows
        int r0, r1;
        share(hid, cta, G, r0, r1);
        if (r0 < r1) {
          stage_rows<MB>(sm, rn, p.attn, B, H * HD, nullptr, 0.f);
          gemv_rows<MB, 1, 2>(sm, H * HD, L.o_q, L.o_s, r0, r1, B, [&](int r, int m, float y) {
            float* hp = p.h + (int64_t)m * hid + r;
            __stcg(hp, y + __ldcg(hp));
          });
        }
      }
      if (!grid_sync(p.barrier, gen)) return;

      // ---- D: act = silu(gate) * up on RMSNorm(h, ln2) ----------------------------------
      {
        if (li + 1 < p.n_layers) {
          if (cta < H + 2 * Hk) {
            const Layer N = layer_at(p, li + 1);
            prefetch_rows(N.qkv_q, N.qkv_s, cta * HD, cta * HD + HD, hid);  // next layer's phase A
          }
        } else {
          int f0, f1;
          share(p.vocab, cta, G, f0, f1);
          prefetch_rows(p.head_q, p.head_s, f0, f1, hid);  // phase F
        }
        int q0, q1;  // gate/up pairs of this CTA
        share(inter, cta, G, q0, q1);
        if (q0 < q1) {
          stage_rows<MB>(sm, rn, p.h, B, hid, L.ln2, p.eps);
          // four (gate, up) pairs per warp batch
          for (int base = q0 + warp; base < q1; base += NW * 4) {
            int rows[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int pr = base + NW * j;
              rows[2 * j] = pr < q1 ? 2 * pr : -1;
              rows[2 * j + 1] = pr < q1 ? 2 * pr + 1 : -1;
            }
            float y[8][MB];
            gemv_batch<MB, 8, 2>(sm, hid, L.gu_q, L.gu_s, rows, y);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int m = 0; m < MB; ++m)
                if (lane == m && m < B && rows[2 * j] >= 0) {
                  const float gt = y[2 * j][m];
                  __stcg(p.act + (int64_t)m * inter + rows[2 * j] / 2, (gt / (1.0f + expf(-gt))) * y[2 * j + 1][m]);
                }
          }
        }
      }
      if (!grid_sync(p.barrier, gen)) return;

      // ---- E: h += act . Wdown^T ---------------------------------------------------------
      {
        int r0, r1;
        share(hid, cta, G, r0, r1);
        if (r0 < r1) {
          stage_rows<MB>(sm, rn, p.act, B, inter, nullptr, 0.f);
          gemv_rows<MB, 1, 10>(sm, inter, L.dn_q, L.dn_s, r0, r1, B, [&](int r, int m, float y) {
            float* hp = p.h + (int64_t)m * hid + r;
            __stcg(hp, y + __ldcg(hp));
          });
        }
      }
      if (!grid_sync(p.barrier, gen)) return;
    }

    // ---- F: logits = RMSNorm(h, norm_f) . Whead^T ------------------------------------------
    {
      if (s + 1 < p.steps && cta < H + 2 * Hk) {
        const Layer N = layer_at(p, 0);
        prefetch_rows(N.qkv_q, N.qkv_s, cta * HD, cta * HD + HD, hid);  // next step's first phase
      }
      int r0, r1;
      share(p.vocab, cta, G, r0, r1);
      if (r0 < r1) {
        stage_rows<MB>(sm, rn, p.h, B, hid, p.final_norm, p.eps);
        gemv_rows<MB, 8, 2>(sm, hid, p.head_q, p.head_s, r0, r1, B,
                      [&](int r, int m, float y) { __stcg(p.logits + (int64_t)m * p.vocab + r, y); });
      }
    }
    if (!grid_sync(p.barrier, gen)) return;

    // ---- G: greedy pick, bookkeeping, next input embedding (one CTA per sequence) ---------
    if (cta < B) {
      const int b = cta;
      float* x = sm;  // this sequence's logits, staged once (eight loads in flight per thread)
      {
        const float* src = p.logits + (int64_t)b * p.vocab;
        for (int i0 = tid; i0 < p.vocab; i0 += 8 * NT) {
          float v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = i0 + u * NT < p.vocab ? __ldcg(src + i0 + u * NT) : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (i0 + u * NT < p.vocab) x[i0 + u * NT] = v[u];
        }
        __syncthreads();
      }
      float mx = -INFINITY;
      for (int i = tid; i < p.vocab; i += NT) mx = fmaxf(mx, x[i]);
      mx = block_max(mx, red);
      float sum = 0.f;
      for (int i = tid; i < p.vocab; i += NT) sum += expf(x[i] - mx);
      sum = block_sum(sum, red);
      const float lse = logf(sum);
      float best = -INFINITY;
      int besti = 0x7FFFFFFF;
      for (int i = tid; i < p.vocab; i += NT) {
        const float lp = (x[i] - mx) - lse;
        if (p.logp) __stcg(p.logp + (int64_t)b * p.vocab + i, lp);
        if (i < p.select && (lp > best || (lp == best && i < besti))) {
          best = lp;
          besti = i;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) {
          best = ov;
          besti = oi;
        }
      }
      __shared__ float bv[NW];
      __shared__ int bi[NW];
      __shared__ int pick;
      if (lane == 0) {
        bv[warp] = best;
        bi[warp] = besti;
      }
      __syncthreads();
      if (tid == 0) {
        float Bv = bv[0];
        int I = bi[0];
        for (int w = 1; w < NW; ++w)
          if (bv[w] > Bv || (bv[w] == Bv && bi[w] < I)) {
            Bv = bv[w];
            I = bi[w];
          }
        pick = I;
        __stcg(p.next_ids + b, (int64_t)I);
        if (step0 + s < p.hist_stride) __stcg(p.history + (int64_t)b * p.hist_stride + step0 + s, (int64_t)I);
        else atomicCAS(&g_dec_err, 0, 3);
        __stcg(p.pos + b, __ldcg(p.pos + b) + 1);
        __stcg(p.lens + b, __ldcg(p.lens + b) + 1);
      }
      __syncthreads();
      const int r = pick;
      const bool ok = r >= 0 && r < p.emb_rows;
      for (int c = tid; c < hid; c += NT) {
        float v = 0.f;
        if (ok) {
          if (!p.emb_scales) v = reinterpret_cast<const float*>(p.emb)[(int64_t)r * hid + c];
          else v = (float)reinterpret_cast<const int8_t*>(p.emb)[(int64_t)r * hid + c] *
                   h2f(p.emb_scales[(int64_t)r * (hid / 64) + c / 64]);
        }
        __stcg(p.h + (int64_t)b * hid + c, v);
      }
    }
    if (!grid_sync(p.barrier, gen)) return;
  }
  if (cta == 0 && tid == 0) __stcg(p.step, step0 + p.steps);
}

template <int MB>
int launch(const cv3_decode_params& pr, cudaStream_t st) {
  auto fn = decode_steps_kernel<MB>;
  const int64_t attn_smem = (int64_t)(HPG * (HD / 4) + PG * HPG * (HD / 4)) * 16 + HPG * 4 +
                            (int64_t)(pr.heads / pr.kv_heads) * pr.cap * 4;
  const int64_t x_smem =
      std::max((int64_t)MB * std::max(pr.hidden + HD, std::max(pr.inter, pr.heads * HD)), (int64_t)pr.vocab) * 4;
  const int64_t smem = std::max(attn_smem, x_smem);
  CV3_REQUIRE(smem <= 220 * 1024, CV3_ERR_UNSUPPORTED, "decode_steps: %lld bytes of shared memory needed",
              (long long)smem);
  int rc = cv3::allow_smem((const void*)fn, (int)smem);
  if (rc) return rc;
  int per_sm = 0;
  CV3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, NT, (size_t)smem));
  CV3_REQUIRE(per_sm >= 1, CV3_ERR_UNSUPPORTED, "decode_steps: kernel does not fit an SM");
  const int grid = cv3::sm_count();
  CV3_REQUIRE(grid >= pr.heads + 2 * pr.kv_heads && grid >= pr.batch * pr.kv_heads && grid >= pr.batch,
              CV3_ERR_UNSUPPORTED, "decode_steps: too few SMs for the head / attention units");
  CV3_CUDA(cudaMemsetAsync(pr.barrier, 0, (size_t)grid * sizeof(uint32_t), st));
  Params P{pr};
  void* args[] = {&P};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)fn, dim3(grid), dim3(NT), args, (size_t)smem, st);
  return cv3::check_launch("decode_steps", e);
}

}  // namespace

extern "C" int cv3_decode_steps(const cv3_decode_params* pr, void* stream) {
  CV3_REQUIRE(pr != nullptr, CV3_ERR_VALUE, "decode_steps: no parameters");
  const cv3_decode_params& p = *pr;
  CV3_REQUIRE(p.batch >= 1 && p.batch <= 8 && p.n_layers >= 1 && p.steps >= 0, CV3_ERR_VALUE,
              "decode_steps: 1..8 sequences, >= 1 layer");
  CV3_REQUIRE(p.head_dim == HD && p.heads % p.kv_heads == 0 && p.heads / p.kv_heads <= HPG, CV3_ERR_UNSUPPORTED,
              "decode_steps: head dim 64 and <= 8 query heads per kv head");
  CV3_REQUIRE(p.hidden % 64 == 0 && p.inter % 64 == 0 && p.hidden == p.heads * HD && p.hidden <= 1024 &&
                  p.inter <= 5120,
              CV3_ERR_UNSUPPORTED,
              "decode_steps: hidden (<= 1024) and intermediate (<= 5120) sizes must be multiples of 64");
  CV3_REQUIRE(p.vocab > 0 && p.select > 0 && p.select <= p.vocab && p.emb_rows > 0, CV3_ERR_VALUE,
              "decode_steps: bad head / embedding sizes");
  CV3_REQUIRE(p.layers && p.h && p.q && p.attn && p.act && p.logits && p.pos && p.lens && p.next_ids && p.history &&
                  p.step && p.barrier && p.head_q && p.head_s && p.emb && p.cos_table && p.sin_table && p.final_norm,
              CV3_ERR_VALUE, "decode_steps: missing pointer");
  if (p.steps == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  if (p.batch == 1) return launch<1>(p, st);
  if (p.batch == 2) return launch<2>(p, st);
  if (p.batch <= 4) return launch<4>(p, st);
  return launch<8>(p, st);
}

extern "C" int cv3_decode_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_dec_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_dec_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

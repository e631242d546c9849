// Persistent greedy decode of the Qwen2 speech LM (cv3cpu/models/qwen2.py:139-179,
// llm.py:112-121): every decode step of a batch of <= 8 sequences in one cooperative
// launch, one CTA per SM, with the int8 weights streamed into shared memory ahead of
// the layer-to-layer dependency chain.
//
// Why: a decode step reads 375 MB of int8 weights once and does little arithmetic on
// them, so its floor is the HBM stream (~57 us at 6.5 TB/s).  Launched as one kernel
// per linear, the step is instead a chain of ~120 dependent launches whose latency,
// not the bandwidth, sets the time.  Here the weights do not wait for the chain: each
// CTA owns fixed 16-row tiles of every matrix, and a producer warp copies the CTA's
// next tiles (cp.async.bulk, completion on an mbarrier) into a 7-slot ring while the
// consumer warps still work on earlier phases; a phase then only waits for its input
// vector, and its MMAs read weights that are already on chip.
//
// Per step and layer, five phases separated by completion counters in global memory
// (each CTA that worked on a phase adds one after its last item; a phase starts when
// the previous phase's counter reaches its target; counters only grow, the target of
// step t is (t + 1) * contributors, so nothing is ever reset):
//   A  qkv = RMSNorm(h, ln1) . Wqkv^T + b                     (16-row tiles)
//   B  attention per (sequence, kv head, 64-key chunk): RoPE of q and of the new key,
//      cache append, partial softmax (max, sum, unnormalised P.V) of the chunk
//   C  h1 = h + merge(chunks) . Wo^T                          (16-row tiles)
//   D  act = silu(gate) * up of RMSNorm(h1, ln2) . Wgu^T      (interleaved gate/up rows)
//   E  h = h1 + act . Wdown^T  -- 16-row tiles in K parts of <= 19 scale groups; the
//      last part of a tile to finish (a ticket per tile) adds the parts in order
// and per step F: logits = RMSNorm(h, norm) . Whead^T and G: per sequence log_softmax,
// first argmax over the speech tokens, bookkeeping and the chosen token's embedding
// as the next input.
//
// Tile arithmetic (tensor cores, mma.sync m16n8k16 f16 -> f32): A = 16 weight rows x
// 16 k, int8 made exact fp16 by placing the byte in the mantissa of 1024 (one byte
// permute and one packed subtraction per pair); B = 16 k x 8 sequences of the
// activations, scaled per sequence by a power of two into fp16 range and split into
// three fp16 parts (x = hi + mid + lo to beyond fp32 precision), done once per phase
// and kept in shared memory in fragment order.  Each 64-wide scale group's three
// partial sums are added small parts first, scaled by the group's fp16 scale and
// accumulated in fp32; warps split a tile's groups and their sums are added in a fixed
// order (deterministic).  The K order inside a 64-group is permuted the same way for
// both operands so that one 16-byte shared load per row and group feeds four k-steps.
//
// Every wait (ring slots, counters, prefetches) is bounded by %globaltimer; on expiry
// the kernel records an error (cv3_decode_status) and every CTA drains the copies it
// issued and leaves.
#include "common.cuh"

namespace {

constexpr int NCW = 8;                 // consumer warps
constexpr int NCT = NCW * 32;
constexpr int NT = NCT + 32;           // + one producer warp
constexpr int MAXB = 8;                // sequences: one MMA n-tile
constexpr int RT = 16;                 // weight rows per tile: one MMA m-tile
constexpr int HD = 64;                 // head dim
constexpr int KCH = 64;                // keys per attention chunk
constexpr int GMAX = 19;               // most scale groups per work item (K <= 1216)
constexpr int KS_MAX = 76;             // most scale groups per matrix row (K <= 4864)
constexpr int SLOT_W = RT * GMAX * 64; // 19,456 B of rows (row stride <= 1216)
constexpr int SLOT_S = RT * KS_MAX * 2;  // 2,432 B: a whole tile's fp16 scales
constexpr int SLOT_BYTES = SLOT_W + SLOT_S;  // 21,888 = 171 * 128
constexpr int NSLOT = 7;
constexpr int XF_GROUP = 3 * 4 * 32 * 8;     // bytes of split activations per scale group
constexpr int XF_BYTES = GMAX * XF_GROUP;    // 58,368
constexpr int RED_FLOATS = 2 * NCW * RT * MAXB;
constexpr unsigned long long WAIT_NS = 2000000000ull;
constexpr int PH_PER_LAYER = 5;

__device__ int g_ds_err = 0;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool failed() { return *reinterpret_cast<volatile int*>(&g_ds_err) != 0; }
__device__ __forceinline__ void fail_with(int code) { atomicCAS(&g_ds_err, 0, code); }

// ---------------------------------------------------------------------------
// mbarriers and bulk copies
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}

// true once the phase with this parity has completed; false after WAIT_NS (error set)
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int code) {
  const unsigned long long t0 = now_ns();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    if (done) return true;
    if (now_ns() - t0 > WAIT_NS || failed()) {
      fail_with(code);
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sa(dst)),
      "l"(src), "r"(bytes), "r"(sa(bar))
      : "memory");
}

// consumer-warps-only barrier (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// the same barrier, returning whether `v` held in every consumer thread: after a bounded
// wait each thread ran on its own, every thread takes the same branch (a named barrier
// that some consumer threads skip would never complete)
__device__ __forceinline__ bool csync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCT)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// completion counters
// ---------------------------------------------------------------------------

// thread 0 of the consumers: after every consumer's writes, publish one completion
__device__ __forceinline__ void signal(uint32_t* ctr) {
  __threadfence();
  atomicAdd(ctr, 1u);
}

// all consumers: wait until *ctr >= target (bounded), then see everything published before
__device__ __forceinline__ bool wait_count(const uint32_t* ctr, uint32_t target, int* ok_s) {
  if (threadIdx.x == 0) {
    const unsigned long long t0 = now_ns();
    int ok = 1;
    while ((int)(*reinterpret_cast<const volatile uint32_t*>(ctr) - target) < 0) {
      if (failed() || now_ns() - t0 > WAIT_NS) {
        fail_with(1);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *ok_s = ok;
  }
  csync();
  return *reinterpret_cast<volatile int*>(ok_s) != 0;
}

// ---------------------------------------------------------------------------
// the static work split
// ---------------------------------------------------------------------------

struct Mat {  // one q8 matrix as GEMV work items: tiles of 16 rows x parts of K
  const int8_t* q;
  const uint16_t* s;
  int tiles, k, parts, gp;  // gp: scale groups per part
  __device__ int items() const { return tiles * parts; }
};

__device__ __forceinline__ Mat make_mat(const void* q, const void* s, int rows, int k) {
  Mat m;
  m.q = static_cast<const int8_t*>(q);
  m.s = static_cast<const uint16_t*>(s);
  m.tiles = rows / RT;
  m.k = k;
  const int ks = k / 64;
  m.parts = (ks + GMAX - 1) / GMAX;
  m.gp = (ks + m.parts - 1) / m.parts;
  return m;
}

// items i of a phase with n items go to CTA (i + off) % G; this CTA's first item
__device__ __forceinline__ int first_item(int off, int G) { return (int)((blockIdx.x + G - (off % G)) % G); }

__device__ __forceinline__ int contributors(int n, int G) { return n < G ? n : G; }

// row stride of a tile's rows in a ring slot: K bytes padded to 64 mod 128 (conflict-free
// 16-byte reads of rows g and g + 1 by the lanes of a quarter warp)
__device__ __forceinline__ int row_stride(int kbytes) { return kbytes + ((64 - (kbytes & 127)) & 127); }

struct Layer {
  const int8_t *qkv_q, *o_q, *gu_q, *dn_q;
  const uint16_t *qkv_s, *o_s, *gu_s, *dn_s;
  const float *qkv_b, *ln1, *ln2;
  float *kc, *vc;
};

__device__ __forceinline__ Layer layer_at(const cv3_decode_params& p, int l) {
  const void* const* t = p.layers + (int64_t)l * CV3_DECODE_LAYER_FIELDS;
  Layer L;
  L.qkv_q = static_cast<const int8_t*>(t[0]);
  L.qkv_s = static_cast<const uint16_t*>(t[1]);
  L.qkv_b = static_cast<const float*>(t[2]);
  L.ln1 = static_cast<const float*>(t[3]);
  L.o_q = static_cast<const int8_t*>(t[4]);
  L.o_s = static_cast<const uint16_t*>(t[5]);
  L.gu_q = static_cast<const int8_t*>(t[6]);
  L.gu_s = static_cast<const uint16_t*>(t[7]);
  L.ln2 = static_cast<const float*>(t[8]);
  L.dn_q = static_cast<const int8_t*>(t[9]);
  L.dn_s = static_cast<const uint16_t*>(t[10]);
  L.kc = static_cast<float*>(const_cast<void*>(t[11]));
  L.vc = static_cast<float*>(const_cast<void*>(t[12]));
  return L;
}

struct Dims {
  int B, hid, H, Hk, inter, qkv_rows, vocab_pad, nch, G;
  int off_a, off_b, off_c, off_d, off_e, off_f, off_g;
};

__device__ __forceinline__ Dims dims_of(const cv3_decode_params& p) {
  Dims d;
  d.B = p.batch;
  d.hid = p.hidden;
  d.H = p.heads;
  d.Hk = p.kv_heads;
  d.inter = p.inter;
  d.qkv_rows = (p.heads + 2 * p.kv_heads) * HD;
  d.vocab_pad = (p.vocab + RT - 1) / RT * RT;
  d.nch = (int)((p.cap + KCH - 1) / KCH);
  d.G = gridDim.x;
  // rotate each phase's items over the CTAs so the small phases do not all land on the
  // same CTAs (their ring slots fill evenly)
  d.off_a = 0;
  d.off_b = d.G / 3;
  d.off_c = d.G / 2;
  d.off_d = 0;
  d.off_e = (2 * d.G) / 3;
  d.off_f = 0;
  d.off_g = d.G / 4;
  return d;
}

// ---------------------------------------------------------------------------
// the producer: this CTA's weight items, in consumption order, into the ring
// ---------------------------------------------------------------------------

struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
};

__device__ __forceinline__ bool produce_mat(const Ring& r, const Mat& m, int off, int G, uint32_t& fill) {
  const int ks = m.k / 64;
  for (int i = first_item(off, G); i < m.items(); i += G) {
    const int tile = i / m.parts, part = i - tile * m.parts;
    const int g0 = part * m.gp, ng = min(m.gp, ks - g0);
    const int kb = 64 * ng, stride = row_stride(kb);
    const int slot = fill % NSLOT;
    const uint32_t use = fill / NSLOT;
    if (!mbar_wait(&r.empty[slot], (use & 1) ^ 1, 4)) return false;
    uint8_t* dst = r.base + slot * SLOT_BYTES;
    const uint32_t sbytes = (uint32_t)(RT * ks * 2);
    mbar_expect_tx(&r.full[slot], (uint32_t)(RT * kb) + sbytes);
    const int8_t* src = m.q + (int64_t)tile * RT * m.k + 64 * g0;
#pragma unroll 1
    for (int row = 0; row < RT; ++row) bulk_g2s(dst + row * stride, src + (int64_t)row * m.k, (uint32_t)kb, &r.full[slot]);
    bulk_g2s(dst + SLOT_W, m.s + (int64_t)tile * RT * ks, sbytes, &r.full[slot]);
    ++fill;
  }
  return true;
}

// ---------------------------------------------------------------------------
// consumers: activation staging (split fp16 fragments) and the tile MMAs
// ---------------------------------------------------------------------------

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

// 2^e as a float for e in [-126, 127]
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// The power of two that brings max|x| of a row into [2^14, 2^15) (fp16 keeps 2^15 * 2).
__device__ __forceinline__ int row_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  const int e = ((__float_as_int(amax) >> 23) & 0xFF) - 127;  // floor(log2) for normals
  int s = 14 - e;
  return s > 126 ? 126 : (s < -126 ? -126 : s);
}

// Sixteen values of one sequence (K positions 16c .. 16c+15 of scale group G) into the
// fragment-ordered split store: xf[G][part][kstep][lane] = uint2 (b0, b1) of lane g*4+c.
__device__ __forceinline__ void split16(uint8_t* xf, int G, int g, int c, const float v[16], float scale) {
  uint2* base = reinterpret_cast<uint2*>(xf + G * XF_GROUP);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = v[4 * j + e] * scale;  // exact: a power of two
    uint32_t w[3][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float a = x[2 * h], b = x[2 * h + 1];
      const uint32_t hi = f2h2(a, b);
      float ha, hb;
      h22f(hi, ha, hb);
      const float ra = a - ha, rb = b - hb;
      const uint32_t mid = f2h2(ra, rb);
      float ma, mb;
      h22f(mid, ma, mb);
      const uint32_t lo = f2h2(ra - ma, rb - mb);
      w[0][h] = hi;
      w[1][h] = mid;
      w[2][h] = lo;
    }
#pragma unroll
    for (int pp = 0; pp < 3; ++pp) base[(pp * 4 + j) * 32 + g * 4 + c] = make_uint2(w[pp][0], w[pp][1]);
  }
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bytes (b0, b1) of a word of int8 (sign-flipped to unsigned) as exact fp16 (b0 - 128, b1 - 128)
__device__ __forceinline__ uint32_t i8pair(uint32_t u, uint32_t sel) {
  const uint32_t h = __byte_perm(u, 0x64646464u, sel);  // (1024 + u0, 1024 + u1)
  __half2 v = *reinterpret_cast<const __half2*>(&h);
  const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
  v = __hsub2(v, bias);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One work item: the consumer warps split its ng scale groups; per-warp sums of rows
// (g, g + 8) x sequences (2c, 2c + 1) go to red[warp] (fixed-order reduction later).
__device__ __forceinline__ void tile_mma(const uint8_t* slot, int ng, int kbytes, int ks, int g0, const uint8_t* xf,
                                         float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int stride = row_stride(kbytes);
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + SLOT_W);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int G = warp; G < ng; G += NCW) {
    const int4 w0 = *reinterpret_cast<const int4*>(slot + g * stride + 64 * G + 16 * c);
    const int4 w1 = *reinterpret_cast<const int4*>(slot + (g + 8) * stride + 64 * G + 16 * c);
    const float s0 = h2f(sc[g * ks + g0 + G]), s1 = h2f(sc[(g + 8) * ks + g0 + G]);
    const uint32_t u0[4] = {(uint32_t)w0.x ^ 0x80808080u, (uint32_t)w0.y ^ 0x80808080u,
                            (uint32_t)w0.z ^ 0x80808080u, (uint32_t)w0.w ^ 0x80808080u};
    const uint32_t u1[4] = {(uint32_t)w1.x ^ 0x80808080u, (uint32_t)w1.y ^ 0x80808080u,
                            (uint32_t)w1.z ^ 0x80808080u, (uint32_t)w1.w ^ 0x80808080u};
    const uint2* xb = reinterpret_cast<const uint2*>(xf + G * XF_GROUP);
    float t[3][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t A0 = i8pair(u0[j], 0x4140u);  // row g,     k 2c, 2c+1
      const uint32_t A1 = i8pair(u1[j], 0x4140u);  // row g + 8, k 2c, 2c+1
      const uint32_t A2 = i8pair(u0[j], 0x4342u);  // row g,     k 2c+8, 2c+9
      const uint32_t A3 = i8pair(u1[j], 0x4342u);  // row g + 8, k 2c+8, 2c+9
#pragma unroll
      for (int pp = 0; pp < 3; ++pp) {
        const uint2 b = xb[(pp * 4 + j) * 32 + lane];
        mma_f16(t[pp], A0, A1, A2, A3, b.x, b.y);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = (t[2][e] + t[1][e]) + t[0][e];
      acc[e] = fmaf(v, e < 2 ? s0 : s1, acc[e]);
    }
  }
  float* rw = red + warp * RT * MAXB;
  rw[g * MAXB + 2 * c] = acc[0];
  rw[g * MAXB + 2 * c + 1] = acc[1];
  rw[(g + 8) * MAXB + 2 * c] = acc[2];
  rw[(g + 8) * MAXB + 2 * c + 1] = acc[3];
}

// Row sum of the warps' partials for (row r, sequence b) in warp order, unscaled.
__device__ __forceinline__ float red_sum(const float* red, int r, int b) {
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < NCW; ++w) v += red[w * RT * MAXB + r * MAXB + b];
  return v;
}

// Stage RMSNorm(src) (norm_w non-null) or src, columns [k0, k0 + kw) of each of the B
// rows (row stride ld), as split fp16 fragments; one warp per sequence.  Rows >= B are
// zeros.  inv_scale[b] receives 2^-e of sequence b's fp16 scaling.
__device__ void stage_rows(uint8_t* xf, const float* src, int64_t ld, int B, int K, int k0, int kw, const float* norm_w,
                           float eps, float* inv_scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = kw / 64, units = ng * 4;  // 16-value units per row
  const int b = warp;                      // NCW == MAXB
  constexpr int UMAX = (GMAX * 4 + 31) / 32;  // units per lane (<= 3)
  float v[UMAX][16];
  if (b < B) {
    const float* row = src + (int64_t)b * ld + k0;
#pragma unroll
    for (int u = 0; u < UMAX; ++u) {
      const int id = lane + 32 * u;
      if (id < units) {
        const int G = id >> 2, c = id & 3;
        const float4* p4 = reinterpret_cast<const float4*>(row + 64 * G + 16 * c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 t = __ldcg(p4 + q);
          v[u][4 * q] = t.x;
          v[u][4 * q + 1] = t.y;
          v[u][4 * q + 2] = t.z;
          v[u][4 * q + 3] = t.w;
        }
      }
    }
    if (norm_w) {
      // RMSNorm over the whole row (kw == K here): x * (1 / sqrt(mean(x^2) + eps)) * w
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < UMAX; ++u)
        if (lane + 32 * u < units) {
          float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int e = 0; e < 16; ++e) s4[e & 3] = fmaf(v[u][e], v[u][e], s4[e & 3]);
          ss += (s4[0] + s4[1]) + (s4[2] + s4[3]);
        }
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss / (float)K + eps);
#pragma unroll
      for (int u = 0; u < UMAX; ++u) {
        const int id = lane + 32 * u;
        if (id < units) {
          const int G = id >> 2, c = id & 3;
          const float4* w4 = reinterpret_cast<const float4*>(norm_w + k0 + 64 * G + 16 * c);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 t = __ldg(w4 + q);
            v[u][4 * q] = (v[u][4 * q] * r) * t.x;
            v[u][4 * q + 1] = (v[u][4 * q + 1] * r) * t.y;
            v[u][4 * q + 2] = (v[u][4 * q + 2] * r) * t.z;
            v[u][4 * q + 3] = (v[u][4 * q + 3] * r) * t.w;
          }
        }
      }
    }
    float am = 0.f;
#pragma unroll
    for (int u = 0; u < UMAX; ++u)
      if (lane + 32 * u < units)
#pragma unroll
        for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(v[u][e]));
    am = warp_max(am);
    const int ex = row_exponent(am);
    const float scale = pow2f(ex);
    if (lane == 0) inv_scale[b] = pow2f(-ex);
#pragma unroll
    for (int u = 0; u < UMAX; ++u) {
      const int id = lane + 32 * u;
      if (id < units) split16(xf, id >> 2, b, id & 3, v[u], scale);
    }
  } else if (b < MAXB) {
    float z[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) z[e] = 0.f;
    for (int id = lane; id < units; id += 32) split16(xf, id >> 2, b, id & 3, z, 1.f);
    if (lane == 0) inv_scale[b] = 1.f;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

struct Smem {
  uint64_t full[NSLOT], empty[NSLOT], kvbar;
  int ok;
  int ticket_last;
  float inv_scale[MAXB];
  uint32_t epoch, step0;
  int tok[MAXB];
};

__global__ void __launch_bounds__(NT, 1) decode_stream_kernel(const cv3_decode_params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* ring = smem_raw;
  uint8_t* xf = ring + NSLOT * SLOT_BYTES;
  float* redbuf = reinterpret_cast<float*>(xf + XF_BYTES);
  Smem& S = *reinterpret_cast<Smem*>(redbuf + RED_FLOATS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Dims d = dims_of(p);
  const int G = d.G, B = d.B, hid = d.hid;
  uint32_t* sync = p.sync;
  // sync words: [0] steps completed, then per layer 5 phase counters, F, G, then E tickets
  const int e_tiles = hid / RT;
  uint32_t* ctr = sync + 1;
  uint32_t* tickets = ctr + PH_PER_LAYER * p.n_layers + 2;

  if (tid == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1);
    }
    mbar_init(&S.kvbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    S.epoch = *reinterpret_cast<volatile uint32_t*>(sync);
    S.step0 = (uint32_t)__ldcg(p.step);
  }
  __syncthreads();
  const uint32_t epoch = S.epoch;
  const Ring R{ring, S.full, S.empty};

  const Mat mA0 = make_mat(nullptr, nullptr, d.qkv_rows, hid), mC0 = make_mat(nullptr, nullptr, hid, hid);
  const Mat mD0 = make_mat(nullptr, nullptr, 2 * d.inter, hid), mE0 = make_mat(nullptr, nullptr, hid, d.inter);
  const Mat mF = make_mat(p.head_q, p.head_s, d.vocab_pad, hid);
  const int nB = B * d.Hk * d.nch;

  // ======================= producer warp ========================================
  if (warp == NCW) {
    if (lane == 0) {
      uint32_t fill = 0;
      bool ok = true;
      for (int s = 0; s < p.steps && ok; ++s) {
        for (int l = 0; l < p.n_layers && ok; ++l) {
          const Layer L = layer_at(p, l);
          Mat m = mA0;
          m.q = L.qkv_q; m.s = L.qkv_s;
          ok = ok && produce_mat(R, m, d.off_a, G, fill);
          m = mC0;
          m.q = L.o_q; m.s = L.o_s;
          ok = ok && produce_mat(R, m, d.off_c, G, fill);
          m = mD0;
          m.q = L.gu_q; m.s = L.gu_s;
          ok = ok && produce_mat(R, m, d.off_d, G, fill);
          m = mE0;
          m.q = L.dn_q; m.s = L.dn_s;
          ok = ok && produce_mat(R, m, d.off_e, G, fill);
        }
        ok = ok && produce_mat(R, mF, d.off_f, G, fill);
      }
      // leave only once every copy issued into this CTA's ring has landed (on success the
      // consumers have waited for all of them already; after a failure some may be pending).
      // A slot is refilled only by this warp, so the parity of its last fill is unambiguous.
      for (uint32_t f = fill > (uint32_t)NSLOT ? fill - NSLOT : 0; f < fill; ++f) {
        const unsigned long long t0 = now_ns();
        while (now_ns() - t0 < 100000000ull) {
          uint32_t done;
          asm volatile(
              "{\n\t.reg .pred p;\n\t"
              "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
              "selp.u32 %0, 1, 0, p;\n\t}"
              : "=r"(done)
              : "r"(sa(&S.full[f % NSLOT])), "r"((f / NSLOT) & 1)
              : "memory");
          if (done) break;
        }
      }
    }
    return;
  }

  // ======================= consumer warps =======================================
  uint32_t use_ctr = 0;   // ring slots consumed
  uint32_t kv_use = 0;    // KV prefetches waited on
  bool kv_pending = false; // one issued and not yet waited on
  int item_parity = 0;
  bool ok = true;

  // one GEMV item: wait for its slot, the MMAs, the fixed-order reduction; epi(r, b, v)
  // runs for every (row r of the tile, sequence b < B); then the slot is released
  auto run_item = [&](const Mat& m, int i, auto&& epi) -> bool {
    const int ks = m.k / 64;
    const int tile = i / m.parts, part = i - tile * m.parts;
    const int g0 = part * m.gp, ng = min(m.gp, ks - g0);
    const int slot = use_ctr % NSLOT;
    if (!csync_and(mbar_wait(&S.full[slot], (use_ctr / NSLOT) & 1, 5))) return false;
    float* red = redbuf + item_parity * (NCW * RT * MAXB);
    tile_mma(ring + slot * SLOT_BYTES, ng, 64 * ng, ks, g0, xf, red);
    csync();
    if (tid == 0) mbar_arrive(&S.empty[slot]);
    ++use_ctr;
    if (tid < RT * MAXB) {
      const int r = tid / MAXB, b = tid % MAXB;
      if (b < B) epi(tile, part, r, b, red_sum(red, r, b) * S.inv_scale[b], red);
    }
    item_parity ^= 1;
    return true;
  };

  for (int s = 0; s < p.steps && ok; ++s) {
    const uint32_t t = epoch + (uint32_t)s;
    // the previous step's G (token, positions, next input) is complete
    if (s > 0 || t > 0) ok = wait_count(ctr + PH_PER_LAYER * p.n_layers + 1, t * (uint32_t)contributors(B, G), &S.ok);
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const Layer L = layer_at(p, l);
      uint32_t* cl = ctr + PH_PER_LAYER * l;
      // ---- A: qkv ------------------------------------------------------------------
      {
        Mat m = mA0;
        m.q = L.qkv_q; m.s = L.qkv_s;
        const int i0 = first_item(d.off_a, G);
        if (i0 < m.items()) {
          if (l > 0) ok = ok && wait_count(ctr + PH_PER_LAYER * (l - 1) + 4, (t + 1) * contributors(mE0.items(), G), &S.ok);
          if (!ok) break;
          stage_rows(xf, p.h, hid, B, hid, 0, hid, L.ln1, p.eps, S.inv_scale);
          csync();
          for (int i = i0; i < m.items() && ok; i += G)
            ok = run_item(m, i, [&](int tile, int, int r, int b, float v, const float*) {
              const int row = tile * RT + r;
              __stcg(p.qkv + (int64_t)b * d.qkv_rows + row, v + L.qkv_b[row]);
            });
          csync();
          if (tid == 0) signal(cl + 0);
        }
      }
      if (!ok) break;
      // ---- B: attention chunks ----------------------------------------------------------
      {
        const int i0 = first_item(d.off_b, G);
        if (i0 < nB) {
          const uint32_t target = (t + 1) * contributors(mA0.items(), G);
          bool waited = false;
          for (int i = i0; i < nB && ok; i += G) {
            const int b = i / (d.Hk * d.nch), rem = i - b * (d.Hk * d.nch);
            const int kh = rem / d.nch, ch = rem - kh * d.nch;
            const int pos = __ldcg(p.pos + b);
            if (pos >= p.cap && tid == 0) fail_with(2);  // the host sizes the cache; never appended
            const int len = min(pos + 1, (int)p.cap);
            const int j0 = ch * KCH, j1 = min(j0 + KCH, len);
            float* kc = L.kc + ((int64_t)b * d.Hk + kh) * p.cap * HD;
            float* vc = L.vc + ((int64_t)b * d.Hk + kh) * p.cap * HD;
            float* ks_ = reinterpret_cast<float*>(xf);            // [KCH][64] keys
            float* vs_ = ks_ + KCH * HD;                          // [KCH][64] values
            float* qs = vs_ + KCH * HD;                           // [8][64] scaled, rotated queries
            float* sc = qs + 8 * HD;                              // [8][KCH] scores -> probabilities
            float* knew = sc + 8 * KCH;                           // [64]
            float* vnew = knew + HD;                              // [64]
            const int hpg = d.H / d.Hk;
            // cached keys/values of this chunk's older positions: copied before the wait
            const int jold = min(j1, pos);                        // positions < pos are in the cache
            const int nold = max(jold - j0, 0);
            if (tid == 0 && nold > 0) {
              mbar_expect_tx(&S.kvbar, (uint32_t)(2 * nold * HD * 4));
              bulk_g2s(ks_, kc + (int64_t)j0 * HD, (uint32_t)(nold * HD * 4), &S.kvbar);
              bulk_g2s(vs_, vc + (int64_t)j0 * HD, (uint32_t)(nold * HD * 4), &S.kvbar);
            }
            kv_pending = nold > 0;
            if (!waited) {
              ok = wait_count(cl + 0, target, &S.ok);
              waited = true;
            }
            if (ok && nold > 0) {
              ok = csync_and(mbar_wait(&S.kvbar, kv_use & 1, 6));
              if (ok) {
                kv_pending = false;
                ++kv_use;
              }
            }
            if (!ok) break;
            if (j0 < j1) {
              // RoPE of the group's queries (pre-scaled) and of the new key, at position pos
              const float* row = p.qkv + (int64_t)b * d.qkv_rows;
              const bool has_new = pos >= j0 && pos < j1;
              const int pt = pos < p.cap ? pos : 0;
              for (int e = tid; e < (hpg + 2) * HD; e += NCT) {
                const int hh = e / HD, dd = e - hh * HD;
                const int slot = hh < hpg ? kh * hpg + hh : (hh == hpg ? d.H + kh : d.H + d.Hk + kh);
                const float* x = row + (int64_t)slot * HD;
                float v = __ldcg(x + dd);
                if (hh <= hpg) {
                  const float rot = dd < HD / 2 ? -__ldcg(x + dd + HD / 2) : __ldcg(x + dd - HD / 2);
                  v = __fadd_rn(__fmul_rn(v, p.cos_table[(int64_t)pt * HD + dd]),
                                __fmul_rn(rot, p.sin_table[(int64_t)pt * HD + dd]));
                }
                if (hh < hpg) qs[hh * HD + dd] = v * p.scale;
                else if (hh == hpg) knew[dd] = v;
                else vnew[dd] = v;
              }
              csync();
              if (has_new) {
                for (int e = tid; e < 2 * HD; e += NCT) {
                  const int dd = e & (HD - 1);
                  if (e < HD) {
                    ks_[(pos - j0) * HD + dd] = knew[dd];
                    kc[(int64_t)pos * HD + dd] = knew[dd];
                  } else {
                    vs_[(pos - j0) * HD + dd] = vnew[dd];
                    vc[(int64_t)pos * HD + dd] = vnew[dd];
                  }
                }
                csync();
              }
              const int n = j1 - j0;
              // scores: warp per query head, lane per key (two keys per lane), dims rotated
              // per lane to spread the shared-memory banks
              if (warp < hpg) {
                const float* qh = qs + warp * HD;
                for (int jj = lane; jj < n; jj += 32) {
                  const float* kr = ks_ + jj * HD;
                  float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                  for (int q = 0; q < HD / 4; ++q) {
                    const int qq = (q + jj) & (HD / 4 - 1);
                    const float4 kv = *reinterpret_cast<const float4*>(kr + 4 * qq);
                    const float4 qv = *reinterpret_cast<const float4*>(qh + 4 * qq);
                    a4[0] = fmaf(qv.x, kv.x, a4[0]);
                    a4[1] = fmaf(qv.y, kv.y, a4[1]);
                    a4[2] = fmaf(qv.z, kv.z, a4[2]);
                    a4[3] = fmaf(qv.w, kv.w, a4[3]);
                  }
                  sc[warp * KCH + jj] = (a4[0] + a4[1]) + (a4[2] + a4[3]);
                }
                float mx = -INFINITY;
                for (int jj = lane; jj < n; jj += 32) mx = fmaxf(mx, sc[warp * KCH + jj]);
                mx = warp_max(mx);
                float sum = 0.f;
                for (int jj = lane; jj < n; jj += 32) {
                  const float pr = expf(sc[warp * KCH + jj] - mx);
                  sc[warp * KCH + jj] = pr;
                  sum += pr;
                }
                sum = warp_sum(sum);
                float* part = p.attn_part + (((int64_t)b * d.H + kh * hpg + warp) * d.nch + ch) * (HD + 2);
                if (lane == 0) {
                  __stcg(part + HD, mx);
                  __stcg(part + HD + 1, sum);
                }
              }
              csync();
              // unnormalised P.V: thread per (head, dim)
              for (int e = tid; e < hpg * HD; e += NCT) {
                const int hh = e / HD, dd = e - hh * HD;
                float o = 0.f;
                for (int jj = 0; jj < n; ++jj) o = fmaf(sc[hh * KCH + jj], vs_[jj * HD + dd], o);
                __stcg(p.attn_part + (((int64_t)b * d.H + kh * hpg + hh) * d.nch + ch) * (HD + 2) + dd, o);
              }
            }
            csync();
          }
          csync();
          if (tid == 0) signal(cl + 1);
        }
      }
      if (!ok) break;
      // ---- C: h1 = h + merge(attention) . Wo^T ---------------------------------------------
      {
        Mat m = mC0;
        m.q = L.o_q; m.s = L.o_s;
        const int i0 = first_item(d.off_c, G);
        if (i0 < m.items()) {
          ok = wait_count(cl + 1, (t + 1) * contributors(nB, G), &S.ok);
          if (!ok) break;
          // merge the chunks of every head into the fp32 attention row of each sequence
          // (staged through the reduction buffer's neighbour: the split store itself)
          {
            const int b = warp;
            if (b < B) {
              const int len = min(__ldcg(p.pos + b) + 1, (int)p.cap);
              const int nc = (len + KCH - 1) / KCH;
              float v[(GMAX * 4 + 31) / 32][16];
              const int units = hid / 16;
              constexpr int UMAX = (GMAX * 4 + 31) / 32;
#pragma unroll
              for (int u = 0; u < UMAX; ++u) {
                const int id = lane + 32 * u;
                if (id < units) {
                  const int col = 16 * id;                 // hid columns: head col / 64
                  const int hh = col / HD, dd0 = col - hh * HD;
                  const float* base = p.attn_part + ((int64_t)b * d.H + hh) * d.nch * (HD + 2);
                  float M = -INFINITY;
                  for (int cc = 0; cc < nc; ++cc) M = fmaxf(M, __ldcg(base + cc * (HD + 2) + HD));
                  float Lsum = 0.f;
#pragma unroll
                  for (int e = 0; e < 16; ++e) v[u][e] = 0.f;
                  for (int cc = 0; cc < nc; ++cc) {
                    const float* pc = base + cc * (HD + 2);
                    const float f = expf(__ldcg(pc + HD) - M);
                    Lsum = fmaf(__ldcg(pc + HD + 1), f, Lsum);
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[u][e] = fmaf(__ldcg(pc + dd0 + e), f, v[u][e]);
                  }
#pragma unroll
                  for (int e = 0; e < 16; ++e) v[u][e] = v[u][e] / Lsum;
                }
              }
              // the staged values are in K order (columns 16 id .. 16 id + 15 = group id/4, c id%4)
              float am = 0.f;
#pragma unroll
              for (int u = 0; u < UMAX; ++u)
                if (lane + 32 * u < units)
#pragma unroll
                  for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(v[u][e]));
              am = warp_max(am);
              const int ex = row_exponent(am);
              if (lane == 0) S.inv_scale[b] = pow2f(-ex);
#pragma unroll
              for (int u = 0; u < UMAX; ++u) {
                const int id = lane + 32 * u;
                if (id < units) split16(xf, id >> 2, b, id & 3, v[u], pow2f(ex));
              }
            } else if (b < MAXB) {
              float z[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) z[e] = 0.f;
              for (int id = lane; id < hid / 16; id += 32) split16(xf, id >> 2, b, id & 3, z, 1.f);
              if (lane == 0) S.inv_scale[b] = 1.f;
            }
          }
          csync();
          for (int i = i0; i < m.items() && ok; i += G)
            ok = run_item(m, i, [&](int tile, int, int r, int b, float v, const float*) {
              const int row = tile * RT + r;
              __stcg(p.h1 + (int64_t)b * hid + row, __ldcg(p.h + (int64_t)b * hid + row) + v);
            });
          csync();
          if (tid == 0) signal(cl + 2);
        }
      }
      if (!ok) break;
      // ---- D: act = silu(gate) * up of RMSNorm(h1) ----------------------------------------
      {
        Mat m = mD0;
        m.q = L.gu_q; m.s = L.gu_s;
        const int i0 = first_item(d.off_d, G);
        if (i0 < m.items()) {
          ok = wait_count(cl + 2, (t + 1) * contributors(mC0.items(), G), &S.ok);
          if (!ok) break;
          stage_rows(xf, p.h1, hid, B, hid, 0, hid, L.ln2, p.eps, S.inv_scale);
          csync();
          for (int i = i0; i < m.items() && ok; i += G)
            ok = run_item(m, i, [&](int tile, int, int r, int b, float v, const float* red) {
              if ((r & 1) == 0) {  // rows 2j (gate) and 2j + 1 (up) of the interleaved matrix
                const float up = red_sum(red, r + 1, b) * S.inv_scale[b];
                const int j = (tile * RT + r) >> 1;
                __stcg(p.act + (int64_t)b * d.inter + j, (v / (1.0f + expf(-v))) * up);
              }
            });
          csync();
          if (tid == 0) signal(cl + 3);
        }
      }
      if (!ok) break;
      // ---- E: h = h1 + act . Wdown^T (K parts, the last part of a tile adds them) ---------
      {
        Mat m = mE0;
        m.q = L.dn_q; m.s = L.dn_s;
        const int i0 = first_item(d.off_e, G);
        if (i0 < m.items()) {
          ok = wait_count(cl + 3, (t + 1) * contributors(mD0.items(), G), &S.ok);
          if (!ok) break;
          for (int i = i0; i < m.items() && ok; i += G) {
            const int tile = i / m.parts, part = i - tile * m.parts;
            const int g0 = part * m.gp, ng = min(m.gp, d.inter / 64 - g0);
            csync();  // the previous item's epilogue has read the staged scales
            stage_rows(xf, p.act, d.inter, B, d.inter, 64 * g0, 64 * ng, nullptr, 0.f, S.inv_scale);
            csync();
            if (m.parts == 1) {
              ok = run_item(m, i, [&](int tl, int, int r, int b, float v, const float*) {
                const int row = tl * RT + r;
                __stcg(p.h + (int64_t)b * hid + row, __ldcg(p.h1 + (int64_t)b * hid + row) + v);
              });
              continue;
            }
            ok = run_item(m, i, [&](int tl, int pt, int r, int b, float v, const float*) {
              __stcg(p.part + (((int64_t)tl * m.parts + pt) * RT + r) * MAXB + b, v);
            });
            if (!ok) break;
            csync();
            if (tid == 0) {
              __threadfence();
              const uint32_t old = atomicAdd(&tickets[l * e_tiles + tile], 1u);
              S.ticket_last = ((old + 1) % (uint32_t)m.parts) == 0;
              __threadfence();
            }
            csync();
            if (S.ticket_last && tid < RT * MAXB) {
              const int r = tid / MAXB, b = tid % MAXB;
              if (b < B) {
                float y = 0.f;
                for (int pt = 0; pt < m.parts; ++pt) y += __ldcg(p.part + (((int64_t)tile * m.parts + pt) * RT + r) * MAXB + b);
                const int row = tile * RT + r;
                __stcg(p.h + (int64_t)b * hid + row, __ldcg(p.h1 + (int64_t)b * hid + row) + y);
              }
            }
            csync();
          }
          csync();
          if (tid == 0) signal(cl + 4);
        }
      }
    }
    if (!ok) break;
    // ---- F: logits = RMSNorm(h, norm) . Whead^T --------------------------------------------
    {
      const int i0 = first_item(d.off_f, G);
      if (i0 < mF.items()) {
        ok = wait_count(ctr + PH_PER_LAYER * (p.n_layers - 1) + 4, (t + 1) * contributors(mE0.items(), G), &S.ok);
        if (!ok) break;
        stage_rows(xf, p.h, hid, B, hid, 0, hid, p.final_norm, p.eps, S.inv_scale);
        csync();
        for (int i = i0; i < mF.items() && ok; i += G)
          ok = run_item(mF, i, [&](int tile, int, int r, int b, float v, const float*) {
            const int row = tile * RT + r;
            if (row < p.vocab) __stcg(p.logits + (int64_t)b * p.vocab + row, v);
          });
        csync();
        if (tid == 0) signal(ctr + PH_PER_LAYER * p.n_layers);
      }
    }
    if (!ok) break;
    // ---- G: greedy pick, bookkeeping, next input (one CTA per sequence) ------------------
    {
      const int i0 = first_item(d.off_g, G);
      if (i0 < B) {
        ok = wait_count(ctr + PH_PER_LAYER * p.n_layers, (t + 1) * contributors(mF.items(), G), &S.ok);
        if (!ok) break;
        float* red = redbuf;
        for (int b = i0; b < B; b += G) {
          float* x = reinterpret_cast<float*>(xf);
          const float* src = p.logits + (int64_t)b * p.vocab;
          for (int i = tid; i < p.vocab; i += NCT) x[i] = __ldcg(src + i);
          csync();
          float mx = -INFINITY;
          for (int i = tid; i < p.vocab; i += NCT) mx = fmaxf(mx, x[i]);
          mx = warp_max(mx);
          if (lane == 0) red[warp] = mx;
          csync();
          mx = red[0];
          for (int w = 1; w < NCW; ++w) mx = fmaxf(mx, red[w]);
          csync();
          float sum = 0.f;
          for (int i = tid; i < p.vocab; i += NCT) sum += expf(x[i] - mx);
          sum = warp_sum(sum);
          if (lane == 0) red[warp] = sum;
          csync();
          sum = 0.f;
          for (int w = 0; w < NCW; ++w) sum += red[w];
          const float lse = logf(sum);
          csync();
          float best = -INFINITY;
          int besti = 0x7FFFFFFF;
          for (int i = tid; i < p.vocab; i += NCT) {
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
          int* bi = reinterpret_cast<int*>(red + NCW);
          if (lane == 0) {
            red[warp] = best;
            bi[warp] = besti;
          }
          csync();
          if (tid == 0) {
            float bv = red[0];
            int ii = bi[0];
            for (int w = 1; w < NCW; ++w)
              if (red[w] > bv || (red[w] == bv && bi[w] < ii)) {
                bv = red[w];
                ii = bi[w];
              }
            if (ii < 0 || ii >= p.emb_rows) {
              fail_with(7);
              ii = 0;
            }
            S.tok[0] = ii;
            __stcg(reinterpret_cast<long long*>(p.next_ids) + b, (long long)ii);
            const int col = (int)S.step0 + s;
            if (col >= 0 && col < p.hist_stride)
              __stcg(reinterpret_cast<long long*>(p.history) + (int64_t)b * p.hist_stride + col, (long long)ii);
            else fail_with(3);
            __stcg(p.pos + b, __ldcg(p.pos + b) + 1);
            __stcg(p.lens + b, __ldcg(p.lens + b) + 1);
          }
          csync();
          // the chosen token's embedding row becomes sequence b's next input
          const int tk = S.tok[0];
          for (int k = tid; k < hid; k += NCT) {
            float v;
            if (p.emb_scales) {
              const int8_t* er = static_cast<const int8_t*>(p.emb) + (int64_t)tk * hid;
              v = (float)er[k] * h2f(p.emb_scales[(int64_t)tk * (hid / 64) + k / 64]);
            } else {
              v = static_cast<const float*>(p.emb)[(int64_t)tk * hid + k];
            }
            __stcg(p.h + (int64_t)b * hid + k, v);
          }
          csync();
        }
        if (tid == 0) signal(ctr + PH_PER_LAYER * p.n_layers + 1);
      }
    }
  }

  // a K/V prefetch issued but not waited for (the wait before it failed) must land first
  if (kv_pending && tid == 0) {
    const unsigned long long t0 = now_ns();
    while (now_ns() - t0 < 100000000ull) {
      uint32_t done;
      asm volatile(
          "{\n\t.reg .pred p;\n\t"
          "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(sa(&S.kvbar)), "r"(kv_use & 1)
          : "memory");
      if (done) break;
    }
  }
  // the steps-completed word: CTA 0 once every CTA has finished its last G phase
  if (ok && blockIdx.x == 0) {
    const uint32_t t_end = epoch + (uint32_t)p.steps;
    ok = wait_count(ctr + PH_PER_LAYER * p.n_layers + 1, t_end * (uint32_t)contributors(B, G), &S.ok);
    if (ok && tid == 0) {
      *reinterpret_cast<volatile uint32_t*>(sync) = t_end;
      *p.step = (int)S.step0 + p.steps;
      __threadfence();
    }
  }
}

}  // namespace

extern "C" int64_t cv3_decode_sync_words(int64_t n_layers, int64_t hidden) {
  return 1 + PH_PER_LAYER * n_layers + 2 + n_layers * (hidden / RT);
}

extern "C" int cv3_decode_steps(const cv3_decode_params* pr, void* stream) {
  CV3_REQUIRE(pr != nullptr, CV3_ERR_VALUE, "decode_steps: no parameters");
  const cv3_decode_params& p = *pr;
  CV3_REQUIRE(p.batch >= 1 && p.batch <= MAXB, CV3_ERR_VALUE, "decode_steps: 1..%d sequences", MAXB);
  CV3_REQUIRE(p.head_dim == HD && p.heads % p.kv_heads == 0 && p.heads / p.kv_heads <= 8 &&
                  p.hidden == p.heads * HD,
              CV3_ERR_UNSUPPORTED, "decode_steps: head dim 64, <= 8 query heads per kv head, hidden = heads * 64");
  CV3_REQUIRE(p.hidden % 64 == 0 && p.hidden <= 64 * GMAX && p.inter % 64 == 0 && p.inter <= 64 * KS_MAX,
              CV3_ERR_UNSUPPORTED, "decode_steps: hidden <= %d and inter <= %d, multiples of 64", 64 * GMAX,
              64 * KS_MAX);
  CV3_REQUIRE(p.vocab > 0 && p.select > 0 && p.select <= p.vocab && p.steps >= 0 && p.cap > 0 &&
                  p.cap <= (int64_t)1 << 20,
              CV3_ERR_VALUE, "decode_steps: bad vocab / steps / cap");
  CV3_REQUIRE(p.sync && p.sync_words >= cv3_decode_sync_words(p.n_layers, p.hidden) && p.h1 && p.qkv &&
                  p.attn_part && p.part && p.act && p.logits,
              CV3_ERR_VALUE, "decode_steps: scratch buffers (sync words: %lld needed)",
              (long long)cv3_decode_sync_words(p.n_layers, p.hidden));
  CV3_REQUIRE(p.vocab <= XF_BYTES / 4, CV3_ERR_UNSUPPORTED, "decode_steps: vocab %d > %d", p.vocab, XF_BYTES / 4);
  CV3_REQUIRE(((uintptr_t)p.head_q & 15) == 0 && ((uintptr_t)p.head_s & 15) == 0, CV3_ERR_VALUE,
              "decode_steps: 16-byte aligned head");
  if (p.steps == 0) return CV3_OK;
  const int smem = NSLOT * SLOT_BYTES + XF_BYTES + RED_FLOATS * 4 + (int)sizeof(Smem);
  int rc = cv3::allow_smem((const void*)decode_stream_kernel, smem);
  if (rc) return rc;
  int per_sm = 0;
  CV3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_stream_kernel, NT, smem));
  CV3_REQUIRE(per_sm >= 1, CV3_ERR_UNSUPPORTED, "decode_steps: the kernel does not fit on an SM");
  const int grid = cv3::sm_count();
  cv3_decode_params local = p;
  void* args[] = {&local};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)decode_stream_kernel, dim3(grid), dim3(NT), args,
                                                    (size_t)smem, cv3::as_stream(stream));
  return cv3::check_launch("decode_steps", e);
}

extern "C" int cv3_decode_status(int* code) {
  int v = 0;
  CV3_CUDA(cudaMemcpyFromSymbol(&v, g_ds_err, sizeof(int)));
  if (v) {
    const int zero = 0;
    CV3_CUDA(cudaMemcpyToSymbol(g_ds_err, &zero, sizeof(int)));
  }
  if (code) *code = v;
  return CV3_OK;
}

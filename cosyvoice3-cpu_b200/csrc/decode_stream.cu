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
// next tiles (cp.async.bulk, completion on an mbarrier) into an 8-slot ring while the
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
// two fp16 parts (x = hi + lo, 22 significant bits), done once per phase and kept in
// shared memory in fragment order.  Each 64-wide scale group's two partial sums are
// added small part first, scaled by the group's fp16 scale and
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
constexpr int MAXCH = 24;              // most chunks per sequence (cap <= 1536)
constexpr int GMAX = 19;               // most scale groups per work item (K <= 1216)
constexpr int KS_MAX = 76;             // most scale groups per matrix row (K <= 4864)
constexpr int SLOT_W = RT * GMAX * 64; // 19,456 B of rows (row stride <= 1216)
constexpr int SLOT_S = RT * KS_MAX * 2;  // 2,432 B: a whole tile's fp16 scales
constexpr int SLOT_BYTES = SLOT_W + SLOT_S;  // 21,888 = 171 * 128
constexpr int NSLOT = 8;
constexpr int NPART = 2;                         // fp16 parts per activation (22 significant bits)
constexpr int XF_GROUP = NPART * 4 * 32 * 8;     // bytes of split activations per scale group
constexpr int XF_BYTES = GMAX * XF_GROUP;        // 38,912
constexpr int RED_FLOATS = 2 * NCW * RT * MAXB;
constexpr unsigned long long WAIT_NS = 2000000000ull;
constexpr int PH_PER_LAYER = 5;
constexpr int TRACE_VALS = 6;

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

__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(sa(b)), "r"(parity)
      : "memory");
  return done != 0;
}

// true once the phase with this parity has completed; false after WAIT_NS (error set).
// The clock and the global error word are read only every 256 polls: many threads of
// every CTA poll at once, and a global read per poll would pile them onto one L2 line.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int code) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(b, parity)) return true;
    if ((it & 255) == 0 && (now_ns() - t0 > WAIT_NS || failed())) {
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

// thread 0 of the consumers, after a consumer barrier: publish one completion.  The
// release orders every consumer's earlier writes (made visible to this thread by the
// barrier) before the increment, without waiting for a reply.
__device__ __forceinline__ void signal(uint32_t* ctr) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// all consumers: wait until *ctr >= target (bounded), then see everything published before
__device__ __forceinline__ bool wait_count(const uint32_t* ctr, uint32_t target, int* ok_s) {
  if (threadIdx.x == 0) {
    int ok = 1;
    if ((int)(ld_acquire(ctr) - target) < 0) {
      const unsigned long long t0 = now_ns();
      for (uint32_t it = 1; (int)(ld_acquire(ctr) - target) < 0; ++it) {
        if ((it & 15) == 0 && (now_ns() - t0 > WAIT_NS || failed())) {
          fail_with(1);
          ok = 0;
          break;
        }
      }
    }
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
// x = hi + lo with hi = fp16(x) and lo = fp16(x - hi): 22 significant bits, a relative
// error of at most 2^-22 per element (the row scaling keeps both parts in fp16 range).
__device__ __forceinline__ void split16(uint8_t* xf, int G, int g, int c, const float v[16], float scale) {
  uint2* base = reinterpret_cast<uint2*>(xf + G * XF_GROUP);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = v[4 * j + e] * scale;  // exact: a power of two
    uint32_t w[NPART][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float a = x[2 * h], b = x[2 * h + 1];
      const uint32_t hi = f2h2(a, b);
      float ha, hb;
      h22f(hi, ha, hb);
      w[0][h] = hi;
      w[1][h] = f2h2(a - ha, b - hb);
    }
#pragma unroll
    for (int pp = 0; pp < NPART; ++pp) base[(pp * 4 + j) * 32 + g * 4 + c] = make_uint2(w[pp][0], w[pp][1]);
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

// One work item on `wpi` warps (this warp is number `sub` of them): they split its ng
// scale groups; per-warp sums of rows (g, g + 8) x sequences (2c, 2c + 1) go to
// red[warp] (fixed-order reduction later).
__device__ __forceinline__ void tile_mma(const uint8_t* slot, int ng, int kbytes, int ks, int g0, const uint8_t* xf,
                                         float* red, int sub, int wpi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int stride = row_stride(kbytes);
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + SLOT_W);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int G = sub; G < ng; G += wpi) {
    const int4 w0 = *reinterpret_cast<const int4*>(slot + g * stride + 64 * G + 16 * c);
    const int4 w1 = *reinterpret_cast<const int4*>(slot + (g + 8) * stride + 64 * G + 16 * c);
    const float s0 = h2f(sc[g * ks + g0 + G]), s1 = h2f(sc[(g + 8) * ks + g0 + G]);
    const uint32_t u0[4] = {(uint32_t)w0.x ^ 0x80808080u, (uint32_t)w0.y ^ 0x80808080u,
                            (uint32_t)w0.z ^ 0x80808080u, (uint32_t)w0.w ^ 0x80808080u};
    const uint32_t u1[4] = {(uint32_t)w1.x ^ 0x80808080u, (uint32_t)w1.y ^ 0x80808080u,
                            (uint32_t)w1.z ^ 0x80808080u, (uint32_t)w1.w ^ 0x80808080u};
    const uint2* xb = reinterpret_cast<const uint2*>(xf + G * XF_GROUP);
    float t[NPART][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t A0 = i8pair(u0[j], 0x4140u);  // row g,     k 2c, 2c+1
      const uint32_t A1 = i8pair(u1[j], 0x4140u);  // row g + 8, k 2c, 2c+1
      const uint32_t A2 = i8pair(u0[j], 0x4342u);  // row g,     k 2c+8, 2c+9
      const uint32_t A3 = i8pair(u1[j], 0x4342u);  // row g + 8, k 2c+8, 2c+9
#pragma unroll
      for (int pp = 0; pp < NPART; ++pp) {
        const uint2 b = xb[(pp * 4 + j) * 32 + lane];
        mma_f16(t[pp], A0, A1, A2, A3, b.x, b.y);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = t[1][e] + t[0][e];
      acc[e] = fmaf(v, e < 2 ? s0 : s1, acc[e]);
    }
  }
  float* rw = red + warp * RT * MAXB;
  rw[g * MAXB + 2 * c] = acc[0];
  rw[g * MAXB + 2 * c + 1] = acc[1];
  rw[(g + 8) * MAXB + 2 * c] = acc[2];
  rw[(g + 8) * MAXB + 2 * c + 1] = acc[3];
}

// Stage RMSNorm(src) (norm_w non-null) or src, columns [k0, k0 + kw) of each of the B
// rows (row stride ld), as split fp16 fragments; one warp per sequence.  Rows >= B are
// zeros.  inv_scale[b] receives 2^-e of sequence b's fp16 scaling.
__device__ __noinline__ void stage_rows(uint8_t* xf, const float* src, int64_t ld, int B, int K, int k0, int kw, const float* norm_w,
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
          const float4* w4 = reinterpret_cast<const float4*>(norm_w + k0 + 64 * G + 16 * c);  // shared memory
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 t = w4[q];
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
  float fst[256];                          // the head tiles' epilogue reductions (two at a time)
  __align__(16) float normw[64 * GMAX];    // the phase's RMSNorm weight
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
  uint32_t use_ctr = 0;    // ring slots consumed
  uint32_t kv_use = 0;     // K/V prefetches waited on
  bool kv_pending = false; // one issued and not yet waited on
  bool ok = true;
  // optional per-phase trace of one step (p.trace, thread 0): [CTA][phase][6] = wait begun,
  // wait done, phase done (ns, %globaltimer), ns spent waiting for ring slots, inputs
  // staged, last item done
  const int nph = PH_PER_LAYER * p.n_layers + 2;
  int cur_step = -1;
  uint64_t ring_ns = 0;
  auto tr = [&](int ph, int k) {
    if (p.trace && tid == 0 && cur_step == p.trace_step)
      p.trace[((int64_t)blockIdx.x * nph + ph) * TRACE_VALS + k] = (k == 3) ? ring_ns : now_ns();
    if (k == 3) ring_ns = 0;
  };
  // A batch of nb <= 8 of this CTA's items of one matrix (items i, i + G, ..., in
  // consecutive ring slots, all reading the same staged activations): item j runs on
  // warps [j wpi, (j + 1) wpi), wpi = 8 / nb, all items at once; then the fixed-order
  // reduction of each item's warps and epi(j, tile, part, r, b, v, red_base, wpi) for every
  // (item, row r of its tile, sequence b), two items at a time (128 threads each)
  auto run_batch = [&](const Mat& m, int ifirst, int nb, auto&& epi) -> bool {
    const int ks = m.k / 64;
    const int wpi = NCW / nb;
    const int j = warp / wpi, sub = warp - j * wpi;
    float* red = redbuf;
    bool okw = true;
    const unsigned long long tw = (p.trace && tid == 0) ? now_ns() : 0;
    if (j < nb) {
      const int i = ifirst + j * G;
      const int tile = i / m.parts, part = i - tile * m.parts;
      const int g0 = part * m.gp, ng = min(m.gp, ks - g0);
      const uint32_t u = use_ctr + (uint32_t)j;
      const int slot = u % NSLOT;
      okw = mbar_wait(&S.full[slot], (u / NSLOT) & 1, 5);
      if (okw) tile_mma(ring + slot * SLOT_BYTES, ng, 64 * ng, ks, g0, xf, red, sub, wpi);
    }
    if (!csync_and(okw)) return false;
    if (p.trace && tid == 0) ring_ns += now_ns() - tw;
    if (tid == 0)
      for (int jj = 0; jj < nb; ++jj) mbar_arrive(&S.empty[(use_ctr + (uint32_t)jj) % NSLOT]);
    use_ctr += (uint32_t)nb;
    for (int k = 0; k < nb; k += 2) {
      const int jj = k + (tid >> 7);
      if (jj < nb) {
        const int i = ifirst + jj * G;
        const int tile = i / m.parts, part = i - tile * m.parts;
        const int r = (tid & 127) / MAXB, b = tid % MAXB;
        float v = 0.f;
        for (int w = jj * wpi; w < (jj + 1) * wpi; ++w) v += red[w * RT * MAXB + r * MAXB + b];
        epi(jj, tile, part, r, b, b < B ? v * S.inv_scale[b] : 0.f, red + jj * wpi * RT * MAXB, wpi);
      }
    }
    csync();  // the reduction buffer is free for the next batch
    return true;
  };
  // this CTA's items i0, i0 + G, ... of a matrix, in batches of up to 8
  auto run_items = [&](const Mat& m, int i0, auto&& epi) -> bool {
    const int n = i0 < m.items() ? (m.items() - 1 - i0) / G + 1 : 0;
    for (int k = 0; k < n; k += NCW)
      if (!run_batch(m, i0 + k * G, min(NCW, n - k), epi)) return false;
    return true;
  };
  // an RMSNorm weight vector into shared memory (cp.async, in flight across the next wait)
  auto fetch_norm = [&](const float* w) {
    for (int i = tid; i < hid / 4; i += NCT)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa(S.normw + 4 * i)), "l"(w + 4 * i) : "memory");
  };
  auto norm_ready = [&]() { asm volatile("cp.async.wait_all;" ::: "memory"); };
  const int erow = tid / MAXB, eb = tid % MAXB;  // the epilogue's (row in tile, sequence)
  const int hpg = d.H / d.Hk;
  uint32_t* btickets = tickets + p.n_layers * e_tiles;

  for (int s = 0; s < p.steps && ok; ++s) {
    const uint32_t t = epoch + (uint32_t)s;
    cur_step = s;
    // the previous step's G (token, positions, next input) is complete
    if (s > 0 || t > 0) ok = wait_count(ctr + PH_PER_LAYER * p.n_layers + 1, t * (uint32_t)contributors(B, G), &S.ok);
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const Layer L = layer_at(p, l);
      uint32_t* cl = ctr + PH_PER_LAYER * l;
      // ---- A: qkv = RMSNorm(h, ln1) . Wqkv^T + b ------------------------------------
      {
        Mat m = mA0;
        m.q = L.qkv_q; m.s = L.qkv_s;
        const int i0 = first_item(d.off_a, G);
        if (i0 < m.items()) {
          fetch_norm(L.ln1);
          const float bias0 = (tid < RT * MAXB) ? __ldg(L.qkv_b + (i0 / m.parts) * RT + erow) : 0.f;
          tr(PH_PER_LAYER * l + 0, 0);
          if (l > 0) ok = wait_count(ctr + PH_PER_LAYER * (l - 1) + 4, (t + 1) * contributors(mE0.items(), G), &S.ok);
          tr(PH_PER_LAYER * l + 0, 1);
          norm_ready();
          csync();
          if (!ok) break;
          stage_rows(xf, p.h, hid, B, hid, 0, hid, S.normw, p.eps, S.inv_scale);
          csync();
          tr(PH_PER_LAYER * l + 0, 4);
          ok = run_items(m, i0, [&](int jj, int tile, int, int r, int b, float v, const float*, int) {
            if (b >= B) return;
            const int row = tile * RT + r;
            __stcg(p.qkv + (int64_t)b * d.qkv_rows + row, v + (jj == 0 ? bias0 : __ldg(L.qkv_b + row)));
          });
          tr(PH_PER_LAYER * l + 0, 5);
          csync();
          if (tid == 0) signal(cl + 0);
          tr(PH_PER_LAYER * l + 0, 2);
          tr(PH_PER_LAYER * l + 0, 3);
        }
      }
      if (!ok) break;
      // ---- B: attention chunks; the last chunk of a (sequence, kv head) merges ----------
      {
        const int i0 = first_item(d.off_b, G);
        if (i0 < nB) {
          const uint32_t target = (t + 1) * contributors(mA0.items(), G);
          bool waited = false;
          float* ks_ = reinterpret_cast<float*>(xf);  // [KCH][64] keys
          float* vs_ = ks_ + KCH * HD;                // [KCH][64] values
          float* qs = vs_ + KCH * HD;                 // [8][64] scaled, rotated queries
          float* sc = qs + 8 * HD;                    // [8][KCH] scores -> probabilities; merge stats
          float* knew = sc + 8 * KCH;                 // [64]
          float* vnew = knew + HD;                    // [64]
          for (int i = i0; i < nB && ok; i += G) {
            const int b = i / (d.Hk * d.nch), rem = i - b * (d.Hk * d.nch);
            const int kh = rem / d.nch, ch = rem - kh * d.nch;
            const int pos = __ldcg(p.pos + b);
            if (pos >= p.cap && tid == 0) fail_with(2);  // the host sizes the cache; never appended
            const int len = min(pos + 1, (int)p.cap);
            const int j0 = ch * KCH, j1 = min(j0 + KCH, len);
            float* kc = L.kc + ((int64_t)b * d.Hk + kh) * p.cap * HD;
            float* vc = L.vc + ((int64_t)b * d.Hk + kh) * p.cap * HD;
            // cached keys/values of this chunk's older positions: copied before the wait
            const int jold = min(j1, pos);
            const int nold = max(jold - j0, 0);
            if (tid == 0 && nold > 0) {
              mbar_expect_tx(&S.kvbar, (uint32_t)(2 * nold * HD * 4));
              bulk_g2s(ks_, kc + (int64_t)j0 * HD, (uint32_t)(nold * HD * 4), &S.kvbar);
              bulk_g2s(vs_, vc + (int64_t)j0 * HD, (uint32_t)(nold * HD * 4), &S.kvbar);
            }
            kv_pending = nold > 0;
            // RoPE tables of this position (constants): loaded before the wait
            const int pt = pos < p.cap ? pos : 0;
            float cs[3], sn[3];
#pragma unroll
            for (int u = 0; u < 3; ++u) {
              const int e = tid + u * NCT;
              const int dd = e & (HD - 1);
              cs[u] = e < (hpg + 1) * HD ? __ldg(p.cos_table + (int64_t)pt * HD + dd) : 0.f;
              sn[u] = e < (hpg + 1) * HD ? __ldg(p.sin_table + (int64_t)pt * HD + dd) : 0.f;
            }
            if (!waited) {
              tr(PH_PER_LAYER * l + 1, 0);
              ok = wait_count(cl + 0, target, &S.ok);
              tr(PH_PER_LAYER * l + 1, 1);
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
              // RoPE of the group's queries (pre-scaled) and of the new key, at position pos:
              // every thread's loads first (one round trip), then the arithmetic
              const float* row = p.qkv + (int64_t)b * d.qkv_rows;
              const bool has_new = pos >= j0 && pos < j1;
              float xv[3], xr[3];
#pragma unroll
              for (int u = 0; u < 3; ++u) {
                const int e = tid + u * NCT;
                xv[u] = xr[u] = 0.f;
                if (e < (hpg + 2) * HD) {
                  const int hh = e / HD, dd = e - hh * HD;
                  const int slot = hh < hpg ? kh * hpg + hh : (hh == hpg ? d.H + kh : d.H + d.Hk + kh);
                  const float* x = row + (int64_t)slot * HD;
                  xv[u] = __ldcg(x + dd);
                  if (hh <= hpg) xr[u] = __ldcg(x + (dd < HD / 2 ? dd + HD / 2 : dd - HD / 2));
                }
              }
#pragma unroll
              for (int u = 0; u < 3; ++u) {
                const int e = tid + u * NCT;
                if (e < (hpg + 2) * HD) {
                  const int hh = e / HD, dd = e - hh * HD;
                  float v = xv[u];
                  if (hh <= hpg) {
                    const float rot = dd < HD / 2 ? -xr[u] : xr[u];
                    v = __fadd_rn(__fmul_rn(v, cs[u]), __fmul_rn(rot, sn[u]));  // x*cos + rotate_half(x)*sin
                  }
                  if (hh < hpg) qs[hh * HD + dd] = v * p.scale;
                  else if (hh == hpg) knew[dd] = v;
                  else vnew[dd] = v;
                }
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
              float* part_base = p.attn_part + ((int64_t)b * d.H + kh * hpg) * d.nch * (HD + 2);
              // scores: warp per query head, lane per key (two keys per lane), the dims rotated
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
                float* part = part_base + ((int64_t)warp * d.nch + ch) * (HD + 2);
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
                __stcg(part_base + ((int64_t)hh * d.nch + ch) * (HD + 2) + dd, o);
              }
              // the last of this (sequence, kv head)'s chunks to finish merges them all
              csync();
              const int nc = (len + KCH - 1) / KCH;
              if (tid == 0) {
                uint32_t old;
                uint32_t* tk = btickets + b * 8 + kh;
                asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(tk) : "memory");
                const bool last = old + 1 == (uint32_t)nc;
                if (last) asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(tk) : "memory");
                S.ticket_last = last;
              }
              csync();
              if (S.ticket_last) {
                // stats of every chunk of the group's heads into shared memory, then per
                // (head, dim): o = sum_c o_c e^{m_c - M} / sum_c l_c e^{m_c - M}
                float* st = sc;  // [hpg][MAXCH][2]
                for (int e = tid; e < hpg * nc; e += NCT) {
                  const int hh = e / nc, cc = e - hh * nc;
                  const float* pc = part_base + ((int64_t)hh * d.nch + cc) * (HD + 2) + HD;
                  st[(hh * MAXCH + cc) * 2] = __ldcg(pc);
                  st[(hh * MAXCH + cc) * 2 + 1] = __ldcg(pc + 1);
                }
                csync();
                for (int e = tid; e < hpg * HD; e += NCT) {
                  const int hh = e / HD, dd = e - hh * HD;
                  float ov[MAXCH];
#pragma unroll
                  for (int cc = 0; cc < MAXCH; ++cc)
                    ov[cc] = cc < nc ? __ldcg(part_base + ((int64_t)hh * d.nch + cc) * (HD + 2) + dd) : 0.f;
                  float M = -INFINITY;
                  for (int cc = 0; cc < nc; ++cc) M = fmaxf(M, st[(hh * MAXCH + cc) * 2]);
                  float o = 0.f, Ls = 0.f;
#pragma unroll
                  for (int cc = 0; cc < MAXCH; ++cc) {
                    if (cc < nc) {
                      const float f = expf(st[(hh * MAXCH + cc) * 2] - M);
                      o = fmaf(ov[cc], f, o);
                      Ls = fmaf(st[(hh * MAXCH + cc) * 2 + 1], f, Ls);
                    }
                  }
                  __stcg(p.attn + (int64_t)b * hid + (kh * hpg + hh) * HD + dd, o / Ls);
                }
              }
            }
            csync();
          }
          tr(PH_PER_LAYER * l + 1, 5);
          csync();
          if (tid == 0) signal(cl + 1);
          tr(PH_PER_LAYER * l + 1, 2);
          tr(PH_PER_LAYER * l + 1, 3);
        }
      }
      if (!ok) break;
      // ---- C: h1 = h + attn . Wo^T ------------------------------------------------------
      {
        Mat m = mC0;
        m.q = L.o_q; m.s = L.o_s;
        const int i0 = first_item(d.off_c, G);
        if (i0 < m.items()) {
          // this CTA's residual rows are final once the previous layer's E has completed
          // (this CTA may not have waited for it yet): then loaded ahead of B's completion
          tr(PH_PER_LAYER * l + 2, 0);
          if (l > 0) ok = wait_count(ctr + PH_PER_LAYER * (l - 1) + 4, (t + 1) * contributors(mE0.items(), G), &S.ok);
          const float res0 = (ok && tid < RT * MAXB && eb < B)
                                 ? __ldcg(p.h + (int64_t)eb * hid + (i0 / m.parts) * RT + erow) : 0.f;
          if (ok) ok = wait_count(cl + 1, (t + 1) * contributors(nB, G), &S.ok);
          tr(PH_PER_LAYER * l + 2, 1);
          if (!ok) break;
          stage_rows(xf, p.attn, hid, B, hid, 0, hid, nullptr, 0.f, S.inv_scale);
          csync();
          tr(PH_PER_LAYER * l + 2, 4);
          ok = run_items(m, i0, [&](int jj, int tile, int, int r, int b, float v, const float*, int) {
            if (b >= B) return;
            const int row = tile * RT + r;
            const float res = jj == 0 ? res0 : __ldcg(p.h + (int64_t)b * hid + row);
            __stcg(p.h1 + (int64_t)b * hid + row, res + v);
          });
          tr(PH_PER_LAYER * l + 2, 5);
          csync();
          if (tid == 0) signal(cl + 2);
          tr(PH_PER_LAYER * l + 2, 2);
          tr(PH_PER_LAYER * l + 2, 3);
        }
      }
      if (!ok) break;
      // ---- D: act = silu(gate) * up of RMSNorm(h1, ln2) . Wgu^T -------------------------
      {
        Mat m = mD0;
        m.q = L.gu_q; m.s = L.gu_s;
        const int i0 = first_item(d.off_d, G);
        if (i0 < m.items()) {
          fetch_norm(L.ln2);
          tr(PH_PER_LAYER * l + 3, 0);
          ok = wait_count(cl + 2, (t + 1) * contributors(mC0.items(), G), &S.ok);
          tr(PH_PER_LAYER * l + 3, 1);
          norm_ready();
          csync();
          if (!ok) break;
          stage_rows(xf, p.h1, hid, B, hid, 0, hid, S.normw, p.eps, S.inv_scale);
          csync();
          tr(PH_PER_LAYER * l + 3, 4);
          ok = run_items(m, i0, [&](int, int tile, int, int r, int b, float v, const float* rj, int wpi) {
            if (b >= B || (r & 1)) return;  // rows 2j (gate) and 2j + 1 (up), interleaved
            float up = 0.f;
            for (int w = 0; w < wpi; ++w) up += rj[w * RT * MAXB + (r + 1) * MAXB + b];
            up *= S.inv_scale[b];
            const int j = (tile * RT + r) >> 1;
            __stcg(p.act + (int64_t)b * d.inter + j, (v / (1.0f + expf(-v))) * up);
          });
          tr(PH_PER_LAYER * l + 3, 5);
          csync();
          if (tid == 0) signal(cl + 3);
          tr(PH_PER_LAYER * l + 3, 2);
          tr(PH_PER_LAYER * l + 3, 3);
        }
      }
      if (!ok) break;
      // ---- E: h = h1 + act . Wdown^T (K parts; the last part of a tile adds them) ---------
      {
        Mat m = mE0;
        m.q = L.dn_q; m.s = L.dn_s;
        const int i0 = first_item(d.off_e, G);
        if (i0 < m.items()) {
          // h1 rows of this CTA's first two items (final since C completed): before the wait
          // (C's completion first: a CTA without D items has not waited for it yet)
          tr(PH_PER_LAYER * l + 4, 0);
          if (mD0.items() < G) ok = wait_count(cl + 2, (t + 1) * contributors(mC0.items(), G), &S.ok);
          // the first two items' rows: thread (tid >> 7) of the pair, row (tid & 127) / 8, sequence tid % 8
          const int pj = tid >> 7, pr = (tid & 127) / MAXB, pb = tid % MAXB;
          const int ipre = i0 + pj * G;
          const float h1pre = (ok && pb < B && ipre < m.items())
                                  ? __ldcg(p.h1 + (int64_t)pb * hid + (ipre / m.parts) * RT + pr) : 0.f;
          if (ok) ok = wait_count(cl + 3, (t + 1) * contributors(mD0.items(), G), &S.ok);
          tr(PH_PER_LAYER * l + 4, 1);
          if (!ok) break;
          // the items of a batch share their K part when the CTA stride is a multiple of the
          // part count (148 and 4 here): one staging for all of them; else one item at a time
          const int nE = (m.items() - 1 - i0) / G + 1;
          const int per = (G % m.parts == 0) ? NCW : 1;
          for (int k = 0; k < nE && ok; k += per) {
            const int nb = min(per, nE - k);
            const int ifirst = i0 + k * G;
            const int part = ifirst % m.parts;
            const int g0 = part * m.gp, ng = min(m.gp, d.inter / 64 - g0);
            csync();  // the previous batch's epilogue has read the staged scales
            stage_rows(xf, p.act, d.inter, B, d.inter, 64 * g0, 64 * ng, nullptr, 0.f, S.inv_scale);
            csync();
            if (k == 0) tr(PH_PER_LAYER * l + 4, 4);
            auto h1_of = [&](int jj, int tl, int r, int b) -> float {
              return (k == 0 && jj < 2) ? h1pre : __ldcg(p.h1 + (int64_t)b * hid + tl * RT + r);
            };
            if (m.parts == 1) {
              ok = run_batch(m, ifirst, nb, [&](int jj, int tl, int, int r, int b, float v, const float*, int) {
                if (b < B) __stcg(p.h + (int64_t)b * hid + tl * RT + r, h1_of(jj, tl, r, b) + v);
              });
              continue;
            }
            ok = run_batch(m, ifirst, nb, [&](int, int tl, int pt, int r, int b, float v, const float*, int) {
              if (b < B) __stcg(p.part + (((int64_t)tl * m.parts + pt) * RT + r) * MAXB + b, v);
            });
            if (!ok) break;
            // one ticket per tile: the last of its K parts to arrive adds the parts in order
            if (tid == 0) {
              int mask = 0;
              for (int jj = 0; jj < nb; ++jj) {
                const int tl = (ifirst + jj * G) / m.parts;
                uint32_t old;
                asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                             : "=r"(old)
                             : "l"(&tickets[l * e_tiles + tl])
                             : "memory");
                if (((old + 1) % (uint32_t)m.parts) == 0) mask |= 1 << jj;
              }
              S.ticket_last = mask;
            }
            csync();
            const int mask = S.ticket_last;
            for (int kk = 0; kk < nb; kk += 2) {
              const int jj = kk + (tid >> 7);
              const int r = (tid & 127) / MAXB, b = tid % MAXB;
              if (jj < nb && ((mask >> jj) & 1) && b < B) {
                const int tl = (ifirst + jj * G) / m.parts;
                float pv[8];
#pragma unroll
                for (int pt = 0; pt < 8; ++pt)
                  pv[pt] = pt < m.parts ? __ldcg(p.part + (((int64_t)tl * m.parts + pt) * RT + r) * MAXB + b) : 0.f;
                float y = 0.f;
#pragma unroll
                for (int pt = 0; pt < 8; ++pt)
                  if (pt < m.parts) y += pv[pt];
                __stcg(p.h + (int64_t)b * hid + tl * RT + r, h1_of(jj, tl, r, b) + y);
              }
            }
          }
          tr(PH_PER_LAYER * l + 4, 5);
          csync();
          if (tid == 0) signal(cl + 4);
          tr(PH_PER_LAYER * l + 4, 2);
          tr(PH_PER_LAYER * l + 4, 3);
        }
      }
    }
    if (!ok) break;
    // ---- F: logits = RMSNorm(h, norm) . Whead^T, with per-tile softmax statistics --------
    {
      const int i0 = first_item(d.off_f, G);
      if (i0 < mF.items()) {
        fetch_norm(p.final_norm);
        tr(nph - 2, 0);
        ok = wait_count(ctr + PH_PER_LAYER * (p.n_layers - 1) + 4, (t + 1) * contributors(mE0.items(), G), &S.ok);
        tr(nph - 2, 1);
        norm_ready();
        csync();
        if (!ok) break;
        stage_rows(xf, p.h, hid, B, hid, 0, hid, S.normw, p.eps, S.inv_scale);
        csync();
        tr(nph - 2, 4);
        const int ntf = mF.items();
        ok = run_items(mF, i0, [&](int, int tile, int, int r, int b, float v, const float*, int) {
            // tid = r * 8 + b: the 16 rows of sequence b sit in lanes b, b + 8, b + 16, b + 24
            // of the four epilogue warps
            const int row = tile * RT + r;
            const bool valid = row < p.vocab && b < B;
            if (valid) __stcg(p.logits + (int64_t)b * p.vocab + row, v);
            float mx = valid ? v : -INFINITY;
            float bx = (valid && row < p.select) ? v : -INFINITY;
            int bi = (valid && row < p.select) ? row : 0x7FFFFFFF;
#pragma unroll
            for (int o = 8; o < 32; o <<= 1) {
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
              const float ov = __shfl_xor_sync(0xffffffffu, bx, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
              if (ov > bx || (ov == bx && oi < bi)) {
                bx = ov;
                bi = oi;
              }
            }
            // two items at a time: threads [0, 128) and [128, 256), each with its own named
            // barrier and scratch ([4 warps][8][3] partials, then [4 warps][8] sums at 96)
            float* fst = S.fst + 128 * (tid >> 7);
            const int w = (tid >> 5) & 3;
            // (the previous item of this thread group has finished reading the scratch)
            asm volatile("bar.sync %0, %1;" ::"r"(2 + (tid >> 7)), "n"(RT * MAXB) : "memory");
            if ((tid & 31) < 8) {
              fst[(w * 8 + b) * 3] = mx;
              fst[(w * 8 + b) * 3 + 1] = bx;
              fst[(w * 8 + b) * 3 + 2] = __int_as_float(bi);
            }
            asm volatile("bar.sync %0, %1;" ::"r"(2 + (tid >> 7)), "n"(RT * MAXB) : "memory");
            float M = -INFINITY;
#pragma unroll
            for (int ww = 0; ww < 4; ++ww) M = fmaxf(M, fst[(ww * 8 + b) * 3]);
            float e = valid ? expf(v - M) : 0.f;
#pragma unroll
            for (int o = 8; o < 32; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
            asm volatile("bar.sync %0, %1;" ::"r"(2 + (tid >> 7)), "n"(RT * MAXB) : "memory");
            if ((tid & 31) < 8) fst[96 + w * 8 + b] = e;
            asm volatile("bar.sync %0, %1;" ::"r"(2 + (tid >> 7)), "n"(RT * MAXB) : "memory");
            if (r == 0 && b < B) {
              float sum = 0.f, BX = -INFINITY;
              int BI = 0x7FFFFFFF;
#pragma unroll
              for (int ww = 0; ww < 4; ++ww) {
                sum += fst[96 + ww * 8 + b];
                const float ov = fst[(ww * 8 + b) * 3 + 1];
                const int oi = __float_as_int(fst[(ww * 8 + b) * 3 + 2]);
                if (ov > BX || (ov == BX && oi < BI)) {
                  BX = ov;
                  BI = oi;
                }
              }
              __stcg(reinterpret_cast<float4*>(p.part) + (int64_t)b * ntf + tile,
                     make_float4(M, sum, BX, __int_as_float(BI)));
            }
          });
        tr(nph - 2, 5);
        csync();
        if (tid == 0) signal(ctr + PH_PER_LAYER * p.n_layers);
        tr(nph - 2, 2);
        tr(nph - 2, 3);
      }
    }
    if (!ok) break;
    // ---- G: token, bookkeeping, next input (one CTA per sequence) -----------------------
    {
      const int i0 = first_item(d.off_g, G);
      if (i0 < B) {
        tr(nph - 1, 0);
        ok = wait_count(ctr + PH_PER_LAYER * p.n_layers, (t + 1) * contributors(mF.items(), G), &S.ok);
        tr(nph - 1, 1);
        if (!ok) break;
        const int ntf = mF.items();
        float* red = redbuf;
        for (int b = i0; b < B; b += G) {
          // the head tiles' statistics: M = max m_i, S = sum s_i e^{m_i - M}, and the best
          // candidate of each tile; the token is the candidate with the largest
          // log-probability (x - M) - lse, lowest id on ties (llm.py:114, np.argmax)
          float4 tv[(6768 / RT + NCT - 1) / NCT];
          constexpr int TU = (6768 / RT + NCT - 1) / NCT;
#pragma unroll
          for (int u = 0; u < TU; ++u) {
            const int it = tid + u * NCT;
            tv[u] = it < ntf ? __ldcg(reinterpret_cast<const float4*>(p.part) + (int64_t)b * ntf + it)
                             : make_float4(-INFINITY, 0.f, -INFINITY, __int_as_float(0x7FFFFFFF));
          }
          for (int it = tid + TU * NCT; it < ntf; it += NCT) {  // larger vocabularies
            const float4 q = __ldcg(reinterpret_cast<const float4*>(p.part) + (int64_t)b * ntf + it);
            if (q.x > tv[0].x) { tv[0].y = tv[0].y * expf(tv[0].x - q.x) + q.y; tv[0].x = q.x; }
            else tv[0].y += q.y * expf(q.x - tv[0].x);
            if (q.z > tv[0].z || (q.z == tv[0].z && __float_as_int(q.w) < __float_as_int(tv[0].w))) {
              tv[0].z = q.z;
              tv[0].w = q.w;
            }
          }
          float mx = -INFINITY;
#pragma unroll
          for (int u = 0; u < TU; ++u) mx = fmaxf(mx, tv[u].x);
          mx = warp_max(mx);
          if (lane == 0) red[warp] = mx;
          csync();
          float M = red[0];
          for (int w = 1; w < NCW; ++w) M = fmaxf(M, red[w]);
          csync();
          float sum = 0.f;
#pragma unroll
          for (int u = 0; u < TU; ++u)
            if (tv[u].x > -INFINITY) sum += tv[u].y * expf(tv[u].x - M);
          sum = warp_sum(sum);
          if (lane == 0) red[warp] = sum;
          csync();
          float Ssum = 0.f;
          for (int w = 0; w < NCW; ++w) Ssum += red[w];
          const float lse = logf(Ssum);
          csync();
          float best = -INFINITY;
          int besti = 0x7FFFFFFF;
#pragma unroll
          for (int u = 0; u < TU; ++u) {
            const int ci = __float_as_int(tv[u].w);
            if (ci != 0x7FFFFFFF) {
              const float lp = (tv[u].z - M) - lse;
              if (lp > best || (lp == best && ci < besti)) {
                best = lp;
                besti = ci;
              }
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
            else
              fail_with(3);
            __stcg(p.pos + b, __ldcg(p.pos + b) + 1);
            __stcg(p.lens + b, __ldcg(p.lens + b) + 1);
          }
          // the log-probabilities, when asked for (every logit once more)
          if (p.logp) {
            const float* src = p.logits + (int64_t)b * p.vocab;
            for (int i0l = tid; i0l < p.vocab; i0l += 8 * NCT) {
              float x8[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) x8[u] = i0l + u * NCT < p.vocab ? __ldcg(src + i0l + u * NCT) : 0.f;
#pragma unroll
              for (int u = 0; u < 8; ++u)
                if (i0l + u * NCT < p.vocab) __stcg(p.logp + (int64_t)b * p.vocab + i0l + u * NCT, (x8[u] - M) - lse);
            }
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
        tr(nph - 1, 2);
        tr(nph - 1, 3);
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
      __stcg(p.step, (int)S.step0 + p.steps);
      __threadfence();
    }
  }
}

}  // namespace

extern "C" int64_t cv3_decode_sync_words(int64_t n_layers, int64_t hidden) {
  // steps done, phase counters, F, G, the down projection's per-tile tickets, the
  // attention merge's per-(sequence, kv head) tickets
  return 1 + PH_PER_LAYER * n_layers + 2 + n_layers * (hidden / RT) + MAXB * 8;
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
                  p.attn_part && p.attn && p.part && p.act && p.logits,
              CV3_ERR_VALUE, "decode_steps: scratch buffers (sync words: %lld needed)",
              (long long)cv3_decode_sync_words(p.n_layers, p.hidden));
  CV3_REQUIRE(p.cap <= (int64_t)MAXCH * KCH, CV3_ERR_UNSUPPORTED, "decode_steps: cap %lld > %d",
              (long long)p.cap, MAXCH * KCH);
  {
    const int64_t ntf = (p.vocab + RT - 1) / RT;
    const int64_t ks = p.inter / 64, parts = (ks + GMAX - 1) / GMAX;
    CV3_REQUIRE(p.part_floats >= 4 * MAXB * ntf && p.part_floats >= (int64_t)(p.hidden / RT) * parts * RT * MAXB,
                CV3_ERR_VALUE, "decode_steps: part scratch of %lld floats too small",
                (long long)p.part_floats);
  }
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

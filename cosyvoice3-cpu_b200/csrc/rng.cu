// PyTorch's CPU random stream on the GPU (cv3cpu/torch_rng.py).
//
// MT19937 is inherently sequential, so one CTA walks the stream: the 624-word
// state is seeded by one thread (init_genrand, torch_rng.py:30-37), then each
// regeneration runs in four dependency-ordered slabs (word i reads word
// i+397 mod 624, which is already regenerated for i >= 227: slabs [0,227),
// [227,454), [454,623) and the last word), every slab fully parallel across
// the CTA.  Tempered words are converted and written coalesced as they are
// produced.  The buffers this feeds (the flow's fixed ODE start and the
// vocoder's NSF dither) are constants per seed, so the stage code draws them
// once and keeps them resident.
//
// Outputs: float32 uniforms from the low 24 bits (torch_rng.py:88-91); normals
// by torch's normal_fill -- 16-element blocks, Box-Muller in float64 pairing
// element j with j+8, the last 16 outputs redrawn from 16 fresh uniforms when
// the count is not a multiple of 16 (torch_rng.py:105-142); below 16 elements
// the scalar float64 path (torch_rng.py:122-133).
#include "common.cuh"

namespace {

constexpr int MT_N = 624, MT_M = 397;
constexpr uint32_t MT_A = 0x9908B0DFu, HI = 0x80000000u, LO = 0x7FFFFFFFu;
constexpr int RT = 256;

__device__ __forceinline__ uint32_t temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9D2C5680u;
  y ^= (y << 15) & 0xEFC60000u;
  y ^= y >> 18;
  return y;
}

__device__ __forceinline__ uint32_t mix(uint32_t cur, uint32_t next, uint32_t far) {
  const uint32_t y = (cur & HI) | (next & LO);
  return far ^ (y >> 1) ^ ((y & 1u) ? MT_A : 0u);
}

// Regenerate `st` in place.  The old word i+1 must be read before slab
// boundaries overwrite it, so every slab first reads, syncs, then writes.
__device__ void regenerate(uint32_t* st) {
  const int lag = MT_N - MT_M;  // 227
  for (int lo = 0; lo < MT_N - 1; lo += lag) {
    const int hi = min(lo + lag, MT_N - 1);
    uint32_t v[3];
    int cnt = 0;
    for (int i = lo + threadIdx.x; i < hi; i += RT) v[cnt++] = mix(st[i], st[i + 1], st[(i + MT_M) % MT_N]);
    __syncthreads();
    cnt = 0;
    for (int i = lo + threadIdx.x; i < hi; i += RT) st[i] = v[cnt++];
    __syncthreads();
  }
  if (threadIdx.x == 0) st[MT_N - 1] = mix(st[MT_N - 1], st[0], st[MT_M - 1]);
  __syncthreads();
}

// mode 0: f32 uniforms; mode 1: raw tempered words (u32); mode 2: f64 uniforms
// from consecutive word pairs (first word high), count = pairs.
__global__ void __launch_bounds__(RT) mt_stream_kernel(uint32_t seed, int64_t skip, int64_t count, int mode,
                                                       void* out) {
  __shared__ uint32_t st[MT_N];
  if (threadIdx.x == 0) {
    st[0] = seed;
    for (int i = 1; i < MT_N; ++i) st[i] = 1812433253u * (st[i - 1] ^ (st[i - 1] >> 30)) + (uint32_t)i;
  }
  __syncthreads();
  const int64_t words = (mode == 2) ? 2 * count : count;
  int64_t pos = 0;  // words consumed so far (including skip)
  const int64_t end = skip + words;
  while (pos < end) {
    regenerate(st);
    const int64_t base = pos;  // stream index of st[0]
    for (int i = threadIdx.x; i < MT_N; i += RT) {
      const int64_t s = base + i;
      if (s < skip || s >= end) continue;
      const int64_t o = s - skip;
      const uint32_t y = temper(st[i]);
      if (mode == 0) {
        reinterpret_cast<float*>(out)[o] = (float)(y & 0xFFFFFFu) * (1.0f / 16777216.0f);
      } else if (mode == 1) {
        reinterpret_cast<uint32_t*>(out)[o] = y;
      } else {
        // word pair (2p, 2p+1) -> double p; assemble via the u32 view first
        reinterpret_cast<uint32_t*>(out)[o] = y;
      }
    }
    pos += MT_N;
    __syncthreads();
  }
}

__global__ void pairs_to_f64_kernel(uint32_t* words, int64_t pairs) {
  double* d = reinterpret_cast<double*>(words);
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < pairs; p += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t v = (((uint64_t)words[2 * p] << 32) | words[2 * p + 1]) & ((1ull << 53) - 1);
    d[p] = (double)v * (1.0 / 9007199254740992.0);
  }
}

__device__ __forceinline__ void box_muller16(const float* u, float* o) {
  double r[8], th[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    r[j] = sqrt(-2.0 * log(1.0 - (double)u[j]));
    th[j] = 2.0 * 3.141592653589793 * (double)u[j + 8];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    o[j] = (float)(r[j] * cos(th[j]));
    o[j + 8] = (float)(r[j] * sin(th[j]));
  }
}

// In-place normal_fill over whole 16-blocks of `buf` (float uniforms in).
__global__ void normal_blocks_kernel(float* buf, int64_t blocks) {
  for (int64_t bi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; bi < blocks; bi += (int64_t)gridDim.x * blockDim.x) {
    float u[16], o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) u[j] = buf[bi * 16 + j];
    box_muller16(u, o);
#pragma unroll
    for (int j = 0; j < 16; ++j) buf[bi * 16 + j] = o[j];
  }
}

// Tail: 16 fresh uniforms -> normals written over the last 16 outputs.
__global__ void normal_tail_kernel(const float* tail_u, float* out_last16) {
  if (threadIdx.x == 0) {
    float u[16], o[16];
    for (int j = 0; j < 16; ++j) u[j] = tail_u[j];
    box_muller16(u, o);
    for (int j = 0; j < 16; ++j) out_last16[j] = o[j];
  }
}

// Scalar path for n < 16: pairs of double uniforms -> (r cos th, r sin th).
__global__ void normal_small_kernel(const double* u, int n, float* out) {
  if (threadIdx.x == 0) {
    const int pairs = (n + 1) / 2;
    for (int p = 0; p < pairs; ++p) {
      const double th = 2.0 * 3.141592653589793 * u[2 * p];
      const double r = sqrt(-2.0 * log1p(-u[2 * p + 1]));
      if (2 * p < n) out[2 * p] = (float)(r * cos(th));
      if (2 * p + 1 < n) out[2 * p + 1] = (float)(r * sin(th));
    }
  }
}

int stream_words(uint64_t seed, int64_t skip, int64_t count, int mode, void* out, cudaStream_t st) {
  mt_stream_kernel<<<1, RT, 0, st>>>((uint32_t)(seed & 0xFFFFFFFFu), skip, count, mode, out);
  return cv3::check_launch("mt19937_stream");
}

}  // namespace

extern "C" int cv3_torch_rand(uint64_t seed, int64_t skip, int64_t n, float* out, void* stream) {
  CV3_REQUIRE(n >= 0 && skip >= 0, CV3_ERR_VALUE, "torch_rand: negative count");
  if (n == 0) return CV3_OK;
  return stream_words(seed, skip, n, 0, out, cv3::as_stream(stream));
}

extern "C" int cv3_torch_u32(uint64_t seed, int64_t skip, int64_t n, uint32_t* out, void* stream) {
  CV3_REQUIRE(n >= 0 && skip >= 0, CV3_ERR_VALUE, "torch_u32: negative count");
  if (n == 0) return CV3_OK;
  return stream_words(seed, skip, n, 1, out, cv3::as_stream(stream));
}

extern "C" int cv3_torch_rand64(uint64_t seed, int64_t skip, int64_t n, double* out, void* stream) {
  CV3_REQUIRE(n >= 0 && skip >= 0, CV3_ERR_VALUE, "torch_rand64: negative count");
  CV3_REQUIRE(((uintptr_t)out & 7) == 0, CV3_ERR_VALUE, "torch_rand64: output must be 8-byte aligned");
  if (n == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  int rc = stream_words(seed, skip, n, 2, out, st);  // 2n words, then each pair -> one double in place
  if (rc) return rc;
  int64_t grid = (n + 255) / 256;
  if (grid > 1024) grid = 1024;
  pairs_to_f64_kernel<<<(unsigned)grid, 256, 0, st>>>(reinterpret_cast<uint32_t*>(out), n);
  return cv3::check_launch("pairs_to_f64");
}

extern "C" int cv3_torch_randn(uint64_t seed, int64_t skip, int64_t n, float* out, void* scratch, void* stream) {
  CV3_REQUIRE(n >= 0 && skip >= 0, CV3_ERR_VALUE, "torch_randn: negative count");
  if (n == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  int rc;
  if (n < 16) {
    // 2*ceil(n/2) double uniforms = 4*ceil(n/2) words; scratch holds 16 doubles.
    const int64_t pairs = (n + 1) / 2;
    CV3_REQUIRE(scratch != nullptr, CV3_ERR_VALUE, "torch_randn: scratch (128 bytes) required");
    rc = stream_words(seed, skip, 2 * pairs, 2, scratch, st);
    if (rc) return rc;
    pairs_to_f64_kernel<<<1, 32, 0, st>>>(reinterpret_cast<uint32_t*>(scratch), 2 * pairs);
    if ((rc = cv3::check_launch("pairs_to_f64"))) return rc;
    normal_small_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const double*>(scratch), (int)n, out);
    return cv3::check_launch("normal_small");
  }
  rc = stream_words(seed, skip, n, 0, out, st);
  if (rc) return rc;
  const int64_t blocks = n / 16;
  int64_t grid = (blocks + 127) / 128;
  if (grid > 4096) grid = 4096;
  normal_blocks_kernel<<<(unsigned)grid, 128, 0, st>>>(out, blocks);
  if ((rc = cv3::check_launch("normal_blocks"))) return rc;
  if (n % 16) {
    CV3_REQUIRE(scratch != nullptr, CV3_ERR_VALUE, "torch_randn: scratch (128 bytes) required");
    rc = stream_words(seed, skip + n, 16, 0, scratch, st);
    if (rc) return rc;
    normal_tail_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const float*>(scratch), out + n - 16);
    return cv3::check_launch("normal_tail");
  }
  return CV3_OK;
}

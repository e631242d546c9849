// Embedding row gathers (cv3cpu/ops.py:126-144): fp32 and fp16 tables are
// gathered and widened; q8 / q4 tables dequantise only the gathered rows
// (float(q) * float(scale), (float(code) - 8) * float(scale): exact).  Ids come from device memory so a token
// chosen on the GPU (greedy argmax) feeds the next step without a host round
// trip.  The host mirror range-checks host ids first (IndexError, as the
// reference); ids outside the table that reach the kernel produce a zero row
// and are counted in *bad (when given), never an out-of-bounds read.
#include "common.cuh"

namespace {

__global__ void embed_kernel(const void* __restrict__ table, int kind, const uint16_t* __restrict__ sc, int64_t rows,
                             int64_t dim, int64_t kp, const int64_t* __restrict__ ids, int64_t n,
                             float* __restrict__ out, int64_t ldo, int* bad) {
  dep_wait();
  dep_release();
  const int64_t i = blockIdx.x;
  if (i >= n) return;
  const int64_t r = ids[i];
  float* o = out + i * ldo;
  const bool ok = r >= 0 && r < rows;
  if (!ok && threadIdx.x == 0 && bad) atomicAdd(bad, 1);
  for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
    float v = 0.f;
    if (ok) {
      if (kind == 0) v = reinterpret_cast<const float*>(table)[r * dim + c];
      else if (kind == 1) v = h2f(reinterpret_cast<const uint16_t*>(table)[r * dim + c]);
      else if (kind == 2) v = (float)reinterpret_cast<const int8_t*>(table)[r * kp + c] * h2f(sc[r * (kp / 64) + c / 64]);
      else {  // q4: byte j of a 32-wide block holds codes j (low) and j + 16 (high)
        const uint8_t byte = reinterpret_cast<const uint8_t*>(table)[r * (kp / 2) + (c >> 5) * 16 + (c & 15)];
        const int code = (c & 31) < 16 ? (byte & 0xF) : (byte >> 4);
        v = ((float)code - 8.0f) * h2f(sc[r * (kp / 32) + (c >> 5)]);
      }
    }
    o[c] = v;
  }
}

}  // namespace

extern "C" int cv3_embedding(const void* table, int kind, const uint16_t* scales, int64_t rows, int64_t dim,
                             int64_t kp, const int64_t* ids, int64_t n, float* out, int64_t ldo, int* bad,
                             void* stream) {
  CV3_REQUIRE(kind >= 0 && kind <= 3, CV3_ERR_VALUE, "embedding: unknown table kind %d", kind);
  CV3_REQUIRE(rows > 0 && dim > 0 && n >= 0 && ldo >= dim, CV3_ERR_VALUE, "embedding: bad shape");
  CV3_REQUIRE(kind != 2 || (scales && kp % 64 == 0 && kp >= dim), CV3_ERR_VALUE, "embedding: bad q8 table");
  CV3_REQUIRE(kind != 3 || (scales && kp % 32 == 0 && kp >= dim), CV3_ERR_VALUE, "embedding: bad q4 table");
  if (n == 0) return CV3_OK;
  CV3_REQUIRE(n <= 0x7FFFFFFF, CV3_ERR_VALUE, "embedding: too many ids");
  const int threads = dim >= 512 ? 256 : 128;
  return cv3::check_launch("embedding", cv3::launch_dep(embed_kernel, dim3((unsigned)n), dim3(threads), 0,
                                                        cv3::as_stream(stream), table, kind, scales, rows, dim, kp,
                                                        ids, n, out, ldo, bad));
}

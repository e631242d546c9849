// Shared helpers for the cv3cuda kernels: status codes, the thread-local error
// message, launch checking and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include <utility>

#include "../../include/cv3cuda.h"

namespace cv3 {

// Records a message for cv3_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Checks the launch that just happened on this thread (and, for launches made
// through an API call that returns its own status, that status).
int check_launch(const char* what, cudaError_t launch_result = cudaSuccess);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs on the current device (cached per device).
int sm_count();

// Sets the dynamic shared memory limit of a kernel once per (kernel, size).
int allow_smem(const void* fn, int bytes);

// Programmatic dependent launch (cv3_set_dependent_launch, on by default) for the
// LM decode step's chain of small kernels: such a launch may start while the
// previous kernel on the stream still runs.  Every kernel launched this way calls
// dep_wait() before it touches anything the previous kernels write (its earlier
// part only reads weights), then dep_release() so that the NEXT kernel may start --
// after the wait, so at most one kernel waits ahead of the running one.
bool dependent_launch_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_dep(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = dependent_launch_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace cv3

// the device side of launch_dep (no-ops for kernels launched normally)
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#define CV3_REQUIRE(cond, code, ...)                  \
  do {                                                \
    if (!(cond)) return ::cv3::fail((code), __VA_ARGS__); \
  } while (0)

#define CV3_CUDA(call)                                                          \
  do {                                                                          \
    cudaError_t e_ = (call);                                                    \
    if (e_ != cudaSuccess)                                                      \
      return ::cv3::fail(CV3_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// ---------------------------------------------------------------------------
// device utilities
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024).  `red` needs 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (wid == 0) v = warp_sum(v);
  if (threadIdx.x == 0) red[0] = v;
  __syncthreads();
  v = red[0];
  return v;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  v = (threadIdx.x < nw) ? red[threadIdx.x] : -INFINITY;
  if (wid == 0) v = warp_max(v);
  if (threadIdx.x == 0) red[0] = v;
  __syncthreads();
  v = red[0];
  return v;
}

// 16-byte streaming load that bypasses L1 (weights are read exactly once).
__device__ __forceinline__ int4 ld_stream16(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float h2f(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// Elementwise activations by CV3_ACT_* code, in the arithmetic order of the
// reference ops (cv3cpu/ops.py:30-118); IEEE-accurate single precision
// transcendentals.  Unknown codes pass x through.
__device__ __forceinline__ float act_apply(int act, float p, float x) {
  switch (act) {
    case CV3_ACT_SILU: return x / (1.0f + expf(-x));
    case CV3_ACT_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case CV3_ACT_GELU_TANH: {
      const float c = 0.7978845608028654f;  // sqrt(2/pi)
      const float inner = x + 0.044715f * x * x * x;
      return 0.5f * x * (1.0f + tanhf(c * inner));
    }
    case CV3_ACT_GELU_ERF: {
      // Abramowitz & Stegun 7.1.26 erf, as the reference evaluates it.
      const float z = x / 1.4142135623730951f;
      const float a = fabsf(z);
      const float t = 1.0f / (1.0f + 0.3275911f * a);
      const float poly = ((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                         0.254829592f;
      const float e = copysignf(1.0f - poly * t * expf(-a * a), z);
      return 0.5f * x * (1.0f + (z == 0.f ? 0.f : e));
    }
    case CV3_ACT_MISH: {
      const float sp = x > 20.0f ? x : log1pf(expf(fminf(x, 20.0f)));
      return x * tanhf(sp);
    }
    case CV3_ACT_ELU: return x > 0.f ? x : p * expm1f(fminf(x, 0.f));
    case CV3_ACT_LEAKY_RELU: return x >= 0.f ? x : x * p;
    case CV3_ACT_TANH: return tanhf(x);
    case CV3_ACT_EXP: return expf(x);
  }
  return x;
}

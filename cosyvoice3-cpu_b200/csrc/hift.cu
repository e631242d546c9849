// HiFT vocoder kernels (cv3cpu/models/hift.py) and small elementwise helpers.
//
// F0 head (hift.py:56-72): the condnet convolutions run in float32 (the
// reference's conv1d casts its float64 inputs), the classifier is a float64
// dot product; |y| is returned rounded to float32 (hift.py:217).
//
// NSF source (hift.py:90-111): per-frame phase increments
// rad = (f0 * h / sr) mod 1 and their running sum are float64 and sequential
// along time (one thread per harmonic, the order of np.cumsum); the sine of a
// frame's phase is shared by the frame's `up` samples, so it is evaluated once
// per (frame, harmonic).  The per-sample kernel then applies the voiced mask,
// the noise amplitude and the fixed uniform dither, the 9 -> 1 projection and
// tanh.
#include "common.cuh"

namespace {

__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }

// x [B][C][T] float32 -> f0 [B][T] = float32(|sum_c double(x) * w[c] + b|)
__global__ void f0_classifier_kernel(const float* __restrict__ x, int C, int T, const double* __restrict__ w,
                                     const double* __restrict__ b, float* __restrict__ f0, int batch) {
  const int64_t total = (int64_t)batch * T;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bb = i / T, t = i - bb * T;
    const float* xb = x + bb * C * T + t;
    double acc = 0.0;
    for (int c = 0; c < C; ++c) acc = fma((double)xb[(int64_t)c * T], w[c], acc);
    f0[i] = (float)fabs(acc + b[0]);
  }
}

// sines[b][t][h] = float32(sin(phase)) * alpha with phase = cumsum_t(rad) * 2pi * up.
__global__ void nsf_phase_kernel(const float* __restrict__ f0, int T, int harm, int sr, int up, float alpha,
                                 float* __restrict__ sines, int batch) {
  const int b = blockIdx.x;
  const int h = threadIdx.x;
  if (b >= batch || h >= harm) return;
  const float* fb = f0 + (int64_t)b * T;
  float* sb = sines + (int64_t)b * T * harm;
  double cum = 0.0;
  for (int t = 0; t < T; ++t) {
    double rad = ((double)fb[t] * (double)(h + 1)) / (double)sr;
    rad = fmod(rad, 1.0);
    if (rad < 0) rad += 1.0;
    cum += rad;
    const double phase = cum * 6.283185307179586 * (double)up;
    sb[(int64_t)t * harm + h] = mul((float)sin(phase), alpha);
  }
}

// source[b][s] = tanh(sum_h (sines*uv + amp*noise[s][h]) * w[h] + bias), s < up*T.
__global__ void nsf_source_kernel(const float* __restrict__ f0, const float* __restrict__ sines,
                                  const float* __restrict__ noise, int T, int harm, int up, float sigma,
                                  float noise_uv0, float vthr, const float* __restrict__ w, const float* __restrict__ bias,
                                  float* __restrict__ out, int batch) {
  const int64_t S = (int64_t)up * T;
  const int64_t total = (int64_t)batch * S;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / S, s = i - b * S;
    const int64_t t = s / up;
    const float uv = f0[b * T + t] > vthr ? 1.0f : 0.0f;
    const float amp = add(mul(uv, sigma), mul(1.0f - uv, noise_uv0));
    const float* sn = sines + (b * T + t) * harm;
    const float* nz = noise + s * harm;
    float acc = 0.f;
    for (int h = 0; h < harm; ++h) {
      const float sw = add(mul(sn[h], uv), mul(amp, nz[h]));
      acc = fmaf(sw, w[h], acc);
    }
    out[i] = tanhf(acc + bias[0]);
  }
}

// y = op(a, b): 0 add, 1 subtract, 2 multiply; 3: a / scalar; 4: a * scalar.
__global__ void binary_kernel(int op, const float* __restrict__ a, const float* __restrict__ b, float s, int64_t n,
                              float* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v;
    switch (op) {
      case 0: v = add(a[i], b[i]); break;
      case 1: v = __fsub_rn(a[i], b[i]); break;
      case 2: v = mul(a[i], b[i]); break;
      case 3: v = __fdiv_rn(a[i], s); break;
      default: v = mul(a[i], s); break;
    }
    y[i] = v;
  }
}

// y [rows][t+1] = [x[:, 1], x]  (ReflectionPad1d((1, 0)), hift.py:144)
__global__ void reflect_left1_kernel(const float* __restrict__ x, int64_t rows, int64_t t, float* __restrict__ y) {
  const int64_t total = rows * (t + 1);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (t + 1), c = i - r * (t + 1);
    y[i] = x[r * t + (c == 0 ? 1 : c - 1)];
  }
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)cv3::sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

extern "C" int cv3_f0_classifier(const float* x, int64_t batch, int64_t channels, int64_t t, const double* w,
                                 const double* b, float* f0, void* stream) {
  CV3_REQUIRE(batch >= 0 && channels > 0 && t >= 0, CV3_ERR_VALUE, "f0_classifier: bad shape");
  if (batch * t == 0) return CV3_OK;
  f0_classifier_kernel<<<grid_for(batch * t, 128), 128, 0, cv3::as_stream(stream)>>>(x, (int)channels, (int)t, w, b,
                                                                                      f0, (int)batch);
  return cv3::check_launch("f0_classifier");
}

extern "C" int cv3_nsf_source(const float* f0, int64_t batch, int64_t t, int64_t harmonics, int64_t sample_rate,
                              int64_t up, double alpha, double sigma, double voiced_threshold, const float* noise,
                              const float* w, const float* bias, float* sines_scratch, float* out, void* stream) {
  CV3_REQUIRE(batch >= 0 && t >= 0 && harmonics > 0 && harmonics <= 1024 && sample_rate > 0 && up > 0,
              CV3_ERR_VALUE, "nsf_source: bad shape");
  if (batch * t == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  nsf_phase_kernel<<<(unsigned)batch, ((int)harmonics + 31) / 32 * 32, 0, st>>>(f0, (int)t, (int)harmonics,
                                                                                (int)sample_rate, (int)up,
                                                                                (float)alpha, sines_scratch, (int)batch);
  int rc = cv3::check_launch("nsf_phase");
  if (rc) return rc;
  // amplitudes as the reference forms them: uv * sigma + (1 - uv) * (alpha / 3)
  nsf_source_kernel<<<grid_for(batch * t * up, 256), 256, 0, st>>>(
      f0, sines_scratch, noise, (int)t, (int)harmonics, (int)up, (float)sigma, (float)(alpha / 3.0),
      (float)voiced_threshold, w, bias, out, (int)batch);
  return cv3::check_launch("nsf_source");
}

extern "C" int cv3_binary(int op, const float* a, const float* b, float scalar, int64_t n, float* y, void* stream) {
  CV3_REQUIRE(op >= 0 && op <= 4 && n >= 0, CV3_ERR_VALUE, "binary: bad op");
  if (n == 0) return CV3_OK;
  binary_kernel<<<grid_for(n, 256), 256, 0, cv3::as_stream(stream)>>>(op, a, b, scalar, n, y);
  return cv3::check_launch("binary");
}

extern "C" int cv3_reflect_left1(const float* x, int64_t rows, int64_t t, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && t >= 2, CV3_ERR_VALUE, "reflect_left1: need at least 2 frames");
  if (rows == 0) return CV3_OK;
  reflect_left1_kernel<<<grid_for(rows * (t + 1), 256), 256, 0, cv3::as_stream(stream)>>>(x, rows, t, y);
  return cv3::check_launch("reflect_left1");
}

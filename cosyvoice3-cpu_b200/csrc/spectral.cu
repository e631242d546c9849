// Short-time Fourier transforms and resampling helpers (fp32).
//
// STFT (cv3cpu/ops.py:346-355): reflect-padded frames of n_fft samples every
// hop, times the window, one-sided DFT evaluated directly with a twiddle table
// (n_fft is 16 on the vocoder path, so a direct DFT per frame beats an FFT).
// Output is the real and imaginary halves stacked: out[b][f] = Re X_f,
// out[b][F + f] = Im X_f, F = n_fft/2 + 1 -- the (18, frames) tensor the
// vocoder consumes (cv3cpu/models/hift.py:198-199).
//
// iSTFT head (cv3cpu/models/hift.py:204-210 + cv3cpu/ops.py:358-377): from the
// (2F, frames) conv_post output, magnitude = min(exp(min(x, 80)), 100) and
// phase = sin(x'), then the inverse one-sided DFT of each frame, window,
// overlap-add normalised by the summed squared window where it exceeds 1e-11,
// centre trim and clip.  Overlap-add is a gather: every output sample sums its
// (at most n_fft/hop) frames in ascending tap order, as the reference's
// per-tap strided adds do.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int NFFT_MAX = 64;

struct Twiddles {
  float cosv[NFFT_MAX];  // cos(2 pi i / n)
  float sinv[NFFT_MAX];
};

__global__ void stft_kernel(const float* __restrict__ x, int64_t len, int n_fft, int hop, const float* __restrict__ win,
                            Twiddles tw, int64_t frames, float* __restrict__ out) {
  const int nbin = n_fft / 2 + 1;
  const int b = blockIdx.y;
  const float* xb = x + (int64_t)b * len;
  float* ob = out + (int64_t)b * 2 * nbin * frames;
  const int half = n_fft / 2;
  for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < frames; f += (int64_t)gridDim.x * blockDim.x) {
    float seg[NFFT_MAX];
    for (int j = 0; j < n_fft; ++j) {
      int64_t p = f * hop + j - half;  // index into the unpadded signal, reflect at both ends
      if (p < 0) p = -p;
      if (p >= len) p = 2 * (len - 1) - p;
      seg[j] = xb[p] * win[j];
    }
    for (int kf = 0; kf < nbin; ++kf) {
      float re = 0.f, im = 0.f;
      for (int j = 0; j < n_fft; ++j) {
        const int idx = (kf * j) % n_fft;
        re = fmaf(seg[j], tw.cosv[idx], re);
        im = fmaf(-seg[j], tw.sinv[idx], im);
      }
      ob[(int64_t)kf * frames + f] = re;
      ob[(int64_t)(nbin + kf) * frames + f] = im;
    }
  }
}

// Windowed time samples of every frame: frames_out[b][f][j].
__global__ void istft_frames_kernel(const float* __restrict__ spec, int mode, int64_t frames, int n_fft,
                                    const float* __restrict__ win, Twiddles tw, float* __restrict__ fr) {
  const int nbin = n_fft / 2 + 1;
  const int b = blockIdx.y;
  const float* sb = spec + (int64_t)b * 2 * nbin * frames;
  float* fb = fr + (int64_t)b * frames * n_fft;
  for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < frames; f += (int64_t)gridDim.x * blockDim.x) {
    float re[NFFT_MAX / 2 + 1], im[NFFT_MAX / 2 + 1];
    for (int kf = 0; kf < nbin; ++kf) {
      const float a = sb[(int64_t)kf * frames + f], c = sb[(int64_t)(nbin + kf) * frames + f];
      if (mode == 1) {
        // np.minimum / np.clip propagate NaN (hift.py:206); fminf would drop it
        const float e = expf(a > 80.0f ? 80.0f : a);
        const float mag = e > 100.0f ? 100.0f : e;
        const float ph = sinf(c);
        re[kf] = mag * cosf(ph);
        im[kf] = mag * sinf(ph);
      } else {
        re[kf] = a;
        im[kf] = c;
      }
    }
    for (int j = 0; j < n_fft; ++j) {
      // irfft: DC and Nyquist real parts once, interior bins twice; imaginary
      // parts of DC and Nyquist are ignored.
      float acc = re[0];
      for (int kf = 1; kf < nbin - 1; ++kf) {
        const int idx = (kf * j) % n_fft;
        acc += 2.0f * (re[kf] * tw.cosv[idx] - im[kf] * tw.sinv[idx]);
      }
      acc += re[nbin - 1] * ((j & 1) ? -1.0f : 1.0f);
      fb[f * n_fft + j] = (acc / (float)n_fft) * win[j];
    }
  }
}

__global__ void istft_ola_kernel(const float* __restrict__ fr, int64_t frames, int n_fft, int hop,
                                 const float* __restrict__ win, int64_t offset, int64_t out_len, float limit,
                                 float* __restrict__ y) {
  const int b = blockIdx.y;
  const float* fb = fr + (int64_t)b * frames * n_fft;
  float* yb = y + (int64_t)b * out_len;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < out_len; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = t + offset;  // position in the untrimmed overlap-add signal
    float acc = 0.f, env = 0.f;
    for (int j = (int)(p % hop); j < n_fft; j += hop) {
      const int64_t f = (p - j) / hop;
      if (f < 0 || f >= frames) continue;
      acc += fb[f * n_fft + j];
      env += win[j] * win[j];
    }
    float v = fabsf(env) > 1e-11f ? acc / env : acc;
    v = v < -limit ? -limit : (v > limit ? limit : v);  // np.clip: NaN stays NaN
    yb[t] = v;
  }
}

__global__ void nearest_kernel(const float* __restrict__ x, int64_t rows, int64_t t, int scale, float* __restrict__ y) {
  const int64_t total = rows * t * scale;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (t * scale), c = i - r * t * scale;
    y[i] = x[r * t + c / scale];
  }
}

__global__ void linear_interp_kernel(const float* __restrict__ x, int64_t rows, int64_t t, const int64_t* __restrict__ i0,
                                     const int64_t* __restrict__ i1, const float* __restrict__ w, int64_t size,
                                     float* __restrict__ y) {
  const int64_t total = rows * size;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / size, c = i - r * size;
    const float a = x[r * t + i0[c]], bb = x[r * t + i1[c]];
    y[i] = a * (1.0f - w[c]) + bb * w[c];
  }
}

unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)cv3::sm_count() * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

Twiddles make_twiddles(int n) {
  Twiddles tw;
  for (int i = 0; i < NFFT_MAX; ++i) {
    const double a = 2.0 * 3.14159265358979323846 * (double)i / (double)n;
    tw.cosv[i] = (float)cos(a);
    tw.sinv[i] = (float)sin(a);
  }
  return tw;
}

}  // namespace

extern "C" int cv3_stft(const float* x, int64_t batch, int64_t len, int64_t n_fft, int64_t hop, const float* win,
                        float* out, int64_t frames, void* stream) {
  CV3_REQUIRE(n_fft >= 2 && n_fft <= NFFT_MAX && n_fft % 2 == 0 && hop > 0, CV3_ERR_UNSUPPORTED,
              "stft: n_fft %lld not built", (long long)n_fft);
  CV3_REQUIRE(len > n_fft / 2, CV3_ERR_VALUE, "stft: signal of %lld samples too short for reflect padding",
              (long long)len);
  CV3_REQUIRE(frames == 1 + (len + 2 * (n_fft / 2) - n_fft) / hop, CV3_ERR_VALUE, "stft: wrong frame count");
  if (batch == 0) return CV3_OK;
  dim3 grid(grid_for(frames, 128), (unsigned)batch);
  stft_kernel<<<grid, 128, 0, cv3::as_stream(stream)>>>(x, len, (int)n_fft, (int)hop, win, make_twiddles((int)n_fft),
                                                        frames, out);
  return cv3::check_launch("stft");
}

extern "C" int cv3_istft(const float* spec, int mode, int64_t batch, int64_t frames, int64_t n_fft, int64_t hop,
                         const float* win, float limit, int64_t offset, float* frame_scratch, float* y,
                         int64_t out_len, void* stream) {
  CV3_REQUIRE(n_fft >= 2 && n_fft <= NFFT_MAX && n_fft % 2 == 0 && hop > 0, CV3_ERR_UNSUPPORTED,
              "istft: n_fft %lld not built", (long long)n_fft);
  CV3_REQUIRE(mode == 0 || mode == 1, CV3_ERR_VALUE, "istft: unknown mode %d", mode);
  CV3_REQUIRE(frames >= 1 && offset >= 0 && out_len >= 0 && offset + out_len <= (frames - 1) * hop + n_fft,
              CV3_ERR_VALUE, "istft: output window outside the overlap-add signal");
  if (batch == 0) return CV3_OK;
  cudaStream_t st = cv3::as_stream(stream);
  Twiddles tw = make_twiddles((int)n_fft);
  istft_frames_kernel<<<dim3(grid_for(frames, 128), (unsigned)batch), 128, 0, st>>>(spec, mode, frames, (int)n_fft,
                                                                                    win, tw, frame_scratch);
  int rc = cv3::check_launch("istft_frames");
  if (rc) return rc;
  if (out_len == 0) return CV3_OK;
  istft_ola_kernel<<<dim3(grid_for(out_len, 256), (unsigned)batch), 256, 0, st>>>(
      frame_scratch, frames, (int)n_fft, (int)hop, win, offset, out_len, limit, y);
  return cv3::check_launch("istft_ola");
}

extern "C" int cv3_interpolate_nearest(const float* x, int64_t rows, int64_t t, int64_t scale, float* y,
                                       void* stream) {
  CV3_REQUIRE(rows >= 0 && t >= 0 && scale >= 1, CV3_ERR_VALUE, "interpolate_nearest: bad shape");
  if (rows * t == 0) return CV3_OK;
  nearest_kernel<<<grid_for(rows * t * scale, 256), 256, 0, cv3::as_stream(stream)>>>(x, rows, t, (int)scale, y);
  return cv3::check_launch("interpolate_nearest");
}

extern "C" int cv3_interpolate_linear(const float* x, int64_t rows, int64_t t, const int64_t* i0, const int64_t* i1,
                                      const float* w, int64_t size, float* y, void* stream) {
  CV3_REQUIRE(rows >= 0 && t >= 1 && size >= 0, CV3_ERR_VALUE, "interpolate_linear: bad shape");
  if (rows * size == 0) return CV3_OK;
  linear_interp_kernel<<<grid_for(rows * size, 256), 256, 0, cv3::as_stream(stream)>>>(x, rows, t, i0, i1, w, size, y);
  return cv3::check_launch("interpolate_linear");
}

// ---------------------------------------------------------------------------
// iSTFT without any device allocation.
//
// Some callers cannot allocate device memory at the moment they need the
// vocoder's inverse STFT: a real-time audio callback must not block on
// cudaMalloc (it can synchronise the device and take unbounded time), and a
// host that has already handed the whole GPU to its own memory pool has no
// allocation left to give.  cv3_istft asks for a caller-provided frame buffer;
// this variant brings its own, a fixed array in the library's device image.
//
// Limits: batch * frames * n_fft <= kIstftScratchFloats (1 Mi floats, 4 MiB,
// enough for one utterance of about 27 s of 24 kHz audio at n_fft 16 / hop 4).
// Every device that loads the library holds the array until the process exits.
// All calls share it: two calls whose kernels can run at the same time (for
// example on two streams without ordering) overwrite each other's frames, so
// such calls must be ordered by the caller.  Each call writes every frame
// sample before reading it, so stale contents from a previous call never
// reach an output and nothing needs clearing.
// ---------------------------------------------------------------------------

namespace {
constexpr int64_t kIstftScratchFloats = int64_t(1) << 20;
}  // namespace

static __device__ __align__(256) float g_istft_scratch[kIstftScratchFloats];

namespace {

constexpr int kMaxDevices = 64;

// Device address of g_istft_scratch for the current device, looked up once
// per device with that device current (a host-side symbol is not a device
// address, so it must never be passed to a kernel directly).  The lookup
// happens inside the first cv3_istft_noalloc call on each device; make that
// first call before any stream capture (a first call on a capturing stream is
// refused: the lookup may load the module, which a capture does not allow).
int istft_scratch_address(cudaStream_t stream, float** out) {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  int dev = 0;
  CV3_CUDA(cudaGetDevice(&dev));
  CV3_REQUIRE(dev >= 0 && dev < kMaxDevices, CV3_ERR_UNSUPPORTED, "istft_noalloc: device index %d", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    CV3_CUDA(cudaStreamIsCapturing(stream, &cap));
    CV3_REQUIRE(cap == cudaStreamCaptureStatusNone, CV3_ERR_VALUE,
                "istft_noalloc: the first call on device %d must come before any stream capture "
                "(it looks up the frame buffer's device address)", dev);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_istft_scratch);
    CV3_REQUIRE(e == cudaSuccess && p != nullptr, CV3_ERR_CUDA, "istft_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return CV3_OK;
}

}  // namespace

extern "C" int cv3_istft_noalloc(const float* spec, int mode, int64_t batch, int64_t frames, int64_t n_fft,
                                 int64_t hop, const float* win, float limit, int64_t offset, float* y,
                                 int64_t out_len, void* stream) {
  CV3_REQUIRE(batch >= 0 && frames >= 0 && n_fft >= 0, CV3_ERR_VALUE, "istft_noalloc: negative size");
  CV3_REQUIRE(batch == 0 || frames == 0 || n_fft <= kIstftScratchFloats / batch / frames, CV3_ERR_VALUE,
              "istft_noalloc: %lld x %lld frames of %lld samples exceed the built-in %lld-float frame buffer; "
              "use cv3_istft with a caller-provided buffer",
              (long long)batch, (long long)frames, (long long)n_fft, (long long)kIstftScratchFloats);
  float* scratch = nullptr;
  const int rc = istft_scratch_address(cv3::as_stream(stream), &scratch);
  if (rc) return rc;
  return cv3_istft(spec, mode, batch, frames, n_fft, hop, win, limit, offset, scratch, y, out_len, stream);
}

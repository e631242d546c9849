// Library-level entry points and the error convention shared by every kernel file.
#include <atomic>
#include <string>
#include <mutex>
#include <map>
#include <utility>

#include "common.cuh"

namespace cv3 {

static thread_local std::string g_last_error;
static std::atomic<unsigned long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error.assign(buf);
  return code;
}

int check_launch(const char* what, cudaError_t launch_result) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = launch_result;
  if (e != cudaSuccess) return fail(CV3_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return CV3_OK;
}

int sm_count() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  cache[dev] = n;
  return n;
}

int allow_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  CV3_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(dev, fn);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return CV3_OK;
  CV3_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done[key] = bytes;
  return CV3_OK;
}

}  // namespace cv3

extern "C" const char* cv3_last_error(void) { return cv3::g_last_error.c_str(); }

extern "C" int cv3_abi_version(void) { return CV3_ABI_VERSION; }

static int g_dependent_launch = 1;

bool cv3::dependent_launch_enabled() { return g_dependent_launch != 0; }

extern "C" int cv3_set_dependent_launch(int enable) {
  g_dependent_launch = enable ? 1 : 0;
  return CV3_OK;
}

extern "C" unsigned long long cv3_launch_count(void) { return cv3::g_launches.load(std::memory_order_relaxed); }

extern "C" int cv3_device_info(int* sm, int* major, int* minor) {
  int dev = 0;
  CV3_CUDA(cudaGetDevice(&dev));
  cudaDeviceProp p;
  CV3_CUDA(cudaGetDeviceProperties(&p, dev));
  if (sm) *sm = p.multiProcessorCount;
  if (major) *major = p.major;
  if (minor) *minor = p.minor;
  return CV3_OK;
}

// ---------------------------------------------------------------------------
// Device memory, copies and stream order for hosts without a GPU framework: the
// NumPy + ctypes host of the ops layer allocates its device arrays and moves data
// through these (plain cudaMalloc / cudaMemcpyAsync, one copy per call).
// ---------------------------------------------------------------------------

extern "C" int cv3_device_alloc(int64_t bytes, void** ptr) {
  CV3_REQUIRE(ptr && bytes >= 0, CV3_ERR_VALUE, "device_alloc: bad arguments");
  *ptr = nullptr;
  if (bytes == 0) return CV3_OK;
  CV3_CUDA(cudaMalloc(ptr, (size_t)bytes));
  return CV3_OK;
}

extern "C" int cv3_device_free(void* ptr) {
  if (ptr) CV3_CUDA(cudaFree(ptr));
  return CV3_OK;
}

// kind: 0 host -> device, 1 device -> host, 2 device -> device; stream-ordered (a copy
// from or to pageable host memory returns once the host side may be reused)
extern "C" int cv3_memcpy(void* dst, const void* src, int64_t bytes, int kind, void* stream) {
  CV3_REQUIRE(bytes >= 0 && kind >= 0 && kind <= 2 && (bytes == 0 || (dst && src)), CV3_ERR_VALUE,
              "memcpy: bad arguments");
  if (bytes == 0) return CV3_OK;
  const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice
                                     : (kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice);
  CV3_CUDA(cudaMemcpyAsync(dst, src, (size_t)bytes, k, cv3::as_stream(stream)));
  return CV3_OK;
}

extern "C" int cv3_memset(void* dst, int value, int64_t bytes, void* stream) {
  CV3_REQUIRE(bytes >= 0 && (bytes == 0 || dst), CV3_ERR_VALUE, "memset: bad arguments");
  if (bytes == 0) return CV3_OK;
  CV3_CUDA(cudaMemsetAsync(dst, value, (size_t)bytes, cv3::as_stream(stream)));
  return CV3_OK;
}

extern "C" int cv3_stream_synchronize(void* stream) {
  CV3_CUDA(cudaStreamSynchronize(cv3::as_stream(stream)));
  return CV3_OK;
}

extern "C" int cv3_mem_get_info(int64_t* free_bytes, int64_t* total_bytes) {
  size_t f = 0, t = 0;
  CV3_CUDA(cudaMemGetInfo(&f, &t));
  if (free_bytes) *free_bytes = (int64_t)f;
  if (total_bytes) *total_bytes = (int64_t)t;
  return CV3_OK;
}

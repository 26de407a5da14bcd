// Host helpers: thread-local error text, launch checks, device properties,
// driver entry points.
#include <atomic>
#include <mutex>
#include <string.h>

#include "host.cuh"

namespace ssd {

static thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<int64_t> g_launches{0};

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(SSD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return SSD_OK;
}

int device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("SSD_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

TensorMapEncodeFn tensor_map_encoder() {
  static TensorMapEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TensorMapEncodeFn>(p);
  });
  return fn;
}

}  // namespace ssd

extern "C" {

int ssd_version(void) { return 1; }

int64_t ssd_launch_count(void) { return ssd::g_launches.load(std::memory_order_relaxed); }

const char* ssd_last_error(void) { return ssd::g_err; }

int ssd_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

}  // extern "C"

// ssd_linear_noalloc: the fused linear entry point for callers that cannot
// allocate device memory.
//
// Some callers of this library cannot call cudaMalloc (or any allocator) at
// the point where they run a projection: an inference server that reserves
// all device memory at start-up and forbids later allocations, a host
// runtime that owns no allocator of its own (a plain C caller linking only
// this .so), or code that must not trigger the allocator's implicit
// synchronisation. ssd_linear needs a caller-provided workspace for its
// split-K partials; this variant takes none. Its scratch is the fixed-size
// array below, part of the library's device image: every GPU that loads the
// library holds these kNoAllocScratchBytes until the process exits.
//
// Sharing rules: all calls on a device use the same array and it keeps the
// last call's contents. Each call clears the split counters it needs before
// its GEMM launch (an asynchronous memset on the caller's stream, not an
// allocation). Calls whose executions overlap on the GPU (different streams
// without ordering between them) race on the array and give wrong results;
// order them on one stream.
//
// Set-up: the first call on each device, with that device current, looks up
// the array's device address with cudaGetSymbolAddress (which can load the
// library's module on that device). Make that first call before any stream
// capture begins.
#include <mutex>

#include "gemm.cuh"
#include "host.cuh"

namespace ssd {

// 20 MiB: the split counters (256 KiB) plus the split-K partials of any call
// of up to 64 token rows on a GPU of up to 148 SMs. A split GEMM runs at most
// 4 CTAs per SM (tiles x splits <= 4 x SMs), each with one 128-row fp32
// partial tile of at most 64 token columns: 4 x 148 x 128 x 64 x 4 bytes =
// 18.5 MiB (the opt-in stream-K variant needs the same: 2 x 2 x SMs tiles).
// fp32 weights use 4-token tiles, so 64 rows need the same bound.
// Each call computes its exact need first and refuses what does not fit.
constexpr int64_t kNoAllocScratchBytes = 20LL << 20;
constexpr int kNoAllocMaxRows = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch array on the current device (looked up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(SSD_ERR_CUDA, "ssd_linear_noalloc: cannot query the current device");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || !p)
      return fail(SSD_ERR_CUDA, "ssd_linear_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SSD_OK;
}
}  // namespace

}  // namespace ssd

using namespace ssd;

extern "C" int ssd_linear_noalloc(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
                                  const int64_t* rows, const void* const* bias, int seg_layout, int epilogue, int act,
                                  void* out, int64_t ldo, float* resid, int64_t ldr, int dtype, uint32_t* status,
                                  void* stream) {
  if (T <= 0 || T > kNoAllocMaxRows)
    return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_noalloc: T = %lld token rows is outside 1..%d (its fixed %lld-byte "
                "scratch holds decode-sized calls only; use ssd_linear with a workspace)",
                (long long)T, kNoAllocMaxRows, (long long)kNoAllocScratchBytes);
  if (!w || !rows || n_seg < 1 || n_seg > 3) return fail(SSD_ERR_INVALID, "ssd_linear_noalloc: bad weight segments");
  const int64_t need = gemm_workspace_need(T, K, n_seg, rows, seg_layout, false, dtype);
  if (need > kNoAllocScratchBytes)
    return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_noalloc: this shape needs %lld bytes of split-K scratch on this GPU, "
                "more than the fixed %lld-byte array; use ssd_linear with a workspace",
                (long long)need, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The split counters must start at zero for this call.
  if (cudaMemsetAsync(scratch, 0, kCounterBytes, s) != cudaSuccess)
    return fail(SSD_ERR_CUDA, "ssd_linear_noalloc: clearing the split counters failed");
  return ssd_linear(x, ldx, T, K, n_seg, w, rows, bias, seg_layout, epilogue, act, out, ldo, resid, ldr, dtype,
                    scratch, kNoAllocScratchBytes, nullptr, nullptr, status, stream);
}

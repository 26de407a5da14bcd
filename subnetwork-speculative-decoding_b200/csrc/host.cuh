// Host-side helpers shared by the C-ABI entry points: error reporting,
// device properties and the driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <utility>

#include "../../include/ssd_b200.h"

namespace ssd {

// Stores a printf-style message for ssd_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps the last CUDA launch error to a status.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int device_sms();

typedef CUresult (*TensorMapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
TensorMapEncodeFn tensor_map_encoder();
// Lets `kern` use all the shared memory a block may have: 227 KB minus the
// kernel's static shared memory (the attribute call fails outright if the
// sum would exceed the limit, which would leave the 48 KB default).
template <typename Kern>
inline void allow_max_dynamic_smem(Kern kern) {
  cudaFuncAttributes at{};
  cudaFuncGetAttributes(&at, kern);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - (int)at.sharedSizeBytes);
}
// Cached 2-D bf16 tensor map: rows of `inner` elements, box {64, box_outer},
// 128-byte swizzle (the K-major tcgen05 operand layout).
int tma_map_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_outer,
                    CUtensorMap* out);

struct EpiArgs;
// Shared GEMM launcher (gemm.cu). `partial_offset_bytes` reserves the start
// of the partials region for a caller (the lm_head heads keep their per-tile
// records there).
int launch_gemm(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
                const int64_t* rows, int layout, const EpiArgs& epi, int dtype, void* workspace,
                int64_t workspace_bytes, uint32_t* status, cudaStream_t stream, int64_t partial_offset_bytes);

// Workspace bytes (split counters + split-K partials) that launch_gemm needs
// for this shape on the current device with no partial offset: 0 when the GEMM
// does not split, -1 for invalid arguments. `head` = an lm_head epilogue
// (argmax / top-k records), which never splits.
int64_t gemm_workspace_need(int64_t T, int64_t K, int n_seg, const int64_t* rows, int layout, bool head, int dtype);

constexpr int64_t kMaxCounters = 1 << 16;
constexpr int64_t kCounterBytes = kMaxCounters * 4;

// Whether launches carry the programmatic-dependent-launch attribute
// (default on; SSD_PDL=0 turns it off for A/B timing).
bool pdl_enabled();

// Launch `kern` with programmatic stream serialization (see pdl_wait in
// common.cuh) and, if cluster_x * cluster_y > 1, a thread-block cluster.
template <typename... KArgs, typename... Args>
int launch_kernel(const char* name, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                  unsigned cluster_x, unsigned cluster_y, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++n;
  if (cluster_x * cluster_y > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (err != cudaSuccess) return fail(SSD_ERR_CUDA, "%s launch: %s", name, cudaGetErrorString(err));
  return check_launch(name);
}

}  // namespace ssd

// Host-side helpers shared by the C-ABI entry points: error reporting,
// device properties and the driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

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

struct EpiArgs;
// Shared GEMM launcher (gemm.cu). `partial_offset_bytes` reserves the start
// of the partials region for a caller (the lm_head heads keep their per-tile
// records there).
int launch_gemm(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
                const int64_t* rows, int layout, const EpiArgs& epi, int dtype, void* workspace,
                int64_t workspace_bytes, uint32_t* status, cudaStream_t stream, int64_t partial_offset_bytes);

constexpr int64_t kMaxCounters = 1 << 16;
constexpr int64_t kCounterBytes = kMaxCounters * 4;

}  // namespace ssd

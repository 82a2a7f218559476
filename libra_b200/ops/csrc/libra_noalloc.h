// Allocation-free C entry points of libra_b200's CUDA library.
//
// libra_rmsnorm_bwd_noalloc has no counterpart in the reference framework; it
// exists for callers that must not allocate device memory: C or C++ code that
// calls the kernel through this plain C symbol (dlopen of the extension module;
// the module itself still links libtorch, so its shared libraries must be
// loadable) from a context where neither PyTorch's caching allocator nor a
// fresh cudaMalloc is acceptable, such as a step that runs with the device at
// its memory limit (a recovery path after an out-of-memory error), where
// cudaMalloc would fail or implicitly synchronize the device.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// RMSNorm backward, the same operation as libra::rmsnorm_bwd:
//   xhat = x * rstd[row];  dx = rstd * (dy*w - xhat * mean_row(dy*w*xhat));  dw = sum_rows dy*xhat
// dy, x, dx: bf16 [T, H] row-major; w: bf16 [H]; rstd: fp32 [T]; dw: fp32 [H].
// dy/x/w/dx 16-byte aligned, H a positive multiple of 8 and at most 51200.
// accumulate_dx != 0: dx += result (dx must hold valid values), else dx = result.
// accumulate_dw != 0: dw += result (dw must hold valid values), else dw = result.
// Nothing else has to start at zero: the scratch rows are written before read.
//
// Allocates nothing.  The weight-gradient partials use a fixed 2 MiB fp32
// device array (file scope, one per device); the grid is capped at
// floor(524288 / H) CTAs so they always fit.  The first call on each device
// resolves that array's address (cudaGetSymbolAddress) with the device
// current; make that first call before any stream capture.  The resolved
// address is cached per device for the life of the process: after a
// cudaDeviceReset the cache is stale and the entry point must not be called
// again in that process.
//
// Calls whose kernels can overlap on the same device race on the shared
// scratch: issue them on one stream, or order them with events.
//
// Returns 0 on success, nonzero on bad arguments (1), sizes beyond the limit
// (2), no usable device or address lookup failure (3), launch failure (4);
// libra_rmsnorm_bwd_noalloc_error() then describes the failure.
int libra_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                              int T, int H, int accumulate_dx, int accumulate_dw, cudaStream_t stream);

const char* libra_rmsnorm_bwd_noalloc_error(void);

#ifdef __cplusplus
}
#endif

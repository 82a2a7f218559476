// Host-side TMA descriptor encoding shared by the kernels of the decode step.
// cuTensorMapEncodeTiled is a driver-API entry point; it is looked up through
// the runtime once and needs the device's primary context bound to the calling
// thread.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace libra {
namespace tmap {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    LIBRA_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p,
                "libra_b200: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 tensor map with 128-byte swizzle: dims[0] is the contiguous one;
// strides (bytes) are for dims 1.. ; box per dim.
inline CUtensorMap make_bf16(const void* ptr, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                             const cuuint32_t* box) {
  static thread_local bool context_bound = false;
  if (!context_bound) {
    cudaFree(nullptr);
    context_bound = true;
  }
  CUtensorMap m;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(ptr), dims,
                           strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LIBRA_CHECK(r == CUDA_SUCCESS, "libra_b200: cuTensorMapEncodeTiled failed with code %d", (int)r);
  return m;
}

// Row-major [outer, inner] matrix with leading dimension ld (elements).
inline CUtensorMap make_2d(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer) {
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  return make_bf16(ptr, 2, dims, strides, box);
}

}  // namespace tmap

// Launch with programmatic dependent launch allowed (the kernel must execute
// griddepcontrol.wait before it reads anything its stream predecessor writes,
// and every CTA must execute it before exiting) or as a plain launch.
template <typename... KArgs, typename... Args>
inline void launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  LIBRA_CHECK(e == cudaSuccess, "libra_b200: kernel launch failed: %s", cudaGetErrorString(e));
}

}  // namespace libra

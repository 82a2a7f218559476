// Shared constants and helpers of the tcgen05 attention kernels.
#pragma once
#include <torch/extension.h>

#include "common.cuh"

namespace libra {
namespace attn {

constexpr int D = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int kThreads = 192;
constexpr int kChunk = 128 * 64 * 2;  // 128 rows x 64 bf16, one SW128 panel
constexpr int kTile = 2 * kChunk;     // 128 x 128 bf16
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  // 128 x 128 K-major tile = two 64-wide panels; step kk covers 16 K elements.
  return make_sw128_desc(base + (kk >> 2) * kChunk + (kk & 3) * 32, 16, 1024);
}

__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  // [128 K rows][2 x 64 N] MN-major tile: step kk advances 16 K rows; LBO = one N panel.
  return make_sw128_desc(base + kk * 2048, kChunk, 1024);
}

// ------------------------------------------------------------------ host helpers
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

// [T rows, H*D cols] bf16 view of a [T, H, D] tensor; box = 64 cols x 128 rows.
inline CUtensorMap head_map(const torch::Tensor& t) {
  static thread_local bool context_bound = false;
  if (!context_bound) {
    cudaFree(nullptr);  // bind the primary context on this thread before the driver call
    context_bound = true;
  }
  const int64_t T = t.size(0), W = t.size(1) * t.size(2);
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)W, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)(W * 2)};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LIBRA_CHECK(r == CUDA_SUCCESS, "flash_attn: cuTensorMapEncodeTiled failed with code %d", (int)r);
  return m;
}

inline void check_qkv(const torch::Tensor& t, const char* name) {
  LIBRA_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.size(2) == D && t.is_contiguous(),
              "flash_attn: %s must be a contiguous CUDA bf16 [T, H, 128] tensor", name);
  LIBRA_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "flash_attn: %s must be 16-byte aligned", name);
}

}  // namespace attn
}  // namespace libra

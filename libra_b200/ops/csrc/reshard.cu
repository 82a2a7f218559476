// Trainer -> rollout weight sync as one kernel: every destination rank pulls
// the pieces of its tensor-parallel slice straight out of the trainer ranks'
// parameter buffers (local, or mapped from peer GPUs over NVLink with CUDA IPC)
// and writes them, cast to bf16, into its own flat weight buffer.
//
// The copy plan is built once on the host (libra_b200/infra/sync/reshard.py):
// a list of 2-D rectangles, each `rows` rows of `row_elems` elements with
// independent source and destination pitches, cut into items of at most a few
// hundred KB so the grid stays balanced.  Row-parallel weights (o-proj, down)
// are column ranges of the source and destination rows; column-parallel
// weights (QKV, gate/up, embedding) are row ranges; replicated weights are
// single rows.  Nothing is gathered first: each byte crosses NVLink once, from
// the trainer rank that owns it to the rollout rank that needs it.
//
// Replaces the reference's full-tensor NCCL broadcast from trainer rank 0
// (infra/sync/nccl_weight_sync.py:126-197).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace libra {
namespace reshard {

// item layout (5 x int64): src address, dst address, rows << 32 | row_elems,
// src_pitch << 32 | dst_pitch (elements), flags (bit 0: fp32 source)
struct Item {
  uint64_t src, dst, shape, pitch, flags;
};

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ uint4 f32x8_to_bf16x8(const float4 a, const float4 b) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
  h[0] = __floats2bfloat162_rn(a.x, a.y);
  h[1] = __floats2bfloat162_rn(a.z, a.w);
  h[2] = __floats2bfloat162_rn(b.x, b.y);
  h[3] = __floats2bfloat162_rn(b.z, b.w);
  return r;
}

__global__ void __launch_bounds__(kThreads) reshard_kernel(const Item* __restrict__ items, int n_items) {
  for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
    const Item d = items[it];
    const uint32_t rows = (uint32_t)(d.shape >> 32), row_elems = (uint32_t)d.shape;
    const uint32_t sp = (uint32_t)(d.pitch >> 32), dp = (uint32_t)d.pitch;
    const bool f32 = d.flags & 1u;
    const uint32_t esz = f32 ? 4u : 2u;
    const bool vec = (row_elems % 8u == 0u) && (sp % 8u == 0u) && (dp % 8u == 0u) && (d.dst % 16u == 0u) &&
                     (d.src % 16u == 0u);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(d.dst);
    if (vec) {
      const uint32_t row_vecs = row_elems / 8u;
      const uint64_t total = (uint64_t)rows * row_vecs;
      for (uint64_t base = threadIdx.x; base < total; base += (uint64_t)kThreads * kUnroll) {
        uint4 v[kUnroll];
        uint64_t dsto[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const uint64_t i = base + (uint64_t)u * kThreads;
          dsto[u] = ~0ull;
          if (i < total) {
            const uint32_t r = (uint32_t)(i / row_vecs), c = (uint32_t)(i % row_vecs) * 8u;
            const uint64_t so = (uint64_t)r * sp + c;
            dsto[u] = (uint64_t)r * dp + c;
            if (f32) {
              const float4* s = reinterpret_cast<const float4*>(d.src + so * esz);
              v[u] = f32x8_to_bf16x8(s[0], s[1]);
            } else {
              v[u] = *reinterpret_cast<const uint4*>(d.src + so * esz);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (dsto[u] != ~0ull) *reinterpret_cast<uint4*>(dst + dsto[u]) = v[u];
      }
    } else {  // ragged shapes: element by element
      const uint64_t total = (uint64_t)rows * row_elems;
      for (uint64_t i = threadIdx.x; i < total; i += kThreads) {
        const uint32_t r = (uint32_t)(i / row_elems), c = (uint32_t)(i % row_elems);
        const uint64_t so = (uint64_t)r * sp + c;
        const float x = f32 ? reinterpret_cast<const float*>(d.src)[so]
                            : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(d.src)[so]);
        dst[(uint64_t)r * dp + c] = __float2bfloat16(x);
      }
    }
  }
}

// items: int64 [n, 5] on the destination device (see Item); grid <= 0 picks 4 CTAs per SM.
void weight_reshard(torch::Tensor items, int64_t grid) {
  LIBRA_CHECK(items.is_cuda() && items.scalar_type() == at::kLong && items.dim() == 2 && items.size(1) == 5 &&
                  items.is_contiguous(),
              "weight_reshard: items must be a contiguous int64 CUDA tensor [n, 5]");
  const int n = (int)items.size(0);
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(items.device());
  int g = (int)grid;
  if (g <= 0) {
    int dev, sms;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g = 4 * sms;
  }
  if (g > n) g = n;
  reshard_kernel<<<g, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const Item*>(items.data_ptr<int64_t>()), n);
  LIBRA_LAUNCH_CHECK();
}

}  // namespace reshard
}  // namespace libra

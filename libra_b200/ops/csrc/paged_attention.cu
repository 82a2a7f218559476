// Paged-KV decode attention (one new query token per sequence) with GQA head
// grouping and split-K ("flash decoding") over the KV range.  Replaces the
// decode attention inside vLLM that the reference's rollout servers use.
//
// Cache layout (per layer): k/v [num_blocks, block_size, kv_heads, D] bf16.
// CTA (b, h, s): sequence b, KV head h, split s of the sequence's tokens.
//   phase 1: each lane scores whole tokens (q of the G query heads of this KV
//            head are broadcast from shared memory); scores -> shared memory
//   phase 2: per-head max / sum over the split
//   phase 3: thread d accumulates sum_t p[g][t] * V[t][d] for the G heads
// Every K/V row of the split is read once and reused by all G query heads,
// so the kernel moves ~2 * len * kv_heads * D * 2 bytes per sequence: the
// memory roofline of decode.  Splits are merged by `merge_splits_kernel`.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace libra {

constexpr int kDecThreads = 128;  // = head_dim: one thread per output dim in phase 3

template <int D, int G>
__global__ void __launch_bounds__(kDecThreads) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q,      // [B, Hq, D]
    const __nv_bfloat16* __restrict__ kc,     // [blocks, bs, Hkv, D]
    const __nv_bfloat16* __restrict__ vc,
    const int* __restrict__ block_tables,     // [B, max_blocks]
    const int* __restrict__ seq_lens,         // [B]
    float* __restrict__ part_out,             // [B, Hq, S, D]
    float* __restrict__ part_ml,              // [B, Hq, S, 2]
    int Hq, int Hkv, int block_size, int max_blocks, int split_len, float scale) {
  static_assert(D == kDecThreads, "one thread per head dim");
  extern __shared__ float sm[];
  float* qs = sm;                         // [G][D]
  float* sc = qs + G * D;                 // [G][split_len]
  __shared__ float red[G][2];
  const int b = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int S = gridDim.z;
  const int len = seq_lens[b];
  const int t0 = s * split_len;
  const int t1 = min(len, t0 + split_len);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < G * D; i += kDecThreads) {
    const int g = i / D, d = i - g * D;
    qs[i] = __bfloat162float(q[((size_t)b * Hq + h * G + g) * D + d]) * scale;
  }
  __syncthreads();
  const int n = t1 - t0;
  // ---- phase 1: scores
  for (int t = tid; t < n; t += kDecThreads) {
    const int pos = t0 + t;
    const int blk = block_tables[(size_t)b * max_blocks + pos / block_size];
    const __nv_bfloat16* krow = kc + (((size_t)blk * block_size + pos % block_size) * Hkv + h) * D;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
#pragma unroll 4
    for (int v8 = 0; v8 < D / 8; ++v8) {
      uint4 u = reinterpret_cast<const uint4*>(krow)[v8];
      const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float kv = __bfloat162float(kb[e]);
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] += qs[g * D + v8 * 8 + e] * kv;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g * split_len + t] = acc[g];
  }
  __syncthreads();
  // ---- phase 2: per-head max and sum (warp w handles heads w, w+4, ...)
  for (int g = warp; g < G; g += kDecThreads / 32) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[g * split_len + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float p = (n > 0) ? __expf(sc[g * split_len + t] - m) : 0.f;
      sc[g * split_len + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      red[g][0] = m;
      red[g][1] = l;
    }
  }
  __syncthreads();
  // ---- phase 3: P V
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
  for (int t = 0; t < n; ++t) {
    const int pos = t0 + t;
    const int blk = block_tables[(size_t)b * max_blocks + pos / block_size];
    const float vv = __bfloat162float(vc[(((size_t)blk * block_size + pos % block_size) * Hkv + h) * D + tid]);
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] += sc[g * split_len + t] * vv;
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const size_t row = ((size_t)b * Hq + h * G + g) * S + s;
    part_out[row * D + tid] = o[g];
    if (tid == 0) {
      part_ml[row * 2] = red[g][0];
      part_ml[row * 2 + 1] = red[g][1];
    }
  }
}

// out[b, hq, d] = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s
template <int D>
__global__ void merge_splits_kernel(const float* __restrict__ part_out, const float* __restrict__ part_ml,
                                    __nv_bfloat16* __restrict__ out, int S) {
  const size_t row = blockIdx.x;  // b * Hq + hq
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, part_ml[(row * S + s) * 2]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < S; ++s) {
    const float m = part_ml[(row * S + s) * 2];
    if (m == -INFINITY) continue;
    const float w = __expf(m - M);
    num += w * part_out[(row * S + s) * D + d];
    den += w * part_ml[(row * S + s) * 2 + 1];
  }
  out[row * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

template <int G>
static void launch_decode(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                          const torch::Tensor& bt, const torch::Tensor& lens, torch::Tensor& po, torch::Tensor& pml,
                          int S, int split_len, float scale, cudaStream_t st) {
  const int B = (int)q.size(0), Hq = (int)q.size(1);
  const int Hkv = (int)kc.size(2), bs = (int)kc.size(1);
  constexpr int D = 128;
  const size_t smem = (size_t)(G * D + G * split_len) * sizeof(float);
  auto kern = paged_decode_kernel<D, G>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(B, Hkv, S);
  kern<<<grid, kDecThreads, smem, st>>>(
      (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)kc.data_ptr(), (const __nv_bfloat16*)vc.data_ptr(),
      bt.data_ptr<int>(), lens.data_ptr<int>(), po.data_ptr<float>(), pml.data_ptr<float>(), Hq, Hkv, bs,
      (int)bt.size(1), split_len, scale);
  LIBRA_LAUNCH_CHECK();
}

// q [B, Hq, 128] bf16; k/v cache [blocks, bs, Hkv, 128] bf16; block_tables [B, max_blocks] int32;
// seq_lens [B] int32 (tokens including the new one, whose KV must already be written).
torch::Tensor paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                     torch::Tensor block_tables, torch::Tensor seq_lens, int64_t max_len,
                                     double scale) {
  LIBRA_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous(),
              "paged_decode_attention: q must be contiguous bf16 [B, Hq, D]");
  LIBRA_CHECK(q.size(2) == 128, "paged_decode_attention: head_dim 128 supported");
  LIBRA_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4,
              "paged_decode_attention: contiguous caches [blocks, block_size, kv_heads, D]");
  LIBRA_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt,
              "paged_decode_attention: int32 block tables / lengths");
  const int B = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k_cache.size(2);
  LIBRA_CHECK(Hq % Hkv == 0, "paged_decode_attention: Hq must be a multiple of Hkv");
  const int G = Hq / Hkv;
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty_like(q);
  if (B == 0) return out;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // enough CTAs to fill the GPU twice, splits of at most 1024 tokens
  int S = 1;
  const int L = (int)std::max<int64_t>(max_len, 1);
  while ((int64_t)B * Hkv * S < 2 * sms && L / (S * 2) >= 128) S *= 2;
  int split_len = (L + S - 1) / S;
  while (split_len > 1024) {
    S *= 2;
    split_len = (L + S - 1) / S;
  }
  auto po = torch::empty({B, Hq, S, 128}, q.options().dtype(at::kFloat));
  auto pml = torch::empty({B, Hq, S, 2}, q.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (G) {
    case 1: launch_decode<1>(q, k_cache, v_cache, block_tables, seq_lens, po, pml, S, split_len, (float)scale, st); break;
    case 2: launch_decode<2>(q, k_cache, v_cache, block_tables, seq_lens, po, pml, S, split_len, (float)scale, st); break;
    case 4: launch_decode<4>(q, k_cache, v_cache, block_tables, seq_lens, po, pml, S, split_len, (float)scale, st); break;
    case 5: launch_decode<5>(q, k_cache, v_cache, block_tables, seq_lens, po, pml, S, split_len, (float)scale, st); break;
    case 8: launch_decode<8>(q, k_cache, v_cache, block_tables, seq_lens, po, pml, S, split_len, (float)scale, st); break;
    default: LIBRA_CHECK(false, "paged_decode_attention: unsupported GQA group size %d", G);
  }
  merge_splits_kernel<128><<<B * Hq, 128, 0, st>>>(po.data_ptr<float>(), pml.data_ptr<float>(),
                                                  (__nv_bfloat16*)out.data_ptr(), S);
  LIBRA_LAUNCH_CHECK();
  return out;
}

}  // namespace libra

// Rollout-engine kernels that run inside the captured decode step:
//
//  * paged_decode_v2 — decode attention over the paged KV cache with a fixed
//    split layout (the grid depends only on the batch capacity and the split
//    count, never on the current sequence lengths), so one CUDA graph serves
//    every step of a generation.  Each half-warp owns one token at a time and
//    each of its 16 lanes reads a 16-byte slice of the 256-byte K (then V) row,
//    so every cache row is one coalesced 256-byte read that all G query heads
//    of the KV head reuse.  Scores live in shared memory in the log2 domain;
//    splits are merged by a second small kernel.
//  * sample_tokens — temperature sampling by the Gumbel-max trick: the token
//    is argmax_v(x_v / T + g_v) with g_v = -log(-log(u_v)), which draws from
//    softmax(x / T) exactly, so no sort, cumulative sum or second pass over
//    the vocabulary is needed.  u_v comes from Philox4x32-10 (Salmon, Moraes,
//    Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011)
//    keyed by the request's seed and counted by (vocabulary index, position),
//    so a seeded request draws the same tokens whatever batch it runs in.  The
//    same pass computes max and sum-exp, which give the sampled token's
//    logprob under the temperature-scaled distribution (the value the
//    reference's rollout servers return with logprobs=1).
//
// Replaces the decode attention and sampler inside the vLLM servers that the
// reference's rollout clients call (engine/rollout_engine.py:168-288).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.cuh"

namespace libra {
namespace rollout {

constexpr int kD = 128;          // head dim
constexpr int kThreads = 128;    // 4 warps = 8 half-warps
constexpr int kHalves = kThreads / 16;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads) paged_decode_v2_kernel(
    const __nv_bfloat16* __restrict__ q,   // [B, Hq, D]
    const __nv_bfloat16* __restrict__ kc,  // [blocks, bs, Hkv, D]
    const __nv_bfloat16* __restrict__ vc,
    const int* __restrict__ block_tables,  // [B, max_blocks]
    const int* __restrict__ seq_lens,      // [B]
    float* __restrict__ part_out,          // [B, Hq, S, D]
    float* __restrict__ part_ml,           // [B, Hq, S, 2]  (max in log2 units, sum)
    int Hq, int Hkv, int block_size, int max_blocks, int split_len, float scale_log2) {
  extern __shared__ float sc[];            // [G][split_len]
  __shared__ float red_o[4][G][kD];
  __shared__ float red_m[G], red_l[G];
  const int b = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int S = gridDim.z;
  const int len = seq_lens[b];
  const int t0 = s * split_len;
  const int n = min(len, t0 + split_len) - t0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hl = tid & 15;
  if (n <= 0) {  // split beyond this sequence: contributes nothing to the merge
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const size_t row = ((size_t)b * Hq + h * G + g) * S + s;
      part_out[row * kD + tid] = 0.f;
      if (tid == 0) {
        part_ml[row * 2] = -INFINITY;
        part_ml[row * 2 + 1] = 0.f;
      }
    }
    return;
  }
  // this lane's 8-dim slice of the G query heads, pre-scaled into log2 units
  float qr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4 u = *reinterpret_cast<const uint4*>(q + ((size_t)b * Hq + h * G + g) * kD + hl * 8);
    bf16x8_to_f32(u, qr[g]);
#pragma unroll
    for (int e = 0; e < 8; ++e) qr[g][e] *= scale_log2;
  }
  const int* tbl = block_tables + (size_t)b * max_blocks;
  const size_t row_stride = (size_t)Hkv * kD;
  // ---- phase 1: scores, one token per half-warp per iteration, two tokens in flight
  // (the loop bound is uniform per warp: the shuffles below need all 32 lanes)
  for (int base = 2 * warp; base < n; base += 2 * kHalves) {
    const int tt = base + (lane >> 4), tt2 = tt + kHalves;
    const bool has1 = tt < n, has2 = tt2 < n;
    const int p1 = t0 + (has1 ? tt : 0), p2 = t0 + (has2 ? tt2 : 0);
    const size_t r1 = (size_t)tbl[p1 / block_size] * block_size + p1 % block_size;
    const size_t r2 = (size_t)tbl[p2 / block_size] * block_size + p2 % block_size;
    const uint4 k1 = *reinterpret_cast<const uint4*>(kc + r1 * row_stride + (size_t)h * kD + hl * 8);
    const uint4 k2 = *reinterpret_cast<const uint4*>(kc + r2 * row_stride + (size_t)h * kD + hl * 8);
    float f1[8], f2[8];
    bf16x8_to_f32(k1, f1);
    bf16x8_to_f32(k2, f2);
    float a1[G], a2[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      a1[g] = 0.f;
      a2[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a1[g] = fmaf(qr[g][e], f1[e], a1[g]);
        a2[g] = fmaf(qr[g][e], f2[e], a2[g]);
      }
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        a1[g] += __shfl_xor_sync(0xffffffffu, a1[g], off);
        a2[g] += __shfl_xor_sync(0xffffffffu, a2[g], off);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (hl == g) {
        if (has1) sc[g * split_len + tt] = a1[g];
        if (has2) sc[g * split_len + tt2] = a2[g];
      }
    }
  }
  __syncthreads();
  // ---- phase 2: per-head max and sum of 2^(s - m); scores become probabilities
  for (int g = warp; g < G; g += kThreads / 32) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, sc[g * split_len + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float p = exp2f(sc[g * split_len + t] - m);
      sc[g * split_len + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      red_m[g] = m;
      red_l[g] = l;
    }
  }
  __syncthreads();
  // ---- phase 3: P V with the same half-warp-per-token layout
  float o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) o[g][e] = 0.f;
  for (int base = 2 * warp; base < n; base += 2 * kHalves) {
    const int tt = base + (lane >> 4), tt2 = tt + kHalves;
    const bool has1 = tt < n, has2 = tt2 < n;
    const int p1 = t0 + (has1 ? tt : 0), p2 = t0 + (has2 ? tt2 : 0);
    const size_t r1 = (size_t)tbl[p1 / block_size] * block_size + p1 % block_size;
    const size_t r2 = (size_t)tbl[p2 / block_size] * block_size + p2 % block_size;
    const uint4 v1 = *reinterpret_cast<const uint4*>(vc + r1 * row_stride + (size_t)h * kD + hl * 8);
    const uint4 v2 = *reinterpret_cast<const uint4*>(vc + r2 * row_stride + (size_t)h * kD + hl * 8);
    float f1[8], f2[8];
    bf16x8_to_f32(v1, f1);
    bf16x8_to_f32(v2, f2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float w1 = has1 ? sc[g * split_len + tt] : 0.f;
      const float w2 = has2 ? sc[g * split_len + tt2] : 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[g][e] = fmaf(w2, f2[e], fmaf(w1, f1[e], o[g][e]));
    }
  }
  // combine the two half-warps, then the four warps through shared memory
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) o[g][e] += __shfl_xor_sync(0xffffffffu, o[g][e], 16);
  if (lane < 16) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) red_o[warp][g][hl * 8 + e] = o[g][e];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float acc = red_o[0][g][tid] + red_o[1][g][tid] + red_o[2][g][tid] + red_o[3][g][tid];
    const size_t row = ((size_t)b * Hq + h * G + g) * S + s;
    part_out[row * kD + tid] = acc;
    if (tid == 0) {
      part_ml[row * 2] = red_m[g];
      part_ml[row * 2 + 1] = red_l[g];
    }
  }
}

// out[b, hq, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s
__global__ void __launch_bounds__(kD) merge_v2_kernel(const float* __restrict__ part_out,
                                                      const float* __restrict__ part_ml,
                                                      __nv_bfloat16* __restrict__ out, int S) {
  const size_t row = blockIdx.x;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, part_ml[(row * S + s) * 2]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < S; ++s) {
    const float m = part_ml[(row * S + s) * 2];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M);
    num = fmaf(w, part_out[(row * S + s) * kD + d], num);
    den = fmaf(w, part_ml[(row * S + s) * 2 + 1], den);
  }
  out[row * kD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

template <int G>
static void launch_v2(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                      const torch::Tensor& bt, const torch::Tensor& lens, torch::Tensor& po, torch::Tensor& pml,
                      int B, int S, int split_len, float scale_log2, cudaStream_t st) {
  const int Hq = (int)q.size(1), Hkv = (int)kc.size(2), bs = (int)kc.size(1);
  const size_t smem = (size_t)G * split_len * sizeof(float);
  auto kern = paged_decode_v2_kernel<G>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(B, Hkv, S);
  kern<<<grid, kThreads, smem, st>>>((const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)kc.data_ptr(),
                                     (const __nv_bfloat16*)vc.data_ptr(), bt.data_ptr<int>(), lens.data_ptr<int>(),
                                     po.data_ptr<float>(), pml.data_ptr<float>(), Hq, Hkv, bs, (int)bt.size(1),
                                     split_len, scale_log2);
  LIBRA_LAUNCH_CHECK();
}

// q [B, Hq, 128] bf16; caches [blocks, bs, Hkv, 128] bf16; block_tables [>=B, max_blocks] int32;
// seq_lens [>=B] int32; out [B, Hq, 128] bf16; part_out [B, Hq, S, 128] fp32 and part_ml [B, Hq, S, 2] fp32
// are caller-owned workspace.  S * split_len must cover every sequence length; nothing is allocated and
// no argument depends on the current lengths, so the call can be captured once and replayed.
void paged_decode_v2(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                     torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_out, torch::Tensor part_ml,
                     int64_t split_len, double scale) {
  LIBRA_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous() &&
                  q.size(2) == kD,
              "paged_decode_v2: q must be contiguous bf16 [B, Hq, 128]");
  LIBRA_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4 && k_cache.size(3) == kD &&
                  k_cache.sizes() == v_cache.sizes() && k_cache.scalar_type() == at::kBFloat16,
              "paged_decode_v2: contiguous bf16 caches [blocks, block_size, kv_heads, 128]");
  LIBRA_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_tables.is_contiguous() && block_tables.dim() == 2,
              "paged_decode_v2: int32 block tables [B, max_blocks] and lengths");
  const int B = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k_cache.size(2);
  LIBRA_CHECK(Hq % Hkv == 0, "paged_decode_v2: Hq must be a multiple of Hkv");
  LIBRA_CHECK(block_tables.size(0) >= B && seq_lens.numel() >= B, "paged_decode_v2: tables shorter than the batch");
  LIBRA_CHECK(out.is_contiguous() && out.sizes() == q.sizes() && out.scalar_type() == at::kBFloat16,
              "paged_decode_v2: out must be bf16 like q");
  LIBRA_CHECK(part_out.is_contiguous() && part_out.dim() == 4 && part_out.size(0) >= B && part_out.size(1) == Hq &&
                  part_out.size(3) == kD && part_out.scalar_type() == at::kFloat,
              "paged_decode_v2: part_out must be fp32 [>=B, Hq, S, 128]");
  const int S = (int)part_out.size(2);
  LIBRA_CHECK(part_ml.is_contiguous() && part_ml.numel() >= (int64_t)B * Hq * S * 2 &&
                  part_ml.scalar_type() == at::kFloat,
              "paged_decode_v2: part_ml must be fp32 [>=B, Hq, S, 2]");
  LIBRA_CHECK(split_len >= 1 && split_len <= 2048, "paged_decode_v2: split_len in [1, 2048]");
  const int G = Hq / Hkv;
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);  // log2(e)
  switch (G) {
    case 1: launch_v2<1>(q, k_cache, v_cache, block_tables, seq_lens, part_out, part_ml, B, S, (int)split_len, sl2, st); break;
    case 2: launch_v2<2>(q, k_cache, v_cache, block_tables, seq_lens, part_out, part_ml, B, S, (int)split_len, sl2, st); break;
    case 4: launch_v2<4>(q, k_cache, v_cache, block_tables, seq_lens, part_out, part_ml, B, S, (int)split_len, sl2, st); break;
    case 5: launch_v2<5>(q, k_cache, v_cache, block_tables, seq_lens, part_out, part_ml, B, S, (int)split_len, sl2, st); break;
    case 8: launch_v2<8>(q, k_cache, v_cache, block_tables, seq_lens, part_out, part_ml, B, S, (int)split_len, sl2, st); break;
    default: LIBRA_CHECK(false, "paged_decode_v2: unsupported GQA group size %d", G);
  }
  merge_v2_kernel<<<B * Hq, kD, 0, st>>>(part_out.data_ptr<float>(), part_ml.data_ptr<float>(),
                                         (__nv_bfloat16*)out.data_ptr(), S);
  LIBRA_LAUNCH_CHECK();
}

// ---------------------------------------------------------------- sampling
// Philox4x32 with 10 rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// uniform in (0, 1): 24 random bits, centred in their cell so 0 and 1 never occur
__device__ __forceinline__ float u01(uint32_t x) { return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

__device__ __forceinline__ float gumbel(uint32_t x) { return -logf(-logf(u01(x))); }

struct SampleAcc {
  float m, s;    // running max of x/T and sum of exp(x/T - m)
  float best;    // best perturbed score
  int idx;       // its index
  float val;     // x/T at idx
};

__device__ __forceinline__ void acc_merge(SampleAcc& a, const SampleAcc& b) {
  if (b.m > a.m) {
    a.s = a.s * expf(a.m - b.m) + b.s;
    a.m = b.m;
  } else if (b.m > -INFINITY) {
    a.s += b.s * expf(b.m - a.m);
  }
  if (b.best > a.best || (b.best == a.best && b.idx < a.idx)) {
    a.best = b.best;
    a.idx = b.idx;
    a.val = b.val;
  }
}

constexpr int kSampleThreads = 512;

// One CTA per row.  temperature <= 0 means greedy (argmax, logprob under T = 1).
// Logits are bf16, or fp32 (the stream-K accumulator of the fused decode
// step, which the kernel zeroes behind itself for the next step).
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
}
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  const float4 f = __ldcs(reinterpret_cast<const float4*>(p));
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load1(const float* p) { return *p; }

template <typename T, bool kZero>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(
    T* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temperature,
    const int64_t* __restrict__ seeds, const int64_t* __restrict__ positions, int64_t* __restrict__ out_tok,
    float* __restrict__ out_lp, int64_t* __restrict__ next_tok) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  T* x = logits + (size_t)row * ld;
  const float Tm = temperature[row];
  const bool greedy = !(Tm > 0.f);
  const float inv = greedy ? 1.f : 1.f / Tm;
  const uint64_t seed = (uint64_t)seeds[row];
  const uint64_t pos = (uint64_t)positions[row];
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  SampleAcc a{-INFINITY, 0.f, -INFINITY, 0x7fffffff, 0.f};
  const int V4 = V / 4;
  for (int i = threadIdx.x; i < V4; i += kSampleThreads) {
    float v[4];
    load4<T>(x + 4 * (size_t)i, v);
    if constexpr (kZero) __stcs(reinterpret_cast<float4*>(x + 4 * (size_t)i), make_float4(0.f, 0.f, 0.f, 0.f));
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] *= inv;
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if (!greedy) r = philox4x32_10(make_uint4((uint32_t)i, (uint32_t)pos, (uint32_t)(pos >> 32), 0x5A17u), key);
    const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
    float vm = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    if (vm > a.m) {
      a.s *= expf(a.m - vm);
      a.m = vm;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a.s += expf(v[e] - a.m);
      const float sc = greedy ? v[e] : v[e] + gumbel(rr[e]);
      if (sc > a.best) {
        a.best = sc;
        a.idx = 4 * i + e;
        a.val = v[e];
      }
    }
  }
  for (int j = 4 * V4 + threadIdx.x; j < V; j += kSampleThreads) {  // vocabulary tail (V % 4)
    const float v = load1(x + j) * inv;
    if constexpr (kZero) x[j] = 0.f;
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if (!greedy) r = philox4x32_10(make_uint4((uint32_t)(j / 4), (uint32_t)pos, (uint32_t)(pos >> 32), 0x5A17u), key);
    const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
    if (v > a.m) {
      a.s *= expf(a.m - v);
      a.m = v;
    }
    a.s += expf(v - a.m);
    const float sc = greedy ? v : v + gumbel(rr[j & 3]);
    if (sc > a.best) {
      a.best = sc;
      a.idx = j;
      a.val = v;
    }
  }
  // warp then block reduction
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    SampleAcc o;
    o.m = __shfl_xor_sync(0xffffffffu, a.m, off);
    o.s = __shfl_xor_sync(0xffffffffu, a.s, off);
    o.best = __shfl_xor_sync(0xffffffffu, a.best, off);
    o.idx = __shfl_xor_sync(0xffffffffu, a.idx, off);
    o.val = __shfl_xor_sync(0xffffffffu, a.val, off);
    acc_merge(a, o);
  }
  __shared__ SampleAcc wacc[kSampleThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) wacc[warp] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    SampleAcc t = wacc[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) acc_merge(t, wacc[w]);
    const bool ok = t.idx >= 0 && t.idx < V;
    const int tok = ok ? t.idx : 0;
    out_tok[row] = tok;
    out_lp[row] = ok ? t.val - t.m - logf(t.s) : -INFINITY;
    if (next_tok) next_tok[row] = tok;
  }
}

// logits [B, V] bf16 (row stride ld, 8-byte aligned rows); temperature [B] fp32; seeds/positions [B] int64;
// out_tok [B] int64, out_lp [B] fp32; next_tok optional [B] int64 (a second copy of the tokens, e.g. the
// next decode step's input buffer).
// fp32 logits (the fused decode step's accumulator) are zeroed behind the read, 16-byte aligned rows.
void sample_tokens(torch::Tensor logits, torch::Tensor temperature, torch::Tensor seeds, torch::Tensor positions,
                   torch::Tensor out_tok, torch::Tensor out_lp, c10::optional<torch::Tensor> next_tok, bool pdl) {
  const bool f32 = logits.scalar_type() == at::kFloat;
  LIBRA_CHECK(logits.is_cuda() && (f32 || logits.scalar_type() == at::kBFloat16) && logits.dim() == 2 &&
                  logits.stride(1) == 1 && logits.stride(0) % 4 == 0 &&
                  (reinterpret_cast<uintptr_t>(logits.data_ptr()) & (f32 ? 15 : 7)) == 0,
              "sample_tokens: logits must be bf16 or fp32 [B, V] with unit inner stride and aligned rows");
  const int B = (int)logits.size(0), V = (int)logits.size(1);
  LIBRA_CHECK(temperature.scalar_type() == at::kFloat && temperature.numel() >= B, "sample_tokens: temperature fp32 [B]");
  LIBRA_CHECK(seeds.scalar_type() == at::kLong && seeds.numel() >= B && positions.scalar_type() == at::kLong &&
                  positions.numel() >= B,
              "sample_tokens: seeds/positions int64 [B]");
  LIBRA_CHECK(out_tok.scalar_type() == at::kLong && out_tok.numel() >= B && out_lp.scalar_type() == at::kFloat &&
                  out_lp.numel() >= B,
              "sample_tokens: outputs int64 / fp32 [B]");
  int64_t* nt = nullptr;
  if (next_tok.has_value()) {
    LIBRA_CHECK(next_tok->scalar_type() == at::kLong && next_tok->numel() >= B, "sample_tokens: next_tok int64 [B]");
    nt = next_tok->data_ptr<int64_t>();
  }
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (f32)
    launch_kernel(sample_kernel<float, true>, dim3(B), dim3(kSampleThreads), 0, st, pdl, logits.data_ptr<float>(),
                  (int64_t)logits.stride(0), V, (const float*)temperature.data_ptr<float>(),
                  (const int64_t*)seeds.data_ptr<int64_t>(), (const int64_t*)positions.data_ptr<int64_t>(),
                  out_tok.data_ptr<int64_t>(), out_lp.data_ptr<float>(), nt);
  else
    launch_kernel(sample_kernel<__nv_bfloat16, false>, dim3(B), dim3(kSampleThreads), 0, st, pdl,
                  (__nv_bfloat16*)logits.data_ptr(), (int64_t)logits.stride(0), V,
                  (const float*)temperature.data_ptr<float>(), (const int64_t*)seeds.data_ptr<int64_t>(),
                  (const int64_t*)positions.data_ptr<int64_t>(), out_tok.data_ptr<int64_t>(),
                  out_lp.data_ptr<float>(), nt);
  LIBRA_LAUNCH_CHECK();
}


// ---------------------------------------------------------------------------
// sample_tokens_filtered — temperature sampling restricted to the top-k tokens
// and to the top-p nucleus, with the same Philox/Gumbel stream as
// sample_tokens (unfiltered rows draw the same token from both kernels).
//
// Both filters keep the tokens whose scaled logit is at least a threshold, so
// each is found by a radix select on the order-preserving 32-bit key of the
// scaled logit, 8 bits per pass from the most significant end (4 passes):
//   * top-k: the key of the k-th largest value (bucket counts);
//   * top-p: the smallest key t whose "probability mass strictly above t" is
//     at most p, the rule of the sorted cumulative-sum formulation (a token is
//     dropped when the mass before it exceeds p); masses are summed in 2^-32
//     fixed point so the threshold does not depend on the order of the
//     shared-memory atomics.
// Tokens tied with the threshold value are all kept.  The combined threshold is
// the larger of the two; Gumbel-max then runs over the kept tokens, and the
// logprob is the token's under the unfiltered temperature-scaled distribution.
// One CTA per row.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kFiltThreads = 512;

struct FiltShared {
  unsigned int cnt[256];
  unsigned long long mass[256];
  uint32_t prefix;
  unsigned long long above;
  float m, s;
};

__device__ __forceinline__ void radix_pass_clear(FiltShared& sh) {
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    sh.cnt[b] = 0u;
    sh.mass[b] = 0ull;
  }
}

// Key of the k-th largest scaled value of the row.
template <typename T>
__device__ uint32_t select_topk_key(const T* x, int V, float inv, int k, FiltShared& sh) {
  uint32_t prefix = 0u, mask = 0u;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    radix_pass_clear(sh);
    __syncthreads();
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const uint32_t key = order_key(load1(x + j) * inv);
      if ((key & mask) == prefix) atomicAdd(&sh.cnt[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int cum = 0, b = 255;
      for (; b > 0; --b) {
        if (cum + (int)sh.cnt[b] >= remaining) break;
        cum += (int)sh.cnt[b];
      }
      remaining -= cum;
      sh.prefix = prefix | ((uint32_t)b << shift);
    }
    __syncthreads();
    prefix = sh.prefix;
    mask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

// Smallest key t with (mass of keys > t) <= p.
template <typename T>
__device__ uint32_t select_topp_key(const T* x, int V, float inv, float m, float s, float p, FiltShared& sh) {
  const double scale = 4294967296.0;  // 2^32 fixed point
  const unsigned long long pq = (unsigned long long)(fmaxf(p, 0.f) * scale);
  const float rs = 1.f / s;
  uint32_t prefix = 0u, mask = 0u;
  if (threadIdx.x == 0) sh.above = 0ull;
  for (int shift = 24; shift >= 0; shift -= 8) {
    radix_pass_clear(sh);
    __syncthreads();
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const float v = load1(x + j) * inv;
      const uint32_t key = order_key(v);
      if ((key & mask) == prefix) {
        const uint32_t b = (key >> shift) & 255u;
        atomicAdd(&sh.cnt[b], 1u);
        const unsigned long long q = (unsigned long long)((double)(expf(v - m) * rs) * scale);
        if (q) atomicAdd(&sh.mass[b], q);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long run = sh.above, run_chosen = sh.above;
      int chosen = -1;
      for (int b = 255; b >= 0; --b) {
        if (sh.cnt[b] == 0u) continue;
        if (run > pq) break;
        chosen = b;
        run_chosen = run;
        run += sh.mass[b];
      }
      if (chosen < 0) chosen = 0;  // unreachable: the first non-empty bucket always qualifies
      sh.above = run_chosen;
      sh.prefix = prefix | ((uint32_t)chosen << shift);
    }
    __syncthreads();
    prefix = sh.prefix;
    mask |= 255u << shift;
    __syncthreads();
  }
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(kFiltThreads) sample_filtered_kernel(
    const T* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temperature,
    const float* __restrict__ top_p, const int64_t* __restrict__ top_k, const int64_t* __restrict__ seeds,
    const int64_t* __restrict__ positions, int64_t* __restrict__ out_tok, float* __restrict__ out_lp) {
  __shared__ FiltShared sh;
  __shared__ SampleAcc wacc[kFiltThreads / 32];
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  const float Tm = temperature[row];
  const bool greedy = !(Tm > 0.f);
  const float inv = greedy ? 1.f : 1.f / Tm;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // pass 1: max and sum of exp of the scaled logits
  float m = -INFINITY, s = 0.f;
  for (int j = threadIdx.x; j < V; j += kFiltThreads) {
    const float v = load1(x + j) * inv;
    if (v > m) {
      s *= expf(m - v);
      m = v;
    }
    s += expf(v - m);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, off), os = __shfl_xor_sync(0xffffffffu, s, off);
    const float nm = fmaxf(m, om);
    s = (m > -INFINITY ? s * expf(m - nm) : 0.f) + (om > -INFINITY ? os * expf(om - nm) : 0.f);
    m = nm;
  }
  if (lane == 0) wacc[warp] = SampleAcc{m, s, 0.f, 0, 0.f};
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, S = 0.f;
    for (int w = 0; w < kFiltThreads / 32; ++w) {
      const float wm = wacc[w].m, ws = wacc[w].s;
      const float nm = fmaxf(M, wm);
      S = (M > -INFINITY ? S * expf(M - nm) : 0.f) + (wm > -INFINITY ? ws * expf(wm - nm) : 0.f);
      M = nm;
    }
    sh.m = M;
    sh.s = S;
  }
  __syncthreads();
  m = sh.m;
  s = sh.s;
  // thresholds
  uint32_t thr = 0u;
  if (!greedy) {
    const int64_t k = top_k[row];
    if (k > 0 && k < V) thr = select_topk_key<T>(x, V, inv, (int)k, sh);
    const float p = top_p[row];
    if (p < 1.f) {
      const uint32_t tp = select_topp_key<T>(x, V, inv, m, s, p, sh);
      thr = tp > thr ? tp : thr;
    }
  }
  // Gumbel-max over the kept tokens (the Philox counter layout of sample_kernel)
  const uint64_t seed = (uint64_t)seeds[row];
  const uint64_t pos = (uint64_t)positions[row];
  const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
  SampleAcc a{-INFINITY, 0.f, -INFINITY, 0x7fffffff, 0.f};
  const int groups = (V + 3) / 4;
  for (int i = threadIdx.x; i < groups; i += kFiltThreads) {
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if (!greedy) r = philox4x32_10(make_uint4((uint32_t)i, (uint32_t)pos, (uint32_t)(pos >> 32), 0x5A17u), key);
    const uint32_t rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = 4 * i + e;
      if (j >= V) break;
      const float v = load1(x + j) * inv;
      if (order_key(v) < thr) continue;
      const float sc = greedy ? v : v + gumbel(rr[e]);
      if (sc > a.best || (sc == a.best && j < a.idx)) {
        a.best = sc;
        a.idx = j;
        a.val = v;
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, a.best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, a.idx, off);
    const float ov = __shfl_xor_sync(0xffffffffu, a.val, off);
    if (ob > a.best || (ob == a.best && oi < a.idx)) {
      a.best = ob;
      a.idx = oi;
      a.val = ov;
    }
  }
  __syncthreads();  // wacc reuse
  if (lane == 0) wacc[warp] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    SampleAcc t = wacc[0];
    for (int w = 1; w < kFiltThreads / 32; ++w)
      if (wacc[w].best > t.best || (wacc[w].best == t.best && wacc[w].idx < t.idx)) t = wacc[w];
    const bool ok = t.idx >= 0 && t.idx < V;
    out_tok[row] = ok ? t.idx : 0;
    out_lp[row] = ok ? t.val - m - logf(s) : -INFINITY;
  }
}

// logits [B, V] bf16 or fp32 (unit inner stride); temperature / top_p fp32 [B]; top_k / seeds / positions
// int64 [B] (top_k <= 0 or >= V: no top-k; top_p >= 1: no nucleus); outputs int64 / fp32 [B].
void sample_tokens_filtered(torch::Tensor logits, torch::Tensor temperature, torch::Tensor top_p, torch::Tensor top_k,
                            torch::Tensor seeds, torch::Tensor positions, torch::Tensor out_tok, torch::Tensor out_lp) {
  const bool f32 = logits.scalar_type() == at::kFloat;
  LIBRA_CHECK(logits.is_cuda() && (f32 || logits.scalar_type() == at::kBFloat16) && logits.dim() == 2 &&
                  logits.stride(1) == 1,
              "sample_tokens_filtered: logits must be bf16 or fp32 [B, V] with unit inner stride");
  const int B = (int)logits.size(0), V = (int)logits.size(1);
  auto dev_vec = [&](const torch::Tensor& t, at::ScalarType ty) {
    return t.is_cuda() && t.device() == logits.device() && t.scalar_type() == ty && t.is_contiguous() &&
           t.numel() >= B;
  };
  LIBRA_CHECK(dev_vec(temperature, at::kFloat) && dev_vec(top_p, at::kFloat),
              "sample_tokens_filtered: temperature / top_p fp32 [B] on the logits' device");
  LIBRA_CHECK(dev_vec(top_k, at::kLong) && dev_vec(seeds, at::kLong) && dev_vec(positions, at::kLong),
              "sample_tokens_filtered: top_k / seeds / positions int64 [B] on the logits' device");
  LIBRA_CHECK(dev_vec(out_tok, at::kLong) && dev_vec(out_lp, at::kFloat),
              "sample_tokens_filtered: outputs int64 / fp32 [B] on the logits' device");
  if (B == 0 || V == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (f32)
    sample_filtered_kernel<float><<<B, kFiltThreads, 0, st>>>(
        logits.data_ptr<float>(), (int64_t)logits.stride(0), V, temperature.data_ptr<float>(),
        top_p.data_ptr<float>(), top_k.data_ptr<int64_t>(), seeds.data_ptr<int64_t>(),
        positions.data_ptr<int64_t>(), out_tok.data_ptr<int64_t>(), out_lp.data_ptr<float>());
  else
    sample_filtered_kernel<__nv_bfloat16><<<B, kFiltThreads, 0, st>>>(
        (const __nv_bfloat16*)logits.data_ptr(), (int64_t)logits.stride(0), V, temperature.data_ptr<float>(),
        top_p.data_ptr<float>(), top_k.data_ptr<int64_t>(), seeds.data_ptr<int64_t>(),
        positions.data_ptr<int64_t>(), out_tok.data_ptr<int64_t>(), out_lp.data_ptr<float>());
  LIBRA_LAUNCH_CHECK();
}

}  // namespace rollout
}  // namespace libra

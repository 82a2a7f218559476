// SwiGLU, fused vocab log-softmax/logprob/entropy, and the flat-buffer AdamW
// update with on-device gradient clipping.
//
// * SwiGLU replaces the activation inside Megatron-Core's fc1/fc2 MLP
//   (engine/megatron_core_train_engine.py:279-317 builds the provider).
// * `logprob_fwd/bwd` is the single-GPU core of the vocab-parallel token
//   logprob (engine/megatron_core_train_engine.py:905-948): it reads bf16 logits
//   once, keeps only (max, log-sum-exp) per row, and writes the logits gradient
//   in place, so no fp32 [tokens, vocab] temporary is ever allocated.
// * `adamw_step` is the optimizer of engine/megatron_core_train_engine.py:228-261
//   (Adam betas (0.9, 0.95), eps 1e-8, wd 0.01, clip 1.0) over one flat fp32
//   master buffer; the clip coefficient is computed on the device from the
//   squared-norm accumulator so the step needs no host synchronisation.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace libra {

__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ------------------------------------------------------------------ SwiGLU
// gu: [T, 2F] with gate in [:, :F] and up in [:, F:]; h: [T, F]
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int64_t T,
                                  int F) {
  const int vper = F >> 3;
  const int64_t n = T * vper;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vper;
    const int v = (int)(i - t * vper);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + v * 8);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + v * 8);
    const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uv);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = __bfloat162float(g[e]);
      o[e] = x * sigmoidf_(x) * __bfloat162float(u[e]);
    }
    uint4 pk;
    pk.x = pack_bf16x2(o[0], o[1]);
    pk.y = pack_bf16x2(o[2], o[3]);
    pk.z = pack_bf16x2(o[4], o[5]);
    pk.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(h + t * F + v * 8) = pk;
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int64_t T, int F) {
  const int vper = F >> 3;
  const int64_t n = T * vper;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vper;
    const int v = (int)(i - t * vper);
    uint4 gv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + v * 8);
    uint4 uv = *reinterpret_cast<const uint4*>(gu + t * 2 * F + F + v * 8);
    uint4 dv = *reinterpret_cast<const uint4*>(dh + t * F + v * 8);
    const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uv);
    const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(&dv);
    float dg[8], du[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = __bfloat162float(g[e]);
      const float s = sigmoidf_(x);
      const float up = __bfloat162float(u[e]);
      const float gd = __bfloat162float(d[e]);
      du[e] = gd * x * s;
      dg[e] = gd * up * s * (1.f + x * (1.f - s));
    }
    uint4 pg, pu;
    pg.x = pack_bf16x2(dg[0], dg[1]); pg.y = pack_bf16x2(dg[2], dg[3]);
    pg.z = pack_bf16x2(dg[4], dg[5]); pg.w = pack_bf16x2(dg[6], dg[7]);
    pu.x = pack_bf16x2(du[0], du[1]); pu.y = pack_bf16x2(du[2], du[3]);
    pu.z = pack_bf16x2(du[4], du[5]); pu.w = pack_bf16x2(du[6], du[7]);
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + v * 8) = pg;
    *reinterpret_cast<uint4*>(dgu + t * 2 * F + F + v * 8) = pu;
  }
}

// ------------------------------------------------------------------ logprob
// One 512-thread CTA per row.  Online (max, sum exp, sum exp*z) per thread,
// merged across the block.  Optional vocab offset/size (for a vocab shard):
// targets outside [v0, v0+V) contribute a zero target logit.
constexpr int kLpThreads = 512;

struct Online {
  float m, s, t;  // running max, sum exp(z - m), sum exp(z - m) * z
};

__device__ __forceinline__ Online online_merge(Online a, Online b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  const float m = fmaxf(a.m, b.m);
  const float ea = __expf(a.m - m), eb = __expf(b.m - m);
  return {m, a.s * ea + b.s * eb, a.t * ea + b.t * eb};
}

__global__ void __launch_bounds__(kLpThreads) logprob_fwd_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                                 const int64_t* __restrict__ targets, int V, int v0,
                                                                 float inv_temp, float* __restrict__ logp,
                                                                 float* __restrict__ entropy, float* __restrict__ stats,
                                                                 float* __restrict__ target_logit) {
  const int row = blockIdx.x;
  const __nv_bfloat16* z = logits + (size_t)row * ld;
  Online o = {-INFINITY, 0.f, 0.f};
  const int nvec = V >> 3;
  for (int v = threadIdx.x; v < nvec; v += kLpThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(z + v * 8);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
    float f[8];
    float lm = -INFINITY;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      f[e] = __bfloat162float(b[e]) * inv_temp;
      lm = fmaxf(lm, f[e]);
    }
    Online c = {lm, 0.f, 0.f};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float ex = __expf(f[e] - lm);
      c.s += ex;
      c.t += ex * f[e];
    }
    o = online_merge(o, c);
  }
  for (int v = nvec * 8 + threadIdx.x; v < V; v += kLpThreads) {  // ragged tail
    const float f = __bfloat162float(z[v]) * inv_temp;
    o = online_merge(o, Online{f, 1.f, f});
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Online p = {__shfl_xor_sync(0xffffffffu, o.m, off), __shfl_xor_sync(0xffffffffu, o.s, off),
                __shfl_xor_sync(0xffffffffu, o.t, off)};
    o = online_merge(o, p);
  }
  __shared__ Online sh[kLpThreads / 32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = o;
  __syncthreads();
  if (w == 0) {
    o = (l < kLpThreads / 32) ? sh[l] : Online{-INFINITY, 0.f, 0.f};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      Online p = {__shfl_xor_sync(0xffffffffu, o.m, off), __shfl_xor_sync(0xffffffffu, o.s, off),
                  __shfl_xor_sync(0xffffffffu, o.t, off)};
      o = online_merge(o, p);
    }
    if (l == 0) {
      const float lse = o.m + __logf(o.s);
      const int64_t tg = targets[row] - v0;
      const bool local = tg >= 0 && tg < V;
      const float zt = local ? __bfloat162float(z[tg]) * inv_temp : 0.f;
      if (stats) {
        stats[2 * row] = o.m;
        stats[2 * row + 1] = o.s;
      }
      if (target_logit) target_logit[row] = zt;
      if (logp) logp[row] = zt - lse;
      if (entropy) entropy[row] = lse - o.t / o.s;
    }
  }
}

// dz_j = g * (1[j == target] - softmax_j) * inv_temp, written over the logits.
__global__ void __launch_bounds__(kLpThreads) logprob_bwd_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld,
                                                                 const int64_t* __restrict__ targets, int V, int v0,
                                                                 float inv_temp, const float* __restrict__ lse,
                                                                 const float* __restrict__ grad) {
  const int row = blockIdx.x;
  __nv_bfloat16* z = logits + (size_t)row * ld;
  const float g = grad[row];
  const float L = lse[row];
  const int64_t tg = targets[row] - v0;
  const int nvec = V >> 3;
  for (int v = threadIdx.x; v < nvec; v += kLpThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(z + v * 8);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
    float d[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float p = __expf(__bfloat162float(b[e]) * inv_temp - L);
      d[e] = g * (((int64_t)(v * 8 + e) == tg ? 1.f : 0.f) - p) * inv_temp;
    }
    uint4 pk;
    pk.x = pack_bf16x2(d[0], d[1]);
    pk.y = pack_bf16x2(d[2], d[3]);
    pk.z = pack_bf16x2(d[4], d[5]);
    pk.w = pack_bf16x2(d[6], d[7]);
    *reinterpret_cast<uint4*>(z + v * 8) = pk;
  }
  for (int v = nvec * 8 + threadIdx.x; v < V; v += kLpThreads) {
    const float p = __expf(__bfloat162float(z[v]) * inv_temp - L);
    z[v] = __float2bfloat16(g * (((int64_t)v == tg ? 1.f : 0.f) - p) * inv_temp);
  }
}

// ------------------------------------------------------------------ AdamW
// sq_norm: device scalar holding sum(grad^2) (filled by grad_sq_norm); the step
// applies clip = min(1, max_norm / (sqrt(sq_norm) + 1e-6)) when max_norm > 0.
__global__ void grad_sq_norm_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ out) {
  float s = 0.f;
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(g)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s += g[i] * g[i];
  s = warp_sum(s);
  __shared__ float sh[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = s;
  __syncthreads();
  if (w == 0) {
    s = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.f;
    s = warp_sum(s);
    if (l == 0) atomicAdd(out, s);
  }
}

// Peer mode of the AdamW kernel (ZeRO-1 step fused with the parameter all-gather): every rank updates
// its shard and stores the new bf16 values straight into the same shard of every rank's parameter
// buffer (IPC-mapped peer memory), then bumps an arrival counter on every rank; CTA 0 waits (bounded)
// until every rank's CTAs have arrived, so the kernel ends only when the whole parameter vector is here.
constexpr int kAdamPeerMax = 8;
struct AdamPeers {
  uint64_t param[kAdamPeerMax];  // this rank's shard inside each rank's bf16 parameter buffer
  uint64_t flags[kAdamPeerMax];  // int32 arrival counters [kAdamPeerMax] of each rank
  int n, me, epoch;
  int* err;
};

// Adam moments in fp32, or in bf16 for the precision-aware optimizer (computed in fp32, stored rounded
// to nearest even): four consecutive moments per thread either way.
__device__ __forceinline__ float4 load_moment4(const float* p, int64_t i) { return reinterpret_cast<const float4*>(p)[i]; }
__device__ __forceinline__ float4 load_moment4(const __nv_bfloat16* p, int64_t i) {
  const uint2 u = reinterpret_cast<const uint2*>(p)[i];
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
__device__ __forceinline__ void store_moment4(float* p, int64_t i, float4 v) { reinterpret_cast<float4*>(p)[i] = v; }
__device__ __forceinline__ void store_moment4(__nv_bfloat16* p, int64_t i, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  reinterpret_cast<uint2*>(p)[i] = u;
}
__device__ __forceinline__ float moment_at(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float moment_at(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ void moment_set(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void moment_set(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16(v); }

template <bool kPeer, typename MT>
__global__ void adamw_kernel(float* __restrict__ master, const float* __restrict__ grad, MT* __restrict__ m,
                             MT* __restrict__ v, __nv_bfloat16* __restrict__ param, int64_t n, float lr, float beta1,
                             float beta2, float eps, float wd, float bc1, float bc2, const float* __restrict__ sq_norm,
                             float max_norm, float grad_scale, const AdamPeers peers) {
  float clip = grad_scale;
  if (max_norm > 0.f && sq_norm) {
    const float norm = sqrtf(*sq_norm) * grad_scale;
    clip = grad_scale * fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 p = reinterpret_cast<float4*>(master)[i];
    const float4 g4 = reinterpret_cast<const float4*>(grad)[i];
    float4 m4 = load_moment4(m, i);
    float4 v4 = load_moment4(v, i);
    float* pp = &p.x;
    const float* gg = &g4.x;
    float* mm = &m4.x;
    float* vv = &v4.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float g = gg[e] * clip;
      mm[e] = beta1 * mm[e] + (1.f - beta1) * g;
      vv[e] = beta2 * vv[e] + (1.f - beta2) * g * g;
      const float mhat = mm[e] / bc1, vhat = vv[e] / bc2;
      pp[e] = pp[e] - lr * (mhat / (sqrtf(vhat) + eps) + wd * pp[e]);
    }
    reinterpret_cast<float4*>(master)[i] = p;
    store_moment4(m, i, m4);
    store_moment4(v, i, v4);
    uint2 pk;
    pk.x = pack_bf16x2(p.x, p.y);
    pk.y = pack_bf16x2(p.z, p.w);
    if constexpr (kPeer) {
      for (int r = 0; r < peers.n; ++r) reinterpret_cast<uint2*>(peers.param[r])[i] = pk;
    } else {
      reinterpret_cast<uint2*>(param)[i] = pk;
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float g = grad[i] * clip;
    const float mi = beta1 * moment_at(m, i) + (1.f - beta1) * g;
    const float vi = beta2 * moment_at(v, i) + (1.f - beta2) * g * g;
    moment_set(m, i, mi);
    moment_set(v, i, vi);
    master[i] -= lr * ((mi / bc1) / (sqrtf(vi / bc2) + eps) + wd * master[i]);
    if constexpr (kPeer) {
      for (int r = 0; r < peers.n; ++r) reinterpret_cast<__nv_bfloat16*>(peers.param[r])[i] = __float2bfloat16(master[i]);
    } else {
      param[i] = __float2bfloat16(master[i]);
    }
  }
  if constexpr (kPeer) {
    __threadfence_system();
    __syncthreads();
    if ((int)threadIdx.x < peers.n)
      red_add_release_sys(reinterpret_cast<int*>(peers.flags[threadIdx.x]) + peers.me, 1);
    if (blockIdx.x == 0 && (int)threadIdx.x < peers.n)
      wait_flag_geq(reinterpret_cast<const int*>(peers.flags[peers.me]) + threadIdx.x,
                    peers.epoch * (int)gridDim.x, peers.err, kTimeoutPeerFlag);
  }
}

// ------------------------------------------------------------------ host wrappers
static int sm_count() {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  LIBRA_CHECK(gu.is_cuda() && gu.scalar_type() == at::kBFloat16 && gu.is_contiguous(), "swiglu_fwd: bf16 contiguous");
  const int F = (int)(gu.size(-1) / 2);
  LIBRA_CHECK(F % 8 == 0, "swiglu_fwd: F %% 8 == 0 required");
  const int64_t T = gu.numel() / (2 * F);
  const c10::cuda::CUDAGuard guard(gu.device());
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto h = torch::empty(sizes, gu.options());
  if (T == 0) return h;
  swiglu_fwd_kernel<<<sm_count() * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)h.data_ptr(), T, F);
  LIBRA_LAUNCH_CHECK();
  return h;
}

torch::Tensor swiglu_bwd(torch::Tensor gu, torch::Tensor dh) {
  LIBRA_CHECK(dh.is_contiguous() && gu.is_contiguous(), "swiglu_bwd: contiguous inputs");
  const int F = (int)(gu.size(-1) / 2);
  const int64_t T = gu.numel() / (2 * F);
  const c10::cuda::CUDAGuard guard(gu.device());
  auto dgu = torch::empty_like(gu);
  if (T == 0) return dgu;
  swiglu_bwd_kernel<<<sm_count() * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (const __nv_bfloat16*)dh.data_ptr(), (__nv_bfloat16*)dgu.data_ptr(), T, F);
  LIBRA_LAUNCH_CHECK();
  return dgu;
}

// Returns {logp [R], entropy [R], stats [R, 2] (max, sumexp), target_logit [R]}.
std::vector<torch::Tensor> logprob_fwd(torch::Tensor logits, torch::Tensor targets, int64_t vocab_start,
                                       double temperature, bool with_entropy) {
  LIBRA_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
              "logprob_fwd: 2-D bf16 logits");
  LIBRA_CHECK(logits.stride(0) % 8 == 0 && targets.scalar_type() == at::kLong, "logprob_fwd: ld %% 8 == 0 and int64 targets required");
  const int R = (int)logits.size(0), V = (int)logits.size(1);
  const c10::cuda::CUDAGuard guard(logits.device());
  auto opts = logits.options().dtype(at::kFloat);
  auto logp = torch::empty({R}, opts);
  auto ent = with_entropy ? torch::empty({R}, opts) : torch::empty({0}, opts);
  auto stats = torch::empty({R, 2}, opts);
  auto tl = torch::empty({R}, opts);
  if (R == 0) return {logp, ent, stats, tl};
  logprob_fwd_kernel<<<R, kLpThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)logits.data_ptr(), logits.stride(0), targets.data_ptr<int64_t>(), V, (int)vocab_start,
      (float)(1.0 / temperature), logp.data_ptr<float>(), with_entropy ? ent.data_ptr<float>() : nullptr,
      stats.data_ptr<float>(), tl.data_ptr<float>());
  LIBRA_LAUNCH_CHECK();
  return {logp, ent, stats, tl};
}

void logprob_bwd_(torch::Tensor logits, torch::Tensor targets, int64_t vocab_start, double temperature,
                  torch::Tensor lse, torch::Tensor grad) {
  const int R = (int)logits.size(0), V = (int)logits.size(1);
  LIBRA_CHECK(lse.is_contiguous() && grad.is_contiguous() && lse.numel() == R && grad.numel() == R,
              "logprob_bwd: lse/grad [R] fp32");
  const c10::cuda::CUDAGuard guard(logits.device());
  if (R == 0) return;
  logprob_bwd_kernel<<<R, kLpThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)logits.data_ptr(), logits.stride(0), targets.data_ptr<int64_t>(), V, (int)vocab_start,
      (float)(1.0 / temperature), lse.data_ptr<float>(), grad.data_ptr<float>());
  LIBRA_LAUNCH_CHECK();
}

void grad_sq_norm(torch::Tensor grad, torch::Tensor out) {
  LIBRA_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous() && out.scalar_type() == at::kFloat,
              "grad_sq_norm: fp32");
  const c10::cuda::CUDAGuard guard(grad.device());
  const int64_t n = grad.numel();
  if (n == 0) return;
  grad_sq_norm_kernel<<<sm_count() * 4, 512, 0, at::cuda::getCurrentCUDAStream()>>>(grad.data_ptr<float>(), n,
                                                                                    out.data_ptr<float>());
  LIBRA_LAUNCH_CHECK();
}

void adamw_step(torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v, torch::Tensor param,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                c10::optional<torch::Tensor> sq_norm, double max_norm, double grad_scale) {
  LIBRA_CHECK(master.scalar_type() == at::kFloat && grad.scalar_type() == at::kFloat &&
                  param.scalar_type() == at::kBFloat16 && m.scalar_type() == v.scalar_type() &&
                  (m.scalar_type() == at::kFloat || m.scalar_type() == at::kBFloat16),
              "adamw_step: fp32 master/grad, fp32 or bf16 moments (both the same), bf16 param");
  const int64_t n = master.numel();
  LIBRA_CHECK(grad.numel() == n && m.numel() == n && v.numel() == n && param.numel() == n, "adamw_step: size mismatch");
  LIBRA_CHECK(master.is_contiguous() && grad.is_contiguous() && m.is_contiguous() && v.is_contiguous() &&
                  param.is_contiguous(),
              "adamw_step: contiguous buffers");
  const c10::cuda::CUDAGuard guard(master.device());
  if (n == 0) return;
  const float bc1 = (float)(1.0 - std::pow(beta1, (double)step));
  const float bc2 = (float)(1.0 - std::pow(beta2, (double)step));
  const float* sq = sq_norm.has_value() ? sq_norm->data_ptr<float>() : nullptr;
  if (m.scalar_type() == at::kBFloat16)
    adamw_kernel<false, __nv_bfloat16><<<sm_count() * 4, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        master.data_ptr<float>(), grad.data_ptr<float>(), (__nv_bfloat16*)m.data_ptr(), (__nv_bfloat16*)v.data_ptr(),
        (__nv_bfloat16*)param.data_ptr(), n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2, sq,
        (float)max_norm, (float)grad_scale, AdamPeers{});
  else
    adamw_kernel<false, float><<<sm_count() * 4, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        master.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
        (__nv_bfloat16*)param.data_ptr(), n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2, sq,
        (float)max_norm, (float)grad_scale, AdamPeers{});
  LIBRA_LAUNCH_CHECK();
}

// AdamW on this rank's shard, fused with the parameter all-gather: param_peers[r] is the address of this
// rank's shard inside rank r's bf16 parameter buffer (mapped into this process), flag_peers[r] rank r's
// int32 arrival counters.  Same grid on every rank (grid_ctas > 0, agreed by the caller; 0 = 4 per SM);
// epoch counts the calls (1, 2, ...).
void adamw_step_allgather(torch::Tensor master, torch::Tensor grad, torch::Tensor m, torch::Tensor v, double lr,
                          double beta1, double beta2, double eps, double wd, int64_t step,
                          c10::optional<torch::Tensor> sq_norm, double max_norm, double grad_scale,
                          std::vector<int64_t> param_peers, std::vector<int64_t> flag_peers, int64_t me, int64_t epoch,
                          torch::Tensor err, int64_t grid_ctas) {
  LIBRA_CHECK(master.scalar_type() == at::kFloat && grad.scalar_type() == at::kFloat &&
                  m.scalar_type() == v.scalar_type() &&
                  (m.scalar_type() == at::kFloat || m.scalar_type() == at::kBFloat16),
              "adamw_step_allgather: fp32 master/grad, fp32 or bf16 moments (both the same)");
  const int64_t n = master.numel();
  LIBRA_CHECK(grad.numel() == n && m.numel() == n && v.numel() == n, "adamw_step_allgather: size mismatch");
  LIBRA_CHECK(master.is_contiguous() && grad.is_contiguous() && m.is_contiguous() && v.is_contiguous(),
              "adamw_step_allgather: contiguous buffers");
  const int nr = (int)param_peers.size();
  LIBRA_CHECK(nr >= 1 && nr <= kAdamPeerMax && (int)flag_peers.size() == nr && me >= 0 && me < nr,
              "adamw_step_allgather: 1..8 ranks with one parameter and one flag pointer each");
  AdamPeers peers{};
  for (int r = 0; r < nr; ++r) {
    LIBRA_CHECK((param_peers[r] & 7) == 0 && (flag_peers[r] & 3) == 0,
                "adamw_step_allgather: parameter shards must be 8-byte aligned");
    peers.param[r] = (uint64_t)param_peers[r];
    peers.flags[r] = (uint64_t)flag_peers[r];
  }
  // the arrival target is epoch * grid, so every rank must launch the same grid: callers agree on it
  const int grid = grid_ctas > 0 ? (int)grid_ctas : sm_count() * 4;
  LIBRA_CHECK(grid <= 65535, "adamw_step_allgather: grid of %d CTAs is too large", grid);
  LIBRA_CHECK(epoch >= 1 && epoch * grid < ((int64_t)1 << 31), "adamw_step_allgather: epoch out of range");
  peers.n = nr;
  peers.me = (int)me;
  peers.epoch = (int)epoch;
  peers.err = err.data_ptr<int>();
  const c10::cuda::CUDAGuard guard(master.device());
  const float bc1 = (float)(1.0 - std::pow(beta1, (double)step));
  const float bc2 = (float)(1.0 - std::pow(beta2, (double)step));
  // launched even for an empty shard: the peers wait for this rank's arrivals
  const float* sq = sq_norm.has_value() ? sq_norm->data_ptr<float>() : nullptr;
  if (m.scalar_type() == at::kBFloat16)
    adamw_kernel<true, __nv_bfloat16><<<grid, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        master.data_ptr<float>(), grad.data_ptr<float>(), (__nv_bfloat16*)m.data_ptr(), (__nv_bfloat16*)v.data_ptr(),
        nullptr, n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2, sq, (float)max_norm,
        (float)grad_scale, peers);
  else
    adamw_kernel<true, float><<<grid, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        master.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), nullptr, n,
        (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2, sq, (float)max_norm,
        (float)grad_scale, peers);
  LIBRA_LAUNCH_CHECK();
}

}  // namespace libra

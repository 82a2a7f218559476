// Distributed-optimizer gradient reduce-scatter over NVLink peer memory, fused
// with the data-parallel average and the global gradient norm.
//
// The reference reduces gradients with Megatron's distributed optimizer
// (engine/megatron_core_train_engine.py:209-222 finalize_model_grads, then the
// optimizer's reduce-scatter and a separate clip-norm all-reduce).  Here every
// data-parallel rank keeps its fp32 gradient in one flat buffer with the same
// layout, and rank r owns shard r of it.  One kernel per step, on every rank:
//
//   1. arrive: each CTA bumps this rank's "ready" counter on every rank (a CTA
//      that runs proves the kernels that wrote this rank's gradient are done);
//      then waits (bounded) until every rank has at least one CTA running;
//   2. reduce: grid-stride over the owned shard, loading the shard from every
//      rank's gradient (peer loads over NVLink, all ranks' float4 in flight at
//      once), summing in rank order, scaling by 1/dp, writing the fp32 shard,
//      and accumulating the sum of squares of the result;
//   3. depart: each CTA adds its partial sum of squares into every rank's
//      norm slot and bumps its "done" counter there; CTA 0 waits (bounded)
//      until every CTA of every rank is done, so when the kernel ends no rank
//      still reads this rank's gradient (the next step may zero it) and the
//      norm slot holds the global sum, which CTA 0 copies out and clears.
//
// Every rank launches the same grid (the callers agree on it); counters count
// calls x grid, so they only grow.  The norm slots alternate by call parity.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace libra {
namespace {

constexpr int kGrsMax = 8;
// counter area of each rank: int32[64]
constexpr int kGrsReady = 0;  // [0, 8): CTAs of rank s that started, per source rank s
constexpr int kGrsDone = 8;   // [8, 16): CTAs of rank s that finished
constexpr int kGrsSlot = 16;  // [16, 18): fp32 sum-of-squares slots, alternating by call parity

struct GrsPeers {
  uint64_t src[kGrsMax];    // this rank's shard inside rank r's fp32 gradient buffer (mapped here)
  uint64_t flags[kGrsMax];  // rank r's counter area (mapped here)
  int me, epoch;
  int* err;
};

__device__ __forceinline__ void red_add_f32_sys(float* p, float v) {
  asm volatile("red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ float ld_acquire_sys_f32(const float* p) {
  float v;
  asm volatile("ld.acquire.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

template <int N>
__global__ void __launch_bounds__(512) grad_rs_peer_kernel(float* __restrict__ out, int64_t n, float scale,
                                                            float* __restrict__ sq_out, const GrsPeers P) {
  __shared__ float red[16];
  const int t = threadIdx.x;
  if (t < N) red_add_release_sys(reinterpret_cast<int*>(P.flags[t]) + kGrsReady + P.me, 1);
  bool ok = true;
  if (t < N)
    ok = wait_flag_geq(reinterpret_cast<const int*>(P.flags[P.me]) + kGrsReady + t,
                       (P.epoch - 1) * (int)gridDim.x + 1, P.err, kTimeoutPeerFlag);
  ok = __syncthreads_and(ok);
  float acc = 0.f;
  if (ok) {
    const int64_t n4 = n >> 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // U grid-stride steps per iteration: N x U 16-byte loads in flight per thread (few ranks leave
    // the loop latency-bound with one step)
    constexpr int U = N <= 4 ? 2 : 1;
    for (int64_t i0 = blockIdx.x * (int64_t)blockDim.x + t; i0 < n4; i0 += stride * U) {
      float4 v[U][N];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * stride;
#pragma unroll
        for (int r = 0; r < N; ++r)
          v[u][r] = i < n4 ? __ldcs(reinterpret_cast<const float4*>(P.src[r]) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * stride;
        if (i >= n4) break;
        float4 s = v[u][0];
#pragma unroll
        for (int r = 1; r < N; ++r) {
          s.x += v[u][r].x;
          s.y += v[u][r].y;
          s.z += v[u][r].z;
          s.w += v[u][r].w;
        }
        s.x *= scale;
        s.y *= scale;
        s.z *= scale;
        s.w *= scale;
        reinterpret_cast<float4*>(out)[i] = s;
        acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
      }
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + t; i < n; i += stride) {
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < N; ++r) s += reinterpret_cast<const float*>(P.src[r])[i];
      s *= scale;
      out[i] = s;
      acc += s * s;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((t & 31) == 0) red[t >> 5] = acc;
  __syncthreads();
  if (t < 32) {
    float a = t < (int)(blockDim.x >> 5) ? red[t] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (t == 0) red[0] = a;
  }
  __syncthreads();
  if (t < N) {
    int* fl = reinterpret_cast<int*>(P.flags[t]);
    red_add_f32_sys(reinterpret_cast<float*>(fl + kGrsSlot + (P.epoch & 1)), red[0]);
    red_add_release_sys(fl + kGrsDone + P.me, 1);  // also orders this CTA's loads of rank t's gradient
  }
  if (blockIdx.x == 0) {
    bool done = true;
    if (t < N)
      done = wait_flag_geq(reinterpret_cast<const int*>(P.flags[P.me]) + kGrsDone + t, P.epoch * (int)gridDim.x,
                           P.err, kTimeoutPeerFlag);
    done = __syncthreads_and(done);
    if (t == 0) {
      float* slot = reinterpret_cast<float*>(reinterpret_cast<int*>(P.flags[P.me]) + kGrsSlot + (P.epoch & 1));
      const float total = ld_acquire_sys_f32(slot);
      // cleared for the call after next, which adds into it only after every rank finished the next call
      *slot = 0.f;
      if (sq_out) *sq_out = done ? total : 0.f;
    }
  }
}

int sm_count_here() {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

// out [S] fp32 (this rank's shard of the reduced, averaged gradient); src_peers[r] = address of this
// rank's shard inside rank r's fp32 gradient; flag_peers[r] = rank r's int32[64] counter area.
// sq_out (fp32 [1], optional) receives the global sum of squares of the averaged gradient.
void grad_reduce_scatter_peer(torch::Tensor out, double scale, c10::optional<torch::Tensor> sq_out,
                              std::vector<int64_t> src_peers, std::vector<int64_t> flag_peers, int64_t me,
                              int64_t epoch, torch::Tensor err, int64_t grid_ctas) {
  LIBRA_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(),
              "grad_reduce_scatter_peer: contiguous fp32 CUDA output");
  const int nr = (int)src_peers.size();
  LIBRA_CHECK(nr >= 1 && nr <= kGrsMax && (int)flag_peers.size() == nr && me >= 0 && me < nr,
              "grad_reduce_scatter_peer: 1..8 ranks with one gradient and one counter pointer each");
  LIBRA_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "grad_reduce_scatter_peer: output 16-byte aligned");
  GrsPeers P{};
  for (int r = 0; r < nr; ++r) {
    LIBRA_CHECK((src_peers[r] & 15) == 0 && (flag_peers[r] & 15) == 0,
                "grad_reduce_scatter_peer: gradient shards and counter areas must be 16-byte aligned");
    P.src[r] = (uint64_t)src_peers[r];
    P.flags[r] = (uint64_t)flag_peers[r];
  }
  if (sq_out.has_value())
    LIBRA_CHECK(sq_out->is_cuda() && sq_out->scalar_type() == at::kFloat && sq_out->numel() >= 1,
                "grad_reduce_scatter_peer: fp32 norm output");
  const int grid = grid_ctas > 0 ? (int)grid_ctas : sm_count_here() * 4;
  LIBRA_CHECK(grid <= 65535, "grad_reduce_scatter_peer: grid of %d CTAs is too large", grid);
  LIBRA_CHECK(epoch >= 1 && epoch * grid < ((int64_t)1 << 31), "grad_reduce_scatter_peer: epoch out of range");
  P.me = (int)me;
  P.epoch = (int)epoch;
  P.err = err.data_ptr<int>();
  const c10::cuda::CUDAGuard guard(out.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  float* o = out.data_ptr<float>();
  float* sq = sq_out.has_value() ? sq_out->data_ptr<float>() : nullptr;
  const int64_t n = out.numel();
  const float s = (float)scale;
  // launched even for an empty shard: the peers count this rank's CTAs
  switch (nr) {
#define LIBRA_GRS_CASE(K) \
  case K:                 \
    grad_rs_peer_kernel<K><<<grid, 512, 0, stream>>>(o, n, s, sq, P); \
    break;
    LIBRA_GRS_CASE(1)
    LIBRA_GRS_CASE(2)
    LIBRA_GRS_CASE(3)
    LIBRA_GRS_CASE(4)
    LIBRA_GRS_CASE(5)
    LIBRA_GRS_CASE(6)
    LIBRA_GRS_CASE(7)
    LIBRA_GRS_CASE(8)
#undef LIBRA_GRS_CASE
  }
  LIBRA_LAUNCH_CHECK();
}

}  // namespace libra

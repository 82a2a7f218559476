// Tensor-parallel all-reduce over NVLink peer memory, fused with the residual
// add and the following RMSNorm (rollout decode: o-proj / down-proj outputs).
//
// Every TP rank owns a peer-visible buffer: 2 slots of [max_rows, H] bf16 for
// partial GEMM outputs (the row-parallel GEMM writes its partial straight into
// the current slot) followed by a flag area [kMaxCtas][kMaxRanks] int32.  One
// launch per call on every rank, same grid everywhere:
//   1. CTA b publishes "partial ready" by storing `epoch` into flag[b][me] of
//      every peer (release, system scope), then waits until its own
//      flag[b][p] >= epoch for every p (acquire, bounded by a time limit);
//   2. each warp takes one row: reads that row of all N partials over NVLink
//      (16-byte loads), sums in fp32, adds the residual, writes x_out, and
//      writes h_out = rmsnorm(x_out) * w.
// Slots alternate between calls, so one barrier per call suffices: a rank can
// only overwrite a slot after every peer has passed the next call's barrier,
// that is, after every peer has finished reading it.  Epochs grow
// monotonically, so flags never need resetting.
// No TMA and no multicast: plain peer loads and stores.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace libra {
namespace tp {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 512;  // up to 4096 rows in one wave of 8-warp CTAs
constexpr int kWarps = 8;

struct PeerPtrs {
  uint64_t data[kMaxRanks];   // base of each rank's slot area
  uint64_t flags[kMaxRanks];  // base of each rank's flag area
};

__global__ void __launch_bounds__(kWarps * 32) allreduce_add_rmsnorm_kernel(
    const PeerPtrs ptrs, int nranks, int me, size_t slot_off, int B, int H, const __nv_bfloat16* __restrict__ residual,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* __restrict__ x_out, __nv_bfloat16* __restrict__ h_out,
    int epoch, int* err) {
  __shared__ int s_ok;
  // ---- barrier: my partial is ready; wait for everyone's
  if (threadIdx.x < nranks) {
    int* peer_flag = reinterpret_cast<int*>(ptrs.flags[threadIdx.x]) + blockIdx.x * kMaxRanks + me;
    __threadfence_system();
    st_release_sys(peer_flag, epoch);
  }
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < nranks) {
    const int* mine = reinterpret_cast<const int*>(ptrs.flags[me]) + blockIdx.x * kMaxRanks + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if ((++spins & 1023u) == 0u && globaltimer_ns() - t0 > wait_budget_ns(err)) {
        atomicCAS(err, 0, kTimeoutPeerFlag);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (!s_ok) return;
  // ---- reduce + residual + RMSNorm, one warp per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = H >> 3;
  for (int row = blockIdx.x * kWarps + warp; row < B; row += gridDim.x * kWarps) {
    float ss = 0.f;
    for (int v = lane; v < nvec; v += 32) {
      float acc[8];
      const uint4 r = reinterpret_cast<const uint4*>(residual + (size_t)row * H)[v];
      const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __bfloat162float(rb[e]);
      for (int p = 0; p < nranks; ++p) {
        const __nv_bfloat16* src =
            reinterpret_cast<const __nv_bfloat16*>(ptrs.data[p] + slot_off) + (size_t)row * H;
        const uint4 u = reinterpret_cast<const uint4*>(src)[v];
        const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += __bfloat162float(ub[e]);
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(x_out + (size_t)row * H)[v] = o;
      const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float q = __bfloat162float(ob[e]);
        ss += q * q;
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / (float)H + eps);
    for (int v = lane; v < nvec; v += 32) {
      const uint4 xv = reinterpret_cast<const uint4*>(x_out + (size_t)row * H)[v];
      const uint4 wv = reinterpret_cast<const uint4*>(w)[v];
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 o;
      o.x = pack_bf16x2(__bfloat162float(xb[0]) * rstd * __bfloat162float(wb[0]),
                        __bfloat162float(xb[1]) * rstd * __bfloat162float(wb[1]));
      o.y = pack_bf16x2(__bfloat162float(xb[2]) * rstd * __bfloat162float(wb[2]),
                        __bfloat162float(xb[3]) * rstd * __bfloat162float(wb[3]));
      o.z = pack_bf16x2(__bfloat162float(xb[4]) * rstd * __bfloat162float(wb[4]),
                        __bfloat162float(xb[5]) * rstd * __bfloat162float(wb[5]));
      o.w = pack_bf16x2(__bfloat162float(xb[6]) * rstd * __bfloat162float(wb[6]),
                        __bfloat162float(xb[7]) * rstd * __bfloat162float(wb[7]));
      reinterpret_cast<uint4*>(h_out + (size_t)row * H)[v] = o;
    }
  }
}

// data_ptrs / flag_ptrs: one int64 address per rank (peer mappings of the
// ranks' buffers in this process).  Returns {x_out, h_out}.
std::vector<torch::Tensor> allreduce_add_rmsnorm(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs,
                                                 int64_t me, int64_t slot_offset_bytes, torch::Tensor residual,
                                                 torch::Tensor w, double eps, int64_t epoch, int64_t grid,
                                                 torch::Tensor err) {
  const int n = (int)data_ptrs.size();
  LIBRA_CHECK(n >= 1 && n <= kMaxRanks && (int)flag_ptrs.size() == n && me >= 0 && me < n,
              "tp_allreduce: 1..8 ranks with one data and one flag pointer each");
  LIBRA_CHECK(residual.is_cuda() && residual.scalar_type() == at::kBFloat16 && residual.dim() == 2 &&
                  residual.is_contiguous(),
              "tp_allreduce: residual must be a contiguous CUDA bf16 [B, H] tensor");
  const int B = (int)residual.size(0), H = (int)residual.size(1);
  LIBRA_CHECK(H % 8 == 0 && w.numel() == H && w.scalar_type() == at::kBFloat16, "tp_allreduce: H %% 8 and w [H]");
  LIBRA_CHECK(grid >= 1 && grid <= kMaxCtas, "tp_allreduce: grid must be in [1, %d]", kMaxCtas);
  LIBRA_CHECK(slot_offset_bytes % 16 == 0, "tp_allreduce: slot offset must be 16-byte aligned");
  PeerPtrs p{};
  for (int i = 0; i < n; ++i) {
    LIBRA_CHECK((data_ptrs[i] & 15) == 0 && (flag_ptrs[i] & 3) == 0, "tp_allreduce: misaligned peer pointer");
    p.data[i] = (uint64_t)data_ptrs[i];
    p.flags[i] = (uint64_t)flag_ptrs[i];
  }
  const c10::cuda::CUDAGuard guard(residual.device());
  auto x_out = torch::empty_like(residual);
  auto h_out = torch::empty_like(residual);
  allreduce_add_rmsnorm_kernel<<<(int)grid, kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, n, (int)me, (size_t)slot_offset_bytes, B, H, reinterpret_cast<const __nv_bfloat16*>(residual.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps,
      reinterpret_cast<__nv_bfloat16*>(x_out.data_ptr()), reinterpret_cast<__nv_bfloat16*>(h_out.data_ptr()),
      (int)epoch, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
  return {x_out, h_out};
}

}  // namespace tp
}  // namespace libra

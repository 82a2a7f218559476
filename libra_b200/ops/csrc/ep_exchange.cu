// Expert-parallel MoE token dispatch and combine over NVLink peer memory.
//
// Every rank of the expert-parallel group owns one peer-visible buffer holding
//   rx : 2 slots of [max_rows, H] bf16   (push target: rows other ranks send here)
//   tx : 2 slots of [max_rows, H] bf16   (pull source: expert outputs / gradients)
//   flags: int32 push_cnt[8], pull_rdy[8] (monotone arrival counters, one per source rank)
// A routing plan gives, for every (token, k) assignment j = t * k + kk, the rank
// that owns its expert and the row it occupies in that rank's slot (rows are
// grouped by local expert on the receiver, so the expert MLP is a plain grouped
// GEMM).  Two kernels, adjoint to each other:
//   ep_push  (dispatch; backward of combine): warp per assignment, stores row
//            x[j / k] (optionally scaled by s[j]) straight into the owner's rx
//            slot with 16-byte peer stores; every CTA then bumps push_cnt[me] on
//            every rank, and CTA 0 waits until each source's counter reaches
//            epoch * grid, so the kernel ends only when all rows addressed to
//            this rank have landed.
//   ep_pull  (combine; backward of dispatch): CTA 0 publishes "my tx slot is
//            written" to every rank, every CTA waits for all ranks' flags, then
//            a warp per token loads its k rows from the owners' tx slots and
//            writes out[t] = residual[t] + sum_k w[t, k] * row (fp32 sum), and
//            optionally the raw gathered rows (saved for the weight gradient).
// Slot reuse: a rank writes slot (c & 1) again at call c + 2, and by then every
// peer has finished call c, because each call waits for every peer's signal of
// call c + 1.  All waits are bounded (LIBRA_WAIT_NS); on timeout the kernel
// records kTimeoutPeerFlag and returns.  Out-of-range rows record kBadArgument
// and are skipped.  Plain peer loads and stores only: no TMA, no multicast.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace libra {
namespace ep {

constexpr int kMaxRanks = 8;
constexpr int kWarps = 8;
constexpr int kPushFlags = 0;
constexpr int kPullFlags = kMaxRanks;

struct Peers {
  uint64_t data[kMaxRanks];   // slot area (rx for push, tx for pull) of each rank
  uint64_t flags[kMaxRanks];  // flag area of each rank
};

__device__ __forceinline__ int* flag_at(uint64_t base, int i) { return reinterpret_cast<int*>(base) + i; }

__device__ __forceinline__ uint4 scale_bf16x8(uint4 u, float s) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(b[e]);
    ow[e] = pack_bf16x2(f.x * s, f.y * s);
  }
  return o;
}

__global__ void __launch_bounds__(kWarps * 32) ep_push_kernel(const Peers P, int n, int me, size_t slot_off,
                                                              const __nv_bfloat16* __restrict__ x,
                                                              const float* __restrict__ scale,
                                                              const int* __restrict__ dst_rank,
                                                              const int* __restrict__ dst_row, int rows, int k, int H,
                                                              int max_rows, int epoch, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = H >> 3;
  for (int j = blockIdx.x * kWarps + warp; j < rows; j += gridDim.x * kWarps) {
    const int r = dst_rank[j];
    const int drow = dst_row[j];
    if (r < 0) continue;  // dropped assignment
    if (r >= n || drow < 0 || drow >= max_rows) {
      if (lane == 0) atomicCAS(err, 0, kBadArgument);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(j / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(P.data[r] + slot_off) + (size_t)drow * nvec;
    const float s = scale ? scale[j] : 1.f;
    for (int v0 = lane; v0 < nvec; v0 += 128) {
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (v0 + 32 * q < nvec) u[q] = src[v0 + 32 * q];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (v0 + 32 * q < nvec) dst[v0 + 32 * q] = scale ? scale_bf16x8(u[q], s) : u[q];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < n) red_add_release_sys(flag_at(P.flags[threadIdx.x], kPushFlags + me), 1);
  if (blockIdx.x == 0 && threadIdx.x < n)
    wait_flag_geq(flag_at(P.flags[me], kPushFlags + threadIdx.x), epoch * (int)gridDim.x, err, kTimeoutPeerFlag);
}

__global__ void __launch_bounds__(kWarps * 32) ep_pull_kernel(const Peers P, int n, int me, size_t slot_off,
                                                              const float* __restrict__ weight,
                                                              const __nv_bfloat16* __restrict__ residual,
                                                              const int* __restrict__ src_rank,
                                                              const int* __restrict__ src_row, int T, int k, int H,
                                                              int max_rows, __nv_bfloat16* __restrict__ out,
                                                              __nv_bfloat16* __restrict__ gath, int epoch, int* err) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x < n) {
    __threadfence_system();
    red_add_release_sys(flag_at(P.flags[threadIdx.x], kPullFlags + me), 1);
  }
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < n && !wait_flag_geq(flag_at(P.flags[me], kPullFlags + threadIdx.x), epoch, err, kTimeoutPeerFlag))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = H >> 3;
  for (int t = blockIdx.x * kWarps + warp; t < T; t += gridDim.x * kWarps) {
    // lane q < k holds assignment q of this token
    int my_r = -1, my_row = 0;
    float my_w = 1.f;
    if (lane < k) {
      const int j = t * k + lane;
      my_r = src_rank[j];
      my_row = src_row[j];
      if (weight) my_w = weight[j];
      if (my_r >= n || (my_r >= 0 && (my_row < 0 || my_row >= max_rows))) {
        atomicCAS(err, 0, kBadArgument);
        my_r = -1;
      }
      if (my_r < 0) my_w = 0.f;
    }
    // warp-uniform trip count: every lane takes part in the shuffles below
    for (int v0 = 0; v0 < nvec; v0 += 32) {
      const int v = v0 + lane;
      const bool act = v < nvec;
      float acc[8];
      if (residual && act) {
        const uint4 rv = reinterpret_cast<const uint4*>(residual + (size_t)t * H)[v];
        const __nv_bfloat162* rb = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(rb[e]);
          acc[2 * e] = f.x;
          acc[2 * e + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      }
      for (int q0 = 0; q0 < k; q0 += 4) {
        uint4 u[4];
        float w[4];
        bool ok[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int src_lane = (q0 + q) & 31;
          const int r = __shfl_sync(0xffffffffu, my_r, src_lane);
          const int row = __shfl_sync(0xffffffffu, my_row, src_lane);
          w[q] = __shfl_sync(0xffffffffu, my_w, src_lane);
          ok[q] = (q0 + q < k) && r >= 0;
          if (ok[q] && act) u[q] = (reinterpret_cast<const uint4*>(P.data[r] + slot_off) + (size_t)row * nvec)[v];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (!ok[q] || !act) continue;
          if (gath) (reinterpret_cast<uint4*>(gath + ((size_t)t * k + q0 + q) * H))[v] = u[q];
          const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u[q]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(b[e]);
            acc[2 * e] = fmaf(w[q], f.x, acc[2 * e]);
            acc[2 * e + 1] = fmaf(w[q], f.y, acc[2 * e + 1]);
          }
        }
        if (gath) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (q0 + q < k && !ok[q] && act)
              (reinterpret_cast<uint4*>(gath + ((size_t)t * k + q0 + q) * H))[v] = make_uint4(0, 0, 0, 0);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      if (act) reinterpret_cast<uint4*>(out + (size_t)t * H)[v] = o;
    }
  }
}

static void check_bf16_rows(const torch::Tensor& t, const char* name) {
  LIBRA_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() &&
                  (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
              "%s must be a contiguous, 16-byte aligned bf16 CUDA tensor", name);
}

static Peers make_peers(const std::vector<int64_t>& data, const std::vector<int64_t>& flags, int64_t me,
                        int64_t slot_off) {
  const int n = (int)data.size();
  LIBRA_CHECK(n >= 1 && n <= kMaxRanks && (int)flags.size() == n && me >= 0 && me < n,
              "ep exchange: 1..8 ranks with one data and one flag pointer each");
  LIBRA_CHECK(slot_off % 16 == 0, "ep exchange: slot offset must be 16-byte aligned");
  Peers p{};
  for (int i = 0; i < n; ++i) {
    LIBRA_CHECK((data[i] & 15) == 0 && (flags[i] & 3) == 0, "ep exchange: misaligned peer pointer");
    p.data[i] = (uint64_t)data[i];
    p.flags[i] = (uint64_t)flags[i];
  }
  return p;
}

static void check_plan(const torch::Tensor& rank, const torch::Tensor& row, int64_t count, const char* what) {
  LIBRA_CHECK(rank.is_cuda() && row.is_cuda() && rank.scalar_type() == at::kInt && row.scalar_type() == at::kInt &&
                  rank.is_contiguous() && row.is_contiguous() && rank.numel() == count && row.numel() == count,
              "%s: plan ranks / rows must be contiguous int32 CUDA tensors of T*k entries", what);
}

// Dispatch: rows x[j / k] (times scale[j]) -> rank dst_rank[j], row dst_row[j] of its rx slot.
void ep_push(std::vector<int64_t> rx, std::vector<int64_t> flags, int64_t me, int64_t slot_off, torch::Tensor x,
             c10::optional<torch::Tensor> scale, torch::Tensor dst_rank, torch::Tensor dst_row, int64_t k,
             int64_t max_rows, int64_t epoch, int64_t grid, torch::Tensor err) {
  const Peers p = make_peers(rx, flags, me, slot_off);
  check_bf16_rows(x, "ep_push x");
  const int64_t T = x.size(0), H = x.size(1);
  LIBRA_CHECK(x.dim() == 2 && H % 8 == 0 && k >= 1 && k <= 32, "ep_push: x [T, H] with H %% 8 == 0, 1 <= k <= 32");
  LIBRA_CHECK(T * k < ((int64_t)1 << 31) && max_rows < ((int64_t)1 << 31), "ep_push: too many rows");
  check_plan(dst_rank, dst_row, T * k, "ep_push");
  if (scale) {
    LIBRA_CHECK(scale->is_cuda() && scale->scalar_type() == at::kFloat && scale->is_contiguous() &&
                    scale->numel() == T * k,
                "ep_push: scale must be contiguous fp32 [T*k]");
  }
  LIBRA_CHECK(grid >= 1 && grid <= 1024 && epoch >= 1 && epoch * grid < ((int64_t)1 << 31),
              "ep_push: grid in [1, 1024] and epoch * grid < 2^31");
  const c10::cuda::CUDAGuard guard(x.device());
  ep_push_kernel<<<(int)grid, kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, (int)rx.size(), (int)me, (size_t)slot_off, reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      scale ? scale->data_ptr<float>() : nullptr, dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(), (int)(T * k),
      (int)k, (int)H, (int)max_rows, (int)epoch, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
}

// Combine: out[t] = residual[t] + sum_kk weight[t*k+kk] * tx_slot[src_rank][src_row]; gath (optional) gets the
// raw gathered rows [T*k, H] (zeros for dropped assignments).
void ep_pull(std::vector<int64_t> tx, std::vector<int64_t> flags, int64_t me, int64_t slot_off,
             c10::optional<torch::Tensor> weight, c10::optional<torch::Tensor> residual, torch::Tensor src_rank,
             torch::Tensor src_row, int64_t k, int64_t max_rows, torch::Tensor out, c10::optional<torch::Tensor> gath,
             int64_t epoch, int64_t grid, torch::Tensor err) {
  const Peers p = make_peers(tx, flags, me, slot_off);
  check_bf16_rows(out, "ep_pull out");
  const int64_t T = out.size(0), H = out.size(1);
  LIBRA_CHECK(out.dim() == 2 && H % 8 == 0 && k >= 1 && k <= 32, "ep_pull: out [T, H] with H %% 8 == 0, 1 <= k <= 32");
  LIBRA_CHECK(T * k < ((int64_t)1 << 31) && max_rows < ((int64_t)1 << 31), "ep_pull: too many rows");
  check_plan(src_rank, src_row, T * k, "ep_pull");
  if (weight) {
    LIBRA_CHECK(weight->is_cuda() && weight->scalar_type() == at::kFloat && weight->is_contiguous() &&
                    weight->numel() == T * k,
                "ep_pull: weight must be contiguous fp32 [T*k]");
  }
  if (residual) {
    check_bf16_rows(*residual, "ep_pull residual");
    LIBRA_CHECK(residual->numel() == T * H, "ep_pull: residual [T, H]");
  }
  if (gath) {
    check_bf16_rows(*gath, "ep_pull gath");
    LIBRA_CHECK(gath->numel() == T * k * H, "ep_pull: gath [T*k, H]");
  }
  LIBRA_CHECK(grid >= 1 && grid <= 1024 && epoch >= 1, "ep_pull: grid in [1, 1024], epoch >= 1");
  const c10::cuda::CUDAGuard guard(out.device());
  ep_pull_kernel<<<(int)grid, kWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, (int)tx.size(), (int)me, (size_t)slot_off, weight ? weight->data_ptr<float>() : nullptr,
      residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr, src_rank.data_ptr<int>(),
      src_row.data_ptr<int>(), (int)T, (int)k, (int)H, (int)max_rows,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      gath ? reinterpret_cast<__nv_bfloat16*>(gath->data_ptr()) : nullptr, (int)epoch, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
}

}  // namespace ep
}  // namespace libra

// Vocab-parallel log-softmax: the per-row (max, sum of exp, target logit)
// exchange over NVLink peer memory.
//
// With the LM head split over the tensor-parallel group by vocabulary, each
// rank's logprob kernel reduces its own shard to three numbers per row: the
// shard's max logit m_q, its sum of exp(z - m_q), and the target logit when the
// target token falls in the shard (0 elsewhere).  The global log-partition is
// lse = M + log(sum_q s_q exp(m_q - M)) with M = max_q m_q, and the target logit
// is sum_q zt_q.  The reference gets these from two NCCL all-reduces (max, then
// sum); here one kernel does it:
//
//   1. push: CTA i stores its rows' (m, s, zt) into this rank's slot of every
//      rank's exchange buffer (peer stores over NVLink), then, after one
//      system-scope fence, publishes the call's epoch in its flag on every rank;
//   2. wait (bounded) until CTA i of every rank has published this epoch;
//   3. combine its rows from the local buffer and write lse and the target logit.
//
// CTA i of every rank covers the same rows, so each CTA synchronises only with
// its counterparts.  Data slots alternate by call parity: a rank can start
// writing a parity again only after every rank finished the call that read it.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace libra {
namespace vx {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;
constexpr int kThreads = 256;

struct Peers {
  uint64_t data[kMaxRanks];   // rank q's exchange area: float4 [2 parity][kMaxRanks][max_rows]
  uint64_t flags[kMaxRanks];  // rank q's flags: int32 [kMaxCtas][kMaxRanks]
};

__global__ void __launch_bounds__(kThreads) vocab_exchange_kernel(const Peers P, int n, int me, int max_rows, int R,
                                                                   const float* __restrict__ m,
                                                                   const float* __restrict__ s,
                                                                   const float* __restrict__ zt,
                                                                   float* __restrict__ lse, float* __restrict__ zt_out,
                                                                   int epoch, int* err) {
  __shared__ int s_ok;
  const int per = (R + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per, r1 = min(R, r0 + per);
  const int parity = epoch & 1;
  // 1. push this CTA's rows into every rank's slot for this rank
  for (int row = r0 + (int)threadIdx.x; row < r1; row += blockDim.x) {
    const float4 v = make_float4(m[row], s[row], zt[row], 0.f);
    for (int q = 0; q < n; ++q)
      reinterpret_cast<float4*>(P.data[q])[((size_t)parity * kMaxRanks + me) * max_rows + row] = v;
  }
  __syncthreads();  // the CTA's stores precede the signalling threads' fence
  if ((int)threadIdx.x < n) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<int*>(P.flags[threadIdx.x]) + blockIdx.x * kMaxRanks + me, epoch);
  }
  // 2. wait for CTA blockIdx.x of every rank
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < n &&
      !wait_flag_geq(reinterpret_cast<const int*>(P.flags[me]) + blockIdx.x * kMaxRanks + threadIdx.x, epoch, err,
                     kTimeoutPeerFlag))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;
  // 3. combine from the local buffer
  const float4* mine = reinterpret_cast<const float4*>(P.data[me]) + (size_t)parity * kMaxRanks * max_rows;
  for (int row = r0 + (int)threadIdx.x; row < r1; row += blockDim.x) {
    float4 v[kMaxRanks];
    float M = -INFINITY;
    for (int q = 0; q < n; ++q) {
      v[q] = mine[(size_t)q * max_rows + row];
      M = fmaxf(M, v[q].x);
    }
    float S = 0.f, Z = 0.f;
    for (int q = 0; q < n; ++q) {
      S += v[q].y * expf(v[q].x - M);
      Z += v[q].z;
    }
    lse[row] = M + logf(S);
    zt_out[row] = Z;
  }
}

}  // namespace vx

// data_ptrs / flag_ptrs: every rank's exchange area and flags as mapped here.  m, s, zt: this rank's
// per-row shard statistics (fp32 [R]).  Returns {lse, target logit}, fp32 [R].
std::vector<torch::Tensor> vocab_stats_exchange(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs,
                                                int64_t me, int64_t max_rows, torch::Tensor m, torch::Tensor s,
                                                torch::Tensor zt, int64_t epoch, torch::Tensor err) {
  using namespace vx;
  const int n = (int)data_ptrs.size();
  LIBRA_CHECK(n >= 1 && n <= kMaxRanks && (int)flag_ptrs.size() == n && me >= 0 && me < n,
              "vocab_stats_exchange: 1..8 ranks with one data and one flag pointer each");
  const int64_t R = m.numel();
  LIBRA_CHECK(m.is_cuda() && m.scalar_type() == at::kFloat && s.scalar_type() == at::kFloat &&
                  zt.scalar_type() == at::kFloat && m.is_contiguous() && s.is_contiguous() && zt.is_contiguous() &&
                  s.numel() == R && zt.numel() == R,
              "vocab_stats_exchange: contiguous fp32 [R] statistics");
  LIBRA_CHECK(R <= max_rows, "vocab_stats_exchange: %lld rows exceed the buffer's %lld", (long long)R,
              (long long)max_rows);
  LIBRA_CHECK(epoch >= 1, "vocab_stats_exchange: epoch counts calls from 1");
  Peers P{};
  for (int q = 0; q < n; ++q) {
    LIBRA_CHECK((data_ptrs[q] & 15) == 0 && (flag_ptrs[q] & 3) == 0, "vocab_stats_exchange: misaligned buffer");
    P.data[q] = (uint64_t)data_ptrs[q];
    P.flags[q] = (uint64_t)flag_ptrs[q];
  }
  const c10::cuda::CUDAGuard guard(m.device());
  auto lse = torch::empty_like(m);
  auto zo = torch::empty_like(m);
  // the same grid on every rank: it depends only on R, which every rank of the group shares
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(kMaxCtas, (R + kThreads - 1) / kThreads));
  vocab_exchange_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      P, n, (int)me, (int)max_rows, (int)R, m.data_ptr<float>(), s.data_ptr<float>(), zt.data_ptr<float>(),
      lse.data_ptr<float>(), zo.data_ptr<float>(), (int)epoch, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
  return {lse, zo};
}

}  // namespace libra

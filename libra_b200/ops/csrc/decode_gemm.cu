// Skinny GEMM of the rollout decode step:
//
//   acc[M, N] += X[M, K] . W[N, K]^T        (M = decode batch <= 256 rows)
//
// At decode batch sizes the cost of a linear layer is the weight read, so the
// kernel is built around streaming W through every SM at HBM speed:
//
//  * transposed on the tensor cores: D[128 features, Mp] = W_tile . X^T with
//    tcgen05.mma M = 128 (weight rows) and N = Mp (the batch padded to 32, 64,
//    128 or 256), so no MMA row is padding and the accumulator is TMEM lanes =
//    features, columns = batch rows;
//  * stream-K: CTA c of the grid (one per SM) takes the contiguous share
//    [c T / G, (c + 1) T / G) of the T = feature-tiles x K-blocks iterations,
//    so every SM moves the same number of weight bytes however few tiles the
//    layer has (o_proj of Qwen3-4B: 20 tiles of 128 features);
//  * epilogue: lane = feature, so for every batch row the 32 lanes of a warp
//    add 32 consecutive fp32 outputs (one 128-byte line) into acc with
//    reductions at L2 (no read on the epilogue's critical path);
//  * programmatic dependent launch: the producer issues the weight loads of
//    the first pipeline stages before griddepcontrol.wait, so the HBM latency
//    of a layer's first weight tiles overlaps the kernel before it (the fused
//    norm / activation kernels); X and acc are touched only after the wait.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-5 epilogue (warp w reads TMEM lanes 32 (w % 4) ...).  Every
// wait is bounded (common.cuh).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.cuh"

namespace libra {
namespace dgemm {

constexpr int kFeat = 128;  // weight rows per tile = MMA M
constexpr int BK = 64;      // one 128-byte swizzle row of bf16
constexpr int kThreads = 192;

template <int NB>
struct Cfg {
  static constexpr int kStageW = kFeat * BK * 2;
  static constexpr int kStageX = NB * BK * 2;
  static constexpr int kStageBytes = kStageW + kStageX;
  static constexpr int kStages = (196608 / kStageBytes) > 8 ? 8 : (196608 / kStageBytes);
  static constexpr int kTmemCols = 2 * NB;  // double-buffered accumulator (64..512 columns)
  static constexpr int kBarBytes = 8 * (2 * kStages + 5) + 16;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarBytes;
};

// This CTA's contiguous share of the tiles x K-blocks iterations, walked as
// segments (tile, [kb0, kb1)).
struct Share {
  int nkb, it, hi;
  __device__ __forceinline__ Share(int num_tiles, int num_kb) : nkb(num_kb) {
    const long long T = (long long)num_tiles * num_kb;
    it = (int)(T * blockIdx.x / gridDim.x);
    hi = (int)(T * (blockIdx.x + 1) / gridDim.x);
  }
  __device__ __forceinline__ bool next(int& tile, int& kb0, int& kb1) {
    if (it >= hi) return false;
    tile = it / nkb;
    kb0 = it - tile * nkb;
    kb1 = min(nkb, kb0 + (hi - it));
    it += kb1 - kb0;
    return true;
  }
};

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       float* __restrict__ acc, int ldc, int M, int N, int K, int* err) {
  using CF = Cfg<NB>;
  constexpr int S = CF::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + S * CF::kStageW;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * CF::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = (N + kFeat - 1) / kFeat;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, CF::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // weights of the first S iterations do not depend on the previous kernel
      int npre = 0;
      {
        Share sh(num_tiles, num_kb);
        int tile, kb0, kb1;
        while (npre < S && sh.next(tile, kb0, kb1)) {
          for (int kb = kb0; kb < kb1 && npre < S; ++kb, ++npre) {
            mbar_expect_tx(&full[npre], CF::kStageBytes);
            tma_load_2d(sW + npre * CF::kStageW, &tmW, &full[npre], kb * BK, tile * kFeat);
          }
        }
      }
      pdl_wait();
      int stage = 0, i = 0;
      uint32_t phase = 0, issued_mask = 0, issued_phase = 0;
      bool ok = true;
      Share sh(num_tiles, num_kb);
      int tile, kb0, kb1;
      while (ok && sh.next(tile, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++i) {
          if (i >= npre) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, err, kTimeoutSmemEmpty)) { ok = false; break; }
            mbar_expect_tx(&full[stage], CF::kStageBytes);
            tma_load_2d(sW + stage * CF::kStageW, &tmW, &full[stage], kb * BK, tile * kFeat);
          }
          tma_load_2d(sX + stage * CF::kStageX, &tmX, &full[stage], kb * BK, 0);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      // the weight loads of the prologue whose iteration was never reached (none
      // unless a wait gave up) and every other copy must land before exit
      for (int s = 0; s < S; ++s) {
        if (s < npre && !(issued_mask & (1u << s))) mbar_wait(&full[s], 0, nullptr, 0);  // never completes fully
        else if (issued_mask & (1u << s)) mbar_wait(&full[s], (issued_phase >> s) & 1u, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kFeat, NB, 0, 0);
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      Share sh(num_tiles, num_kb);
      int tile, kb0, kb1;
      for (; ok && sh.next(tile, kb0, kb1); ++local) {
        const int a = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[a], aph ^ 1u, err, kTimeoutTmemEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * NB;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kTimeoutTmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_addr = smem_u32(sW + stage * CF::kStageW);
          const uint32_t x_addr = smem_u32(sX + stage * CF::kStageX);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d_tmem, make_sw128_desc(w_addr + k * 32, 16, 1024), make_sw128_desc(x_addr + k * 32, 16, 1024),
                     idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[a]);
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    int local = 0;
    Share sh(num_tiles, num_kb);
    int tile, kb0, kb1;
    for (; sh.next(tile, kb0, kb1); ++local) {
      const int a = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&tfull[a], aph, err, kTimeoutTmemFull)) break;
      tc_fence_after();
      const int f = tile * kFeat + quarter * 32 + lane;
      float* col = acc + f;
#pragma unroll 1
      for (int c = 0; c < NB / 32 && c * 32 < M; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + a * NB + c * 32, r);
        tmem_ld_wait();
        if (f < N) {
          // fire-and-forget reductions for whole and partial tiles alike: a read-add-write would put an
          // L2 round trip per row on the epilogue's critical path
          const int jn = min(32, M - c * 32);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < jn) red_add_f32(col + (size_t)(c * 32 + j) * ldc, __uint_as_float(r[j]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, CF::kTmemCols);
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int NB>
static void launch(const CUtensorMap& tw, const CUtensorMap& tx, float* acc, int ldc, int M, int N, int K, int* err,
                   cudaStream_t st, bool pdl) {
  auto kern = gemm_decode_kernel<NB>;
  constexpr int smem = Cfg<NB>::kSmemBytes;
  static bool configured[kMaxDevices] = {};  // per device: the attribute is set on the current one
  const int cfg_dev = current_device_index();
  if (!configured[cfg_dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    LIBRA_CHECK(e == cudaSuccess, "gemm_decode: cannot reserve %d bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
    configured[cfg_dev] = true;
  }
  const long long units = (long long)((N + kFeat - 1) / kFeat) * ((K + BK - 1) / BK);
  const int grid = units < num_sms() ? (int)units : num_sms();
  launch_kernel(kern, dim3(grid), dim3(kThreads), smem, st, pdl, tw, tx, acc, ldc, M, N, K, err);
}

}  // namespace dgemm

// acc [M, N] fp32 (row stride ldc, inner stride 1) += x [M, K] . w [N, K]^T, bf16 K-major operands,
// 1 <= M <= 256.  pdl: launch with programmatic dependent launch (the weight loads of the first
// pipeline stages start before the previous kernel on the stream has finished).
void gemm_decode(torch::Tensor x, torch::Tensor w, torch::Tensor acc, torch::Tensor err, bool pdl) {
  using namespace dgemm;
  LIBRA_CHECK(x.is_cuda() && w.is_cuda() && acc.is_cuda() && x.scalar_type() == at::kBFloat16 &&
                  w.scalar_type() == at::kBFloat16 && acc.scalar_type() == at::kFloat,
              "gemm_decode: bf16 x / w and fp32 acc on the GPU");
  LIBRA_CHECK(x.dim() == 2 && w.dim() == 2 && acc.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 &&
                  acc.stride(1) == 1,
              "gemm_decode: 2-D operands with unit inner stride");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  LIBRA_CHECK(w.size(1) == K && acc.size(0) == M && acc.size(1) == N, "gemm_decode: shape mismatch");
  LIBRA_CHECK(M >= 1 && M <= 256, "gemm_decode: 1 <= M <= 256 rows, got %lld", (long long)M);
  LIBRA_CHECK(x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0,
              "gemm_decode: 16-byte aligned operands with leading dimensions that are multiples of 8");
  LIBRA_CHECK(K >= 1 && N >= 1, "gemm_decode: empty operand");
  LIBRA_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "gemm_decode: int32 error word");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int NB = M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  const CUtensorMap tw = tmap::make_2d(w.data_ptr(), K, N, w.stride(0), BK, kFeat);
  const CUtensorMap tx = tmap::make_2d(x.data_ptr(), K, M, x.stride(0), BK, NB);
  float* accp = acc.data_ptr<float>();
  const int ldc = (int)acc.stride(0);
  int* errp = err.data_ptr<int>();
  switch (NB) {
    case 32: launch<32>(tw, tx, accp, ldc, (int)M, (int)N, (int)K, errp, st, pdl); break;
    case 64: launch<64>(tw, tx, accp, ldc, (int)M, (int)N, (int)K, errp, st, pdl); break;
    case 128: launch<128>(tw, tx, accp, ldc, (int)M, (int)N, (int)K, errp, st, pdl); break;
    default: launch<256>(tw, tx, accp, ldc, (int)M, (int)N, (int)K, errp, st, pdl); break;
  }
}

}  // namespace libra

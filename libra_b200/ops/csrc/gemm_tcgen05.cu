// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   C[M, N] (op)= sum_k A(m, k) * B(n, k)
//
// A is given either K-major ([M, K] row-major) or MN-major ([K, M] row-major),
// and likewise B ([N, K] or [K, N]).  That covers the three GEMMs of a linear
// layer without transposing anything in memory:
//   forward  Y  = X  W^T : A = X  (K-major), B = W (K-major)
//   dgrad    dX = dY W   : A = dY (K-major), B = W (MN-major)
//   wgrad    dW = dY^T X : A = dY (MN-major), B = X (MN-major)
// which replace the cuBLAS calls the reference reaches through Megatron-Core /
// F.linear (engine/megatron_core_train_engine.py:887-903, engine/qwen3d_modules.py:149).
//
// Structure (one CTA per SM, 192 threads):
//   warp 0  TMA producer: 128B-swizzled tiles of A and B into an S-stage smem ring
//   warp 1  TMEM owner + single-thread tcgen05.mma issuer (M=128, N=BN, K=16 per
//           instruction); commits free smem stages and publish finished tiles
//   warps 2-5 epilogue: tcgen05.ld the fp32 accumulator (4 warps x 32 TMEM lanes),
//           convert and store; TMEM is double-buffered (2 x BN columns) so the
//           epilogue of tile i overlaps the main loop of tile i+1.
// Every wait is bounded (common.cuh); on a timeout the kernel records an error
// code, drains its own outstanding TMA copies and MMAs, frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace libra {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kThreads = 192;
// The peer modes of the pair kernel add four warps (6-9) that sleep through
// the GEMM and join the reduce / copy phases and the all-gather copy, which
// are bound by the number of loads in flight.
constexpr int kPeerThreads = 320;

enum Epilogue : int {
  kStoreBf16 = 0,
  kStoreF32 = 1,
  kAccumF32 = 2,
  kStoreBf16AddResidual = 3,
  kSwiGLU = 4
};

// kSwiGLU (fused gate/up projection + SwiGLU): B is the [2F, K] gate_up
// weight; the B tile of output block nb stacks gate rows [128 nb, 128 nb + 128)
// on top of up rows [F + 128 nb, ...), so TMEM columns [0,128) hold the gate
// and [128,256) the up projection of the same 128 features.  The epilogue
// writes a = silu(gate) * up into C ([M, F]) and, when C2 is given, the
// pre-activation gate/up values into C2 ([M, 2F]) for the backward pass.
// fast reciprocal-based division (MUFU) instead of the IEEE divide: the
// result is rounded to bf16 anyway
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

template <int BN>
struct Cfg {
  static constexpr int kStageA = BM * BK * 2;
  static constexpr int kStageB = BN * BK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (196608 / kStageBytes) > 8 ? 8 : (196608 / kStageBytes);
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  static constexpr int kBarBytes = 8 * (2 * kStages + 4 + 1) + 16;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + kBarBytes;
};

// Grouped rasterisation: consecutive tiles (which run concurrently on the
// persistent CTAs) cover kGroupM M-blocks x a few N-blocks, so both operand
// panels of a wave stay in L2 instead of re-streaming the larger operand.
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int in = tile - group * per_group;
  mb = first_m + in % gm;
  nb = in / gm;
}

// Epilogue of one output tile: this thread's accumulator row (TMEM lane
// quarter*32+lane, columns from tacc) to row `row` of C, columns of block nb.
// With `atomic` (split-K partial tiles of the accumulate epilogue) the fp32
// additions into C are reductions at L2, so the splits of a tile may overlap.
template <int BN, int EPI>
__device__ __forceinline__ void store_tile_row(uint32_t tacc, int row, int nb, int M, int N, void* __restrict__ C,
                                               const __nv_bfloat16* __restrict__ R, int ldc, int ldr,
                                               __nv_bfloat16* __restrict__ C2, int ldc2, bool atomic = false) {
  const bool row_ok = row < M;
  if constexpr (EPI == kSwiGLU) {
#pragma unroll 1
    for (int chunk = 0; chunk < 4; ++chunk) {
      uint32_t g[32], u[32];
      const uint32_t t0 = tacc + chunk * 32;
      tmem_ld_32x32b_x32(t0, g);
      tmem_ld_32x32b_x32(t0 + 128, u);
      tmem_ld_wait();
      const int col0 = nb * 128 + chunk * 32;
      if (!row_ok || col0 >= N) continue;
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc + col0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // round gate/up to bf16 first so the result equals the unfused gate_up -> swiglu path
          const float gv = __bfloat162float(__float2bfloat16(__uint_as_float(g[j * 8 + e])));
          const float uv = __bfloat162float(__float2bfloat16(__uint_as_float(u[j * 8 + e])));
          a[e] = silu_f(gv) * uv;
        }
        uint4 pk;
        pk.x = pack_bf16x2(a[0], a[1]);
        pk.y = pack_bf16x2(a[2], a[3]);
        pk.z = pack_bf16x2(a[4], a[5]);
        pk.w = pack_bf16x2(a[6], a[7]);
        *reinterpret_cast<uint4*>(out + j * 8) = pk;
        if (C2 != nullptr) {
          uint4 pg, pu;
          pg.x = pack_bf16x2(__uint_as_float(g[j * 8 + 0]), __uint_as_float(g[j * 8 + 1]));
          pg.y = pack_bf16x2(__uint_as_float(g[j * 8 + 2]), __uint_as_float(g[j * 8 + 3]));
          pg.z = pack_bf16x2(__uint_as_float(g[j * 8 + 4]), __uint_as_float(g[j * 8 + 5]));
          pg.w = pack_bf16x2(__uint_as_float(g[j * 8 + 6]), __uint_as_float(g[j * 8 + 7]));
          pu.x = pack_bf16x2(__uint_as_float(u[j * 8 + 0]), __uint_as_float(u[j * 8 + 1]));
          pu.y = pack_bf16x2(__uint_as_float(u[j * 8 + 2]), __uint_as_float(u[j * 8 + 3]));
          pu.z = pack_bf16x2(__uint_as_float(u[j * 8 + 4]), __uint_as_float(u[j * 8 + 5]));
          pu.w = pack_bf16x2(__uint_as_float(u[j * 8 + 6]), __uint_as_float(u[j * 8 + 7]));
          __nv_bfloat16* gr = C2 + (size_t)row * ldc2 + col0 + j * 8;
          *reinterpret_cast<uint4*>(gr) = pg;
          *reinterpret_cast<uint4*>(gr + N) = pu;
        }
      }
    }
  } else {
#pragma unroll 1
    for (int chunk = 0; chunk < BN / 32; ++chunk) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tacc + chunk * 32, r);
      tmem_ld_wait();
      const int col0 = nb * BN + chunk * 32;
      if (!row_ok || col0 >= N) continue;
      if (EPI == kStoreBf16 || EPI == kStoreBf16AddResidual) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(C) + (size_t)row * ldc + col0;
        const __nv_bfloat16* res = (EPI == kStoreBf16AddResidual) ? R + (size_t)row * ldr + col0 : nullptr;
        uint4 rvs[4];
        if (EPI == kStoreBf16AddResidual) {  // the chunk's residual loads in flight together
#pragma unroll
          for (int j = 0; j < 4; ++j)
            rvs[j] = col0 + j * 8 < N ? __ldg(reinterpret_cast<const uint4*>(res + j * 8)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (col0 + j * 8 >= N) break;
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[j * 8 + e]);
          if (EPI == kStoreBf16AddResidual) {
            const uint4 rv = rvs[j];
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] += __bfloat162float(rb[e]);
          }
          uint4 pk;
          pk.x = pack_bf16x2(v[0], v[1]);
          pk.y = pack_bf16x2(v[2], v[3]);
          pk.z = pack_bf16x2(v[4], v[5]);
          pk.w = pack_bf16x2(v[6], v[7]);
          *reinterpret_cast<uint4*>(out + j * 8) = pk;
        }
      } else {
        float* out = reinterpret_cast<float*>(C) + (size_t)row * ldc + col0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (col0 + j * 4 >= N) break;
          float4 v = make_float4(__uint_as_float(r[j * 4]), __uint_as_float(r[j * 4 + 1]),
                                 __uint_as_float(r[j * 4 + 2]), __uint_as_float(r[j * 4 + 3]));
          if (EPI == kAccumF32) {
            if (atomic) {
              red_add_f32x4(out + j * 4, v);
              continue;
            }
            float4 o = *reinterpret_cast<const float4*>(out + j * 4);
            v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
          }
          *reinterpret_cast<float4*>(out + j * 4) = v;
        }
      }
    }
  }
}

// Work of one CTA of the single-CTA kernel, as segments (tile, [kb0, kb1)):
//  * streamk == 0: whole tiles blockIdx.x, blockIdx.x + gridDim.x, ...
//  * streamk != 0 (accumulate epilogue): the contiguous share
//    [c * T / G, (c + 1) * T / G) of the T = tiles x K-blocks iterations,
//    walked tile by tile.  Skinny GEMMs (a decode step's M <= 128 rows) have
//    too few output tiles to keep every SM streaming the weight; this way all
//    G CTAs move the same number of K blocks whatever the tile count.
struct Work {
  int nkb, step, it, hi;
  bool sk;
  __device__ __forceinline__ Work(int num_tiles, int num_kb, int streamk) : nkb(num_kb), sk(streamk != 0) {
    if (sk) {
      const long long T = (long long)num_tiles * num_kb;
      it = (int)(T * blockIdx.x / gridDim.x);
      hi = (int)(T * (blockIdx.x + 1) / gridDim.x);
      step = 0;
    } else {
      it = blockIdx.x;
      hi = num_tiles;
      step = gridDim.x;
    }
  }
  __device__ __forceinline__ bool next(int& tile, int& kb0, int& kb1) {
    if (it >= hi) return false;
    if (!sk) {
      tile = it;
      kb0 = 0;
      kb1 = nkb;
      it += step;
      return true;
    }
    tile = it / nkb;
    kb0 = it - tile * nkb;
    kb1 = min(nkb, kb0 + (hi - it));
    it += kb1 - kb0;
    return true;
  }
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* __restrict__ C,
                     const __nv_bfloat16* __restrict__ R, int M, int N, int K, int ldc, int ldr, int* err,
                     __nv_bfloat16* __restrict__ C2, int ldc2, int streamk = 0) {
  static_assert(EPI != kSwiGLU || (BN == 256 && !B_MN), "SwiGLU epilogue: BN 256, K-major weight");
  // output columns per tile: BN, or 128 features for SwiGLU (N is then F)
  constexpr int kTileN = EPI == kSwiGLU ? 128 : BN;
  using CF = Cfg<BN>;
  constexpr int S = CF::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * CF::kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * CF::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* done = tempty + 2;   // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + kTileN - 1) / kTileN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);  // one arrive per epilogue warp
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, CF::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;  // per stage: ever issued / parity of last issue
      bool ok = true;
      Work wk(num_tiles, num_kb, streamk);
      int tile, kb0, kb1;
      while (ok && wk.next(tile, kb0, kb1)) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, kTimeoutSmemEmpty)) { ok = false; break; }
          mbar_expect_tx(&full[stage], CF::kStageBytes);
          uint8_t* a_dst = smA + stage * CF::kStageA;
          uint8_t* b_dst = smB + stage * CF::kStageB;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 64 * BK * 2, &tmA, &full[stage], m0 + j * 64, k0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
          }
          if (EPI == kSwiGLU) {  // gate rows then up rows of the same 128 features
            tma_load_2d(b_dst, &tmB, &full[stage], k0, nb * 128);
            tma_load_2d(b_dst + 128 * BK * 2, &tmB, &full[stage], k0, N + nb * 128);
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 64 * BK * 2, &tmB, &full[stage], n0 + j * 64, k0);
          } else {
            tma_load_2d(b_dst, &tmB, &full[stage], k0, n0);
          }
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: every copy this thread started must land before the CTA exits.
      for (int s = 0; s < S; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&full[s], (issued_phase >> s) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      Work wk(num_tiles, num_kb, streamk);
      int tile, kb0, kb1;
      for (; ok && wk.next(tile, kb0, kb1); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kTimeoutTmemEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kTimeoutTmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * CF::kStageA);
          const uint32_t b_addr = smem_u32(smB + stage * CF::kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 16 elements (32 B) inside the swizzle row; SBO = 8 rows x 128 B.
            // MN-major: advance 16 K-rows (2 KB); LBO = one 64-wide MN chunk (64 rows x 128 B).
            const uint64_t adesc = A_MN ? make_sw128_desc(a_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sw128_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      // Make sure no MMA is in flight before TMEM is released.
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    Work wk(num_tiles, num_kb, streamk);
    int tile, kb0, kb1;
    for (; wk.next(tile, kb0, kb1); ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, err, kTimeoutTmemFull)) break;
      tc_fence_after();
      // a tile that this CTA covers over the whole K range is added with plain
      // loads and stores; a partial one (stream-K) with reductions at L2
      store_tile_row<BN, EPI>(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, mb * BM + row_in_tile, nb, M,
                              N, C, R, ldc, ldr, C2, ldc2, kb0 > 0 || kb1 < num_kb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, CF::kTmemCols);
}

// ------------------------------------------------------------------ CTA-pair kernel
// 256 x 256 output tiles on a cluster of two CTAs (cta_group::2).  Each CTA
// TMA-loads its own 128 rows of A and its own 128 rows (N) of B per K block
// into its shared memory, with the completion counted on the leader's "full"
// barrier; the leader issues M=256 x N=256 MMAs that read both CTAs' halves
// and accumulate rows 0-127 into its TMEM and rows 128-255 into the peer's.
// Per SM and K block this moves 32 KB of operands for 2 x 128 x 256 x 64
// FLOPs, half of what the single-CTA 128 x 256 tile needs, so the tensor
// pipe is no longer held back by shared-memory bandwidth.  Commits arrive on
// both CTAs' barriers (tcgen05.commit multicast); the epilogue warps of both
// CTAs release an accumulator on the leader's barrier.  Loads are never
// multicast.  Same bounded waits as the single-CTA kernel; at exit the two
// CTAs wait for each other (bounded) so neither frees TMEM or shared memory
// the other may still use.
namespace pair {
constexpr int BN = 256;
constexpr int kStageA = BM * BK * 2;   // this CTA's 128 rows of A
constexpr int kStageB = 128 * BK * 2;  // this CTA's 128 rows (N) of B
constexpr int kStageBytes = kStageA + kStageB;
constexpr int kStages = 6;
constexpr int kTmemCols = 2 * BN;
// full[S] empty[S] tfull[2] tempty[2] done exitb
constexpr int kBarBytes = 8 * (2 * kStages + 4 + 2) + 16;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarBytes;
}  // namespace pair

// Tensor-parallel all-reduce fused into the GEMM (kPeerAR): every rank of the
// group computes its partial Y_r = A_r B_r^T; the output is sum_r Y_r (plus an
// optional residual) on every rank.  Over NVLink peer memory, in one launch:
//   A  GEMM tiles; the epilogue stores each 256-row block's bf16 partial in
//      this rank's own partial buffer and bumps the arrival counter of the
//      block's owner (rank mb % n) on that rank (release).  (Pushing the tile
//      rows to the owner instead means one 16-byte NVLink store per row and
//      lane, measured several times slower than the owner pulling whole rows.)
//   B  each CTA takes (owned row block, 256-column chunk) units: waits until
//      all n * num_n * 8 epilogue warps have arrived, reads the n partials
//      (peers' over NVLink, 512 contiguous bytes per warp load), sums them in
//      fp32 and writes the bf16 sum into every rank's gathered buffer, then
//      bumps every rank's "done" counter for the block (reduce-scatter +
//      all-gather, each byte crossing NVLink once per direction).
//   C  each CTA copies finished row blocks of its own gathered buffer (plus
//      the residual) into the output tensor, so the kernel ends only when the
//      full sum is here.  The row blocks this rank owns went to the output
//      directly in phase B.
// Counters live in two parity sets; a call zeroes the set the next call uses
// (safe: no peer can start the next call before this rank's phase B).  Every
// wait is bounded.  Plain loads and stores to peer memory, no multicast.
constexpr int kMaxPeers = 8;
// With rs_rows > 0 the same kernel is a GEMM + reduce-scatter (sequence
// parallel): rank q owns rows [q rs_rows, (q+1) rs_rows) (rs_rows a multiple of
// 256), phase B writes the owned sum (+ residual shard) straight into y
// ([rs_rows, N]) and there is no all-gather; phase C only waits until every
// owner is done reading this rank's partial.
struct PeerAR {
  uint64_t recv[kMaxPeers];   // rank q's partial [max_rows, N] bf16
  uint64_t gath[kMaxPeers];   // rank q's gathered sum: [max_rows, N] bf16
  uint64_t flags[kMaxPeers];  // rank q's counters: int32 [2 parity][2 kind][max_rb]
  __nv_bfloat16* y;           // this rank's output: [M, N], or [rs_rows, N]
  const __nv_bfloat16* residual;  // optional, shaped like y
  int n, me, parity, max_rb, rs_rows;
};

__device__ __forceinline__ int peer_owner(const PeerAR& p, int mb) {
  return p.rs_rows > 0 ? (mb * 2 * BM) / p.rs_rows : mb % p.n;
}

// All-gather fused into the GEMM (sequence-parallel column-parallel linear):
// the A operand's rows are sharded over the group (rank q holds rows
// [q shard_rows, (q+1) shard_rows), shard_rows a multiple of 256).  At kernel
// start the epilogue warps of every CTA copy the peers' shards over NVLink into
// the local gathered buffer (each byte crosses once) and count themselves done
// on a local counter; meanwhile the producer and MMA warps run the tiles of
// the local shard (row blocks rotated so they come first), whose A tiles come
// from the local shard directly.  Tiles of remote rows wait (bounded) for the
// counter before their first TMA load.
// Shards sit in per-rank symmetric slots (two, alternating by call parity);
// rank q publishes "slot ready for call c" in ready[q][parity] at kernel start
// (its host copied the shard in before the launch), and readers wait for it.
// A slot is rewritten two calls later, which no rank reaches before every
// peer has started the call in between, i.e. finished reading this one.
struct PeerAG {
  uint64_t shard[kMaxPeers];  // rank q's A shard slot for this call [shard_rows, K] bf16, mapped here
  uint64_t ready[kMaxPeers];  // rank q's int32 ready[2]
  __nv_bfloat16* gath;        // local [M, K] buffer for the peers' rows
  int* counter;               // local, zero at launch; every epilogue warp adds 1 when its copy is done
  int shard_rows, n, me, parity, call;
};

// kPeer: 0 plain GEMM, 1 GEMM + all-reduce / reduce-scatter (PeerAR),
// 2 all-gather + GEMM (PeerAG).
template <bool A_MN, bool B_MN, int EPI, int kPeer>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPeer ? kPeerThreads : kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     void* __restrict__ C, const __nv_bfloat16* __restrict__ R, int M, int N, int K, int ldc, int ldr,
                     int* err, __nv_bfloat16* __restrict__ C2, int ldc2, int splits, const __grid_constant__ PeerAR par,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ PeerAG ag) {
  using namespace pair;
  constexpr bool kPeerAR = kPeer == 1, kPeerAG = kPeer == 2;
  static_assert(!kPeer || (EPI == kStoreBf16 && !A_MN), "peer modes: K-major A, bf16 output");
  static_assert(EPI != kSwiGLU || !B_MN, "SwiGLU epilogue: K-major weight");
  constexpr int kTileN = EPI == kSwiGLU ? 128 : BN;
  constexpr int S = kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;   // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint64_t* done = tempty + 2;
  uint64_t* exitb = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(exitb + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_n = (N + kTileN - 1) / kTileN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  // Work unit u = split * num_tiles + tile; split s covers K blocks
  // [s * kb_per, min(num_kb, (s + 1) * kb_per)).  splits > 1 only with the
  // accumulate epilogue (the host checks), whose partial tiles add atomically.
  const int num_units = num_tiles * splits;
  const int kb_per = (num_kb + splits - 1) / splits;
  auto unit_range = [&](int u, int& tile, int& kb0, int& kb1) {
    tile = u % num_tiles;
    kb0 = (u / num_tiles) * kb_per;
    kb1 = min(num_kb, kb0 + kb_per);
  };
  // tile -> (row block, column block); with the all-gather the local shard's
  // row blocks come first
  const int rb_rot = kPeerAG ? ag.me * (ag.shard_rows / (2 * BM)) : 0;
  auto coords = [&](int tile, int& mb, int& nb) {
    tile_coords(tile, num_m, num_n, mb, nb);
    if (kPeerAG) mb = (mb + rb_rot) % num_m;
  };

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(done, 1);
    mbar_init(exitb, 1);
    fence_barrier_init();
  }
  if (kPeerAG && blockIdx.x == 0 && threadIdx.x == 0) {  // this rank's shard slot is in place
    __threadfence_system();
    st_release_sys(reinterpret_cast<int*>(ag.ready[ag.me]) + ag.parity, ag.call);
  }
  if (kPeerAR && blockIdx.x == 0) {  // counters of the next call (see PeerAR)
    int* nxt = reinterpret_cast<int*>(par.flags[par.me]) + (par.parity ^ 1) * 2 * par.max_rb;
    for (int i = threadIdx.x; i < 2 * par.max_rb; i += blockDim.x) nxt[i] = 0;
    __threadfence_system();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or copy targets them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, gathered = false;
      for (int u = cluster; u < num_units && ok; u += nclusters) {
        int tile, kb0, kb1, mb, nb;
        unit_range(u, tile, kb0, kb1);
        coords(tile, mb, nb);
        const int m0 = mb * 2 * BM + (int)rank * BM;
        const int n0 = EPI == kSwiGLU ? (rank ? N + nb * 128 : nb * 128) : nb * BN + (int)rank * 128;
        const CUtensorMap* mapA = &tmA;
        int ya = m0;
        if (kPeerAG) {
          const int owner = m0 / ag.shard_rows;
          if (owner == ag.me) {
            ya = m0 - ag.me * ag.shard_rows;  // rows of the local shard
          } else {
            mapA = &tmA2;  // the gathered buffer, indexed by global row
            if (!gathered) {
              if (!wait_flag_geq(ag.counter, 4 * (int)gridDim.x, err, kTimeoutPeerFlag)) { ok = false; break; }
              fence_proxy_async_global();
              gathered = true;
            }
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, kTimeoutSmemEmpty)) { ok = false; break; }
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * kStageBytes);  // both CTAs' bytes
          const uint32_t bar = full_leader + 8u * stage;
          uint8_t* a_dst = smA + stage * kStageA;
          uint8_t* b_dst = smB + stage * kStageB;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * 64 * BK * 2, &tmA, bar, m0 + j * 64, k0);
          } else {
            tma_load_2d_pair(a_dst, mapA, bar, k0, ya);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < 2; ++j) tma_load_2d_pair(b_dst + j * 64 * BK * 2, &tmB, bar, n0 + j * 64, k0);
          } else {
            tma_load_2d_pair(b_dst, &tmB, bar, k0, n0);
          }
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(2 * BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = cluster; u < num_units && ok; u += nclusters, ++local) {
        int tile, kb0, kb1;
        unit_range(u, tile, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kTimeoutTmemEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kTimeoutTmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * kStageA);
          const uint32_t b_addr = smem_u32(smB + stage * kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? make_sw128_desc(a_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sw128_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(b_addr + k * 32, 16, 1024);
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
      }
      umma_commit_pair(done, 0x3);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    int local = 0;
    for (int u = cluster; u < num_units; u += nclusters, ++local) {
      int tile, kb0, kb1, mb, nb;
      unit_range(u, tile, kb0, kb1);
      coords(tile, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, err, kTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      const int row = mb * 2 * BM + (int)rank * BM + row_in_tile;
      if constexpr (kPeerAR) {  // the partial stays here; its owner pulls it
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(par.recv[par.me]);
        store_tile_row<BN, EPI>(tacc, row, nb, M, N, dst, nullptr, N, 0, nullptr, 0);
      } else {
        store_tile_row<BN, EPI>(tacc, row, nb, M, N, C, R, ldc, ldr, C2, ldc2, splits > 1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + 8u * acc);
      if constexpr (kPeerAR) {
        // the warp's partial rows are visible to the owner before the count: the warp barrier orders every
        // lane's stores before lane 0's system-scope fence (cumulative), which precedes the release; one
        // fence per warp instead of one per lane (the per-lane fences were the kernel's top stall)
        __syncwarp();
        if (lane == 0) {
          __threadfence_system();
          red_add_release_sys(reinterpret_cast<int*>(par.flags[peer_owner(par, mb)]) + par.parity * 2 * par.max_rb + mb,
                              1);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ extra warps of the peer modes
    if constexpr (kPeerAG) {  // all-gather of the peers' A shards, 16 bytes per lane and step (warps 6-9)
      const int64_t vrow = K / 8, per_rank = (int64_t)ag.shard_rows * vrow;
      const int64_t total = (int64_t)(ag.n - 1) * per_rank;
      const int64_t gw = (int64_t)blockIdx.x * 4 + (warp - 6), nw = (int64_t)gridDim.x * 4;
      bool ready_ok = true;
      for (int q = 0; q < ag.n && ready_ok; ++q) {
        if (q == ag.me) continue;
        if (lane == 0)
          ready_ok = wait_flag_geq(reinterpret_cast<const int*>(ag.ready[q]) + ag.parity, ag.call, err,
                                   kTimeoutPeerFlag);
        ready_ok = __shfl_sync(0xffffffffu, ready_ok, 0);
      }
      constexpr int kBatch = 8;  // loads in flight per lane
      for (int64_t f0 = gw * 32 + lane; ready_ok && f0 < total; f0 += nw * 32 * kBatch) {
        uint4 v[kBatch];
        int64_t dst[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int64_t f = f0 + (int64_t)u * nw * 32;
          dst[u] = -1;
          if (f < total) {
            const int oi = (int)(f / per_rank);
            const int o = oi < ag.me ? oi : oi + 1;  // skip this rank
            const int64_t rem = f - (int64_t)oi * per_rank;
            v[u] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(ag.shard[o]) + rem * 8);
            dst[u] = ((int64_t)o * ag.shard_rows) * K + rem * 8;
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (dst[u] >= 0) *reinterpret_cast<uint4*>(ag.gath + dst[u]) = v[u];
      }
      fence_proxy_async_global();  // the TMA loads that read these rows go through the async proxy
      __threadfence();
      __syncwarp();
      if (lane == 0 && ready_ok) atomicAdd(ag.counter, 1);
    }
  }

  if constexpr (kPeerAR) {
    __syncthreads();
    __shared__ int s_ok;
    int* my_flags = reinterpret_cast<int*>(par.flags[par.me]) + par.parity * 2 * par.max_rb;
    const int n = par.n, me = par.me;
    const int chunks = (N + BN - 1) / BN;
    const bool rs = par.rs_rows > 0;
    const int rb_per = rs ? par.rs_rows / (2 * BM) : 0;
    const int owned = rs ? rb_per : (me < num_m ? (num_m - me + n - 1) / n : 0);
    const int arrivals = n * num_n * 8;  // epilogue warps of every rank's tiles in a row block
    // ---- B: reduce owned row blocks; the sum goes to every rank (all-reduce)
    // or into this rank's shard of y (reduce-scatter)
    for (int w = blockIdx.x; w < owned * chunks; w += gridDim.x) {
      const int mb = rs ? me * rb_per + w / chunks : me + (w / chunks) * n, ch = w % chunks;
      __syncthreads();  // every thread has read the previous unit's s_ok
      if (threadIdx.x == 0) s_ok = wait_flag_geq(my_flags + mb, arrivals, err, kTimeoutPeerFlag);
      __syncthreads();
      if (!s_ok) break;
      const int r0 = mb * 2 * BM, c0 = ch * BN;
      // kBatch vectors per thread in flight at once: these loops are bound by
      // load latency, not bandwidth, when each thread has one load outstanding
      constexpr int kBatch = 4, kVec = BN / 8;
      for (int v0 = threadIdx.x; v0 < 2 * BM * kVec; v0 += blockDim.x * kBatch) {
        int64_t off[kBatch];
        bool in[kBatch];
        float acc[kBatch][8];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int v = v0 + u * blockDim.x;
          const int row = r0 + v / kVec, col = c0 + (v % kVec) * 8;
          in[u] = v < 2 * BM * kVec && row < M && col < N;
          off[u] = (int64_t)row * N + col;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
        }
        for (int q = 0; q < n; ++q) {  // rank q's partial, over NVLink for q != me (coalesced rows)
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(par.recv[q]);
          uint4 ld[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u)
            ld[u] = in[u] ? *reinterpret_cast<const uint4*>(src + off[u]) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&ld[u]);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[u][e] += __bfloat162float(ub[e]);
          }
        }
        // the owner's own output: written here (with its residual), not gathered
        if (!rs) {
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            if (!in[u]) continue;
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = acc[u][e];
            if (par.residual != nullptr) {
              const uint4 rr = *reinterpret_cast<const uint4*>(par.residual + off[u]);
              const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __bfloat162float(__float2bfloat16(f[e])) + __bfloat162float(rb[e]);
            }
            uint4 o;
            o.x = pack_bf16x2(f[0], f[1]);
            o.y = pack_bf16x2(f[2], f[3]);
            o.z = pack_bf16x2(f[4], f[5]);
            o.w = pack_bf16x2(f[6], f[7]);
            *reinterpret_cast<uint4*>(par.y + off[u]) = o;
          }
        }
        if (rs && par.residual != nullptr) {
          uint4 rr[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u)
            rr[u] = in[u] ? *reinterpret_cast<const uint4*>(par.residual + off[u] - (int64_t)me * par.rs_rows * N)
                          : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rr[u]);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[u][e] += __bfloat162float(rb[e]);
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (!in[u]) continue;
          uint4 o;
          o.x = pack_bf16x2(acc[u][0], acc[u][1]);
          o.y = pack_bf16x2(acc[u][2], acc[u][3]);
          o.z = pack_bf16x2(acc[u][4], acc[u][5]);
          o.w = pack_bf16x2(acc[u][6], acc[u][7]);
          if (rs) {
            *reinterpret_cast<uint4*>(par.y + off[u] - (int64_t)me * par.rs_rows * N) = o;
          } else {
            for (int q = 0; q < n; ++q)
              if (q != me) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(par.gath[q]) + off[u]) = o;
          }
        }
      }
      __syncthreads();  // every thread's sums are stored; the signalling threads fence once for the CTA
      if (threadIdx.x < n) {
        __threadfence_system();
        red_add_release_sys(reinterpret_cast<int*>(par.flags[threadIdx.x]) + par.parity * 2 * par.max_rb +
                                par.max_rb + mb, 1);
      }
    }
    // ---- C: gathered row blocks (+ residual) into the output.  With the
    // reduce-scatter the wait alone remains: no rank may overwrite its partial
    // in the next call before every owner has read it.
    for (int mb = blockIdx.x; mb < num_m; mb += gridDim.x) {
      if (!rs && peer_owner(par, mb) == me) continue;  // written by phase B
      __syncthreads();
      if (threadIdx.x == 0) s_ok = wait_flag_geq(my_flags + par.max_rb + mb, chunks, err, kTimeoutPeerFlag);
      __syncthreads();
      if (!s_ok) break;
      if (rs) continue;
      const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(par.gath[me]);
      const int r0 = mb * 2 * BM, nv = N / 8;
      constexpr int kBatch = 8;
      for (int v0 = threadIdx.x; v0 < 2 * BM * nv; v0 += blockDim.x * kBatch) {
        int64_t off[kBatch];
        bool in[kBatch];
        uint4 o[kBatch], rr[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int v = v0 + u * blockDim.x;
          const int row = r0 + v / nv, col = (v % nv) * 8;
          in[u] = v < 2 * BM * nv && row < M;
          off[u] = (int64_t)row * N + col;
          o[u] = in[u] ? *reinterpret_cast<const uint4*>(g + off[u]) : make_uint4(0, 0, 0, 0);
          if (par.residual != nullptr)
            rr[u] = in[u] ? *reinterpret_cast<const uint4*>(par.residual + off[u]) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (!in[u]) continue;
          if (par.residual != nullptr) {
            const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o[u]);
            const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rr[u]);
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __bfloat162float(ob[e]) + __bfloat162float(rb[e]);
            o[u].x = pack_bf16x2(f[0], f[1]);
            o[u].y = pack_bf16x2(f[2], f[3]);
            o[u].z = pack_bf16x2(f[4], f[5]);
            o[u].w = pack_bf16x2(f[6], f[7]);
          }
          *reinterpret_cast<uint4*>(par.y + off[u]) = o[u];
        }
      }
    }
  }

  // Teardown: once every role of this CTA is through, wait for the last MMA
  // (done), then for the peer to get here too before TMEM is freed and shared
  // memory goes away.
  tc_fence_before();
  __syncthreads();
  if (warp == 1 && lane == 0) mbar_wait(done, 0, err, kTimeoutPairExit);
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(mapa_shared(smem_u32(exitb), rank ^ 1u));
    mbar_wait(exitb, 0, err, kTimeoutPairExit);
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ grouped (expert) GEMM
// The groups are the experts of a MoE layer; their row ranges live in device
// memory (offs[0..G], rows of a padded layout where every group starts at a
// multiple of 128 rows and its padding rows are zero), so the layer never
// reads expert counts back to the host and one launch covers every expert.
//   kGroupRows (forward, dgrad):  C[rows of g] = A[rows of g] . B_g^T, with B_g
//       the g-th [N, K] block of B (K-major) or [K, N] block (MN-major);
//   kGroupK (weight gradient):    C_g [M, N] (op)= sum over rows r of g of
//       A[r, m] B[r, n]  (A, B MN-major, the K loop runs over the group's rows).
// Every role walks the same list of (group, tile) units, found by a binary
// search over the per-group tile prefix kept in shared memory.
constexpr int kGroupRows = 0, kGroupK = 1;
constexpr int kMaxGroups = 256;

template <int BN, bool A_MN, bool B_MN, int EPI, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        void* __restrict__ C, const int* __restrict__ offs, int G, int M, int N, int K, int ldc,
                        int* err, __nv_bfloat16* __restrict__ C2, int ldc2) {
  static_assert(MODE == kGroupK ? (A_MN && B_MN) : !A_MN, "grouped GEMM operand layouts");
  static_assert(EPI != kSwiGLU || (BN == 256 && !B_MN && MODE == kGroupRows), "grouped SwiGLU layout");
  constexpr int kTileN = EPI == kSwiGLU ? 128 : BN;
  using CF = Cfg<BN>;
  constexpr int S = CF::kStages;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_off[kMaxGroups + 1];
  __shared__ int s_tile[kMaxGroups + 1];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * CF::kStageA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * CF::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;  // kGroupK only
  const int num_n = (N + kTileN - 1) / kTileN;
  const int num_kb_rows = (K + BK - 1) / BK;  // kGroupRows only

  for (int g = threadIdx.x; g <= G; g += blockDim.x) s_off[g] = offs[g];
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
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
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < G; ++g) {
      s_tile[g] = acc;
      const int rows = max(0, s_off[g + 1] - s_off[g]);
      acc += MODE == kGroupRows ? ((rows + BM - 1) / BM) * num_n : (rows >= BK ? num_m * num_n : 0);
    }
    s_tile[G] = acc;
  }
  __syncthreads();
  const uint32_t tmem_base = *tmem_slot;
  const int total = s_tile[G];

  // unit -> (group, m block, n block, first row of the group)
  auto locate = [&](int u, int& g, int& mb, int& nb) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {  // last g with s_tile[g] <= u
      const int mid = (lo + hi + 1) >> 1;
      if (s_tile[mid] <= u) lo = mid; else hi = mid - 1;
    }
    g = lo;
    const int t = u - s_tile[g];
    mb = t / num_n;
    nb = t - mb * num_n;
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        int g, mb, nb;
        locate(u, g, mb, nb);
        const int row0 = s_off[g];
        const int kbs = MODE == kGroupRows ? num_kb_rows : (s_off[g + 1] - row0) / BK;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, kTimeoutSmemEmpty)) { ok = false; break; }
          mbar_expect_tx(&full[stage], CF::kStageBytes);
          uint8_t* a_dst = smA + stage * CF::kStageA;
          uint8_t* b_dst = smB + stage * CF::kStageB;
          if (MODE == kGroupRows) {
            const int k0 = kb * BK;
            tma_load_2d(a_dst, &tmA, &full[stage], k0, row0 + mb * BM);
            if (EPI == kSwiGLU) {  // group g's gate rows then its up rows, same 128 features
              tma_load_2d(b_dst, &tmB, &full[stage], k0, g * 2 * N + nb * 128);
              tma_load_2d(b_dst + 128 * BK * 2, &tmB, &full[stage], k0, g * 2 * N + N + nb * 128);
            } else if (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(b_dst + j * 64 * BK * 2, &tmB, &full[stage], nb * BN + j * 64, g * K + k0);
            } else {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, g * N + nb * BN);
            }
          } else {
            const int k0 = row0 + kb * BK;
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(a_dst + j * 64 * BK * 2, &tmA, &full[stage], mb * BM + j * 64, k0);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 64 * BK * 2, &tmB, &full[stage], nb * BN + j * 64, k0);
          }
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      for (int s = 0; s < S; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&full[s], (issued_phase >> s) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++local) {
        int g, mb, nb;
        locate(u, g, mb, nb);
        const int kbs = MODE == kGroupRows ? num_kb_rows : (s_off[g + 1] - s_off[g]) / BK;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kTimeoutTmemEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kbs; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kTimeoutTmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * CF::kStageA);
          const uint32_t b_addr = smem_u32(smB + stage * CF::kStageB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? make_sw128_desc(a_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sw128_desc(b_addr + k * 2048, 64 * BK * 2, 1024)
                                        : make_sw128_desc(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
      int g, mb, nb;
      locate(u, g, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, err, kTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (MODE == kGroupRows) {
        store_tile_row<BN, EPI>(tacc, s_off[g] + mb * BM + row_in_tile, nb, s_off[g + 1], N, C, nullptr, ldc, 0,
                                C2, ldc2);
      } else {
        void* cg = reinterpret_cast<uint8_t*>(C) + (size_t)g * M * ldc * (EPI == kStoreBf16 ? 2 : 4);
        store_tile_row<BN, EPI>(tacc, mb * BM + row_in_tile, nb, M, N, cg, nullptr, ldc, 0, nullptr, 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, CF::kTmemCols);
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with leading
// dimension `ld` (elements), box {box_inner, box_outer}, 128-byte swizzle.
static CUtensorMap make_map(const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer) {
  // The encoder is a driver-API call and needs the device's primary context to
  // be current on this thread.  Threads that have not issued a runtime call yet
  // (autograd's backward worker, for one) do not have it bound: bind it once.
  static thread_local bool context_bound = false;
  if (!context_bound) {
    cudaFree(nullptr);
    context_bound = true;
  }
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LIBRA_CHECK(r == CUDA_SUCCESS, "libra_b200: cuTensorMapEncodeTiled failed with code %d", (int)r);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, void* c, const __nv_bfloat16* r, int M, int N, int K,
                   int ldc, int ldr, int* err, cudaStream_t st, bool streamk = false) {
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, EPI>;
  constexpr int smem = Cfg<BN>::kSmemBytes;
  static bool configured[kMaxDevices] = {};  // per instantiation and device
  if (!configured[current_device_index()]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[current_device_index()] = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  // stream-K: every SM takes a share of the tiles x K-blocks iterations (at least one each)
  const long long units = (EPI == kAccumF32 && streamk) ? (long long)tiles * ((K + BK - 1) / BK) : tiles;
  const int grid = units < num_sms() ? (int)units : num_sms();
  kern<<<grid, kThreads, smem, st>>>(ta, tb, c, r, M, N, K, ldc, ldr, err, nullptr, 0,
                                     (EPI == kAccumF32 && streamk) ? 1 : 0);
  LIBRA_LAUNCH_CHECK();
}

// The CTA-pair kernel takes every GEMM with more than one 128-row block and
// more than 128 output columns; LIBRA_GEMM_PAIR=0 keeps the single-CTA kernel
// (for comparisons).
static bool use_pair(int64_t M, int64_t N) {
  static const bool enabled = [] {
    const char* e = std::getenv("LIBRA_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return enabled && M > BM && N > 128 && num_sms() >= 2;
}

// Clusters of the pair kernel that fit on the device at once (SMs that cannot
// be paired inside a GPC stay out), so the persistent grid has no tail wave
// and the peer all-reduce's intra-grid waits always have their producers
// resident.
template <typename Kern>
static int pair_clusters(Kern kern, int smem, int threads) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / 2;
  }
  return n < num_sms() / 2 ? n : num_sms() / 2;
}

template <bool A_MN, bool B_MN, int EPI, int kPeer = 0>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, void* c, const __nv_bfloat16* r, int M, int N,
                        int K, int ldc, int ldr, int* err, cudaStream_t st, __nv_bfloat16* c2 = nullptr,
                        int ldc2 = 0, const PeerAR* par = nullptr, const CUtensorMap* ta2 = nullptr,
                        const PeerAG* ag = nullptr) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI, kPeer>;
  constexpr int smem = pair::kSmemBytes;
  static int max_clusters_dev[kMaxDevices] = {};  // per instantiation and device
  int& max_clusters = max_clusters_dev[current_device_index()];
  if (!max_clusters) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    max_clusters = pair_clusters(kern, smem, kPeer ? kPeerThreads : kThreads);
  }
  constexpr int kTileN = EPI == kSwiGLU ? 128 : pair::BN;
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + kTileN - 1) / kTileN);
  // Split K (accumulate epilogue only) when the tiles leave the last wave of
  // the persistent grid mostly idle: pick the split count (up to 4, at least
  // 8 K blocks each) whose work units fill the waves best.
  int splits = 1;
  if (EPI == kAccumF32 && tiles < 8 * max_clusters) {
    const int num_kb = (K + BK - 1) / BK;
    double best = 0.0;
    for (int s = 1; s <= 4 && num_kb >= 8 * s; ++s) {
      const int units = tiles * s;
      const int waves = (units + max_clusters - 1) / max_clusters;
      const double fill = (double)units / ((double)waves * max_clusters);
      if (fill > best + 0.02) {
        best = fill;
        splits = s;
      }
    }
  }
  const int units = tiles * splits;
  // the peer phases need every cluster resident (their waits depend on each other)
  const int clusters = kPeer ? max_clusters : (units < max_clusters ? units : max_clusters);
  const PeerAR no_par = {};
  PeerAG no_ag = {};
  kern<<<2 * clusters, kPeer ? kPeerThreads : kThreads, smem, st>>>(ta, tb, c, r, M, N, K, ldc, ldr, err, c2, ldc2, splits,
                                             par ? *par : no_par, ta2 ? *ta2 : ta, ag ? *ag : no_ag);
  LIBRA_LAUNCH_CHECK();
}

template <int EPI>
static void dispatch_pair(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, void* c,
                          const __nv_bfloat16* r, int M, int N, int K, int ldc, int ldr, int* err, cudaStream_t st) {
  if (!a_mn && !b_mn) launch_pair<false, false, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st);
  else if (!a_mn && b_mn) launch_pair<false, true, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st);
  else if (a_mn && b_mn) launch_pair<true, true, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st);
  else launch_pair<true, false, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st);
}

template <int BN, int EPI>
static void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, void* c,
                           const __nv_bfloat16* r, int M, int N, int K, int ldc, int ldr, int* err, cudaStream_t st,
                           bool streamk = false) {
  if (!a_mn && !b_mn) launch<BN, false, false, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st, streamk);
  else if (!a_mn && b_mn) launch<BN, false, true, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st, streamk);
  else if (a_mn && b_mn) launch<BN, true, true, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st, streamk);
  else launch<BN, true, false, EPI>(ta, tb, c, r, M, N, K, ldc, ldr, err, st, streamk);
}

// SwiGLU launch (K-major A, K-major gate_up weight).
static void launch_swiglu(const CUtensorMap& ta, const CUtensorMap& tb, __nv_bfloat16* a_out, int lda_out,
                          __nv_bfloat16* gu_out, int ldgu, int M, int F, int K, int* err, cudaStream_t st) {
  if (use_pair(M, 2 * F)) {
    launch_pair<false, false, kSwiGLU>(ta, tb, a_out, nullptr, M, F, K, lda_out, 0, err, st, gu_out, ldgu);
    return;
  }
  auto kern = gemm_bf16_kernel<256, false, false, kSwiGLU>;
  constexpr int smem = Cfg<256>::kSmemBytes;
  static bool configured[kMaxDevices] = {};  // per device
  if (!configured[current_device_index()]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[current_device_index()] = true;
  }
  const int tiles = ((M + BM - 1) / BM) * (F / 128);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kThreads, smem, st>>>(ta, tb, a_out, nullptr, M, F, K, lda_out, 0, err, gu_out, ldgu, 0);
  LIBRA_LAUNCH_CHECK();
}

}  // namespace gemm

// Fused gate/up projection + SwiGLU: a = silu(x w_gate^T) * (x w_up^T) with
// w = [w_gate; w_up] ([2F, K], K-major), x [M, K].  a: [M, F] bf16.  gu
// (optional, [M, 2F] bf16) receives the pre-activation gate/up outputs.
void gemm_swiglu(torch::Tensor x, torch::Tensor w, torch::Tensor a, c10::optional<torch::Tensor> gu,
                 torch::Tensor err) {
  using namespace gemm;
  LIBRA_CHECK(x.is_cuda() && w.is_cuda() && a.is_cuda() && x.scalar_type() == at::kBFloat16 &&
                  w.scalar_type() == at::kBFloat16 && a.scalar_type() == at::kBFloat16,
              "gemm_swiglu: CUDA bf16 tensors required");
  LIBRA_CHECK(x.dim() == 2 && w.dim() == 2 && a.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 &&
                  a.stride(1) == 1, "gemm_swiglu: 2-D tensors with inner stride 1");
  const int64_t M = x.size(0), K = x.size(1), F2 = w.size(0);
  LIBRA_CHECK(w.size(1) == K && F2 % 256 == 0, "gemm_swiglu: weight [2F, K] with F a multiple of 128");
  const int64_t F = F2 / 2;
  LIBRA_CHECK(a.size(0) == M && a.size(1) == F, "gemm_swiglu: output must be [M, F]");
  LIBRA_CHECK(x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0 && a.stride(0) % 8 == 0 && K >= 1,
              "gemm_swiglu: leading dimensions must be multiples of 8");
  LIBRA_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0,
              "gemm_swiglu: 16-byte aligned base pointers required");
  __nv_bfloat16* gup = nullptr;
  int ldgu = 0;
  if (gu.has_value()) {
    LIBRA_CHECK(gu->scalar_type() == at::kBFloat16 && gu->dim() == 2 && gu->size(0) == M && gu->size(1) == F2 &&
                    gu->stride(1) == 1 && gu->stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(gu->data_ptr()) & 15) == 0,
                "gemm_swiglu: gu must be bf16 [M, 2F] with 16-byte rows");
    gup = reinterpret_cast<__nv_bfloat16*>(gu->data_ptr());
    ldgu = (int)gu->stride(0);
  }
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta = make_map(x.data_ptr(), K, M, x.stride(0), 64, BM);
  CUtensorMap tb = make_map(w.data_ptr(), K, F2, w.stride(0), 64, 128);
  launch_swiglu(ta, tb, reinterpret_cast<__nv_bfloat16*>(a.data_ptr()), (int)a.stride(0), gup, ldgu, (int)M, (int)F,
                (int)K, err.data_ptr<int>(), st);
}

// Tensor-parallel GEMM + all-reduce over peer memory (see PeerAR):
//   y = sum over the group of (a_r b_r^T) (+ residual), on every rank.
//   a: [M, K] bf16 K-major; b: [N, K] (b_mn=false) or [K, N] (b_mn=true);
//   y, residual: [M, N] bf16 contiguous; recv/gath/flags: one device address
//   per rank (this rank's own at index me), all mapped in this context.
void gemm_allreduce(torch::Tensor a, torch::Tensor b, bool b_mn, c10::optional<torch::Tensor> residual, torch::Tensor y,
                    std::vector<int64_t> recv, std::vector<int64_t> gath, std::vector<int64_t> flags, int64_t me,
                    int64_t parity, int64_t max_rows, int64_t rs_rows, torch::Tensor err) {
  using namespace gemm;
  const int n = (int)recv.size();
  LIBRA_CHECK(n >= 1 && n <= kMaxPeers && (int)gath.size() == n && (int)flags.size() == n && me >= 0 && me < n,
              "gemm_allreduce: 1..8 ranks with one address of each buffer per rank");
  LIBRA_CHECK(a.is_cuda() && b.is_cuda() && y.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
              "gemm_allreduce: CUDA bf16 tensors required");
  LIBRA_CHECK(a.dim() == 2 && b.dim() == 2 && y.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && y.is_contiguous(),
              "gemm_allreduce: 2-D operands with inner stride 1 and a contiguous output");
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  LIBRA_CHECK((b_mn ? b.size(0) : b.size(1)) == K && y.size(1) == N && y.size(0) == (rs_rows > 0 ? rs_rows : M),
              "gemm_allreduce: shape mismatch (y is [M, N], or [rs_rows, N] for a reduce-scatter)");
  LIBRA_CHECK(rs_rows == 0 || (rs_rows % (2 * BM) == 0 && rs_rows * n == M),
              "gemm_allreduce: reduce-scatter needs M = n * rs_rows with rs_rows a multiple of 256");
  LIBRA_CHECK(M >= 1 && M <= max_rows && K >= 1 && N % 8 == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0,
              "gemm_allreduce: need 1 <= M <= max_rows, N and leading dimensions multiples of 8");
  const __nv_bfloat16* rp = nullptr;
  if (residual.has_value()) {
    LIBRA_CHECK(residual->scalar_type() == at::kBFloat16 && residual->is_contiguous() &&
                    residual->size(0) == y.size(0) && residual->size(1) == N,
                "gemm_allreduce: residual must be a contiguous bf16 tensor shaped like y");
    rp = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
  }
  for (int q = 0; q < n; ++q)
    LIBRA_CHECK(((recv[q] | gath[q]) & 15) == 0 && (flags[q] & 3) == 0, "gemm_allreduce: misaligned peer buffer");
  PeerAR par = {};
  for (int q = 0; q < n; ++q) {
    par.recv[q] = (uint64_t)recv[q];
    par.gath[q] = (uint64_t)gath[q];
    par.flags[q] = (uint64_t)flags[q];
  }
  par.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  par.residual = rp;
  par.n = n;
  par.me = (int)me;
  par.parity = (int)(parity & 1);
  par.max_rb = (int)((max_rows + 2 * BM - 1) / (2 * BM));
  par.rs_rows = (int)rs_rows;
  const c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta = make_map(a.data_ptr(), K, M, a.stride(0), 64, BM);
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, b.stride(0), 64, 64) : make_map(b.data_ptr(), K, N, b.stride(0), 64, 128);
  int* errp = err.data_ptr<int>();
  if (b_mn)
    launch_pair<false, true, kStoreBf16, 1>(ta, tb, nullptr, nullptr, (int)M, (int)N, (int)K, (int)N, 0, errp, st,
                                            nullptr, 0, &par);
  else
    launch_pair<false, false, kStoreBf16, 1>(ta, tb, nullptr, nullptr, (int)M, (int)N, (int)K, (int)N, 0, errp, st,
                                             nullptr, 0, &par);
}

// All-gather fused into the GEMM (see PeerAG): y = concat_q(a_q) b^T with a_q
// the row shards of the group, y [n * shard_rows, N] on every rank.
//   a: this rank's shard [shard_rows, K] bf16, already copied into its slot;
//   shards: the slot of this call (parity = call & 1) on every rank and
//   ready: every rank's int32 ready[2] (all mapped here); gath: local
//   [n * shard_rows, K] buffer; counter: a local int32 this call resets;
//   call: 1-based call index, the same on every rank.
void gemm_allgather(torch::Tensor a, torch::Tensor b, bool b_mn, torch::Tensor y, std::vector<int64_t> shards,
                    std::vector<int64_t> ready, torch::Tensor gath, torch::Tensor counter, int64_t me, int64_t call,
                    torch::Tensor err) {
  using namespace gemm;
  const int n = (int)shards.size();
  LIBRA_CHECK(n >= 1 && n <= kMaxPeers && (int)ready.size() == n && me >= 0 && me < n && call >= 1,
              "gemm_allgather: 1..8 ranks, one shard slot and one ready pair per rank, call >= 1");
  LIBRA_CHECK(a.is_cuda() && b.is_cuda() && y.is_cuda() && gath.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16 &&
                  gath.scalar_type() == at::kBFloat16 && counter.scalar_type() == at::kInt,
              "gemm_allgather: CUDA bf16 operands and an int32 counter");
  LIBRA_CHECK(a.is_contiguous() && b.dim() == 2 && b.stride(1) == 1 && y.is_contiguous() && gath.is_contiguous(),
              "gemm_allgather: contiguous shard, output and gather buffer");
  const int64_t S = a.size(0), K = a.size(1), M = S * n;
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  LIBRA_CHECK((b_mn ? b.size(0) : b.size(1)) == K && y.size(0) == M && y.size(1) == N && gath.size(0) >= M &&
                  gath.size(1) == K,
              "gemm_allgather: shape mismatch");
  LIBRA_CHECK(S % (2 * BM) == 0 && K % 8 == 0 && N % 8 == 0 && b.stride(0) % 8 == 0,
              "gemm_allgather: shard rows a multiple of 256, K and N multiples of 8");
  for (int q = 0; q < n; ++q) LIBRA_CHECK((shards[q] & 15) == 0, "gemm_allgather: misaligned shard");
  PeerAG ag = {};
  for (int q = 0; q < n; ++q) {
    LIBRA_CHECK((ready[q] & 7) == 0, "gemm_allgather: misaligned ready flags");
    ag.shard[q] = (uint64_t)shards[q];
    ag.ready[q] = (uint64_t)ready[q];
  }
  ag.parity = (int)(call & 1);
  ag.call = (int)call;
  ag.gath = reinterpret_cast<__nv_bfloat16*>(gath.data_ptr());
  ag.counter = counter.data_ptr<int>();
  ag.shard_rows = (int)S;
  ag.n = n;
  ag.me = (int)me;
  const c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  LIBRA_CHECK(cudaMemsetAsync(counter.data_ptr(), 0, sizeof(int), st) == cudaSuccess, "gemm_allgather: memset failed");
  CUtensorMap ta = make_map(a.data_ptr(), K, S, K, 64, BM);
  CUtensorMap tg = make_map(gath.data_ptr(), K, M, K, 64, BM);
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, b.stride(0), 64, 64) : make_map(b.data_ptr(), K, N, b.stride(0), 64, 128);
  void* yp = y.data_ptr();
  int* errp = err.data_ptr<int>();
  if (b_mn)
    launch_pair<false, true, kStoreBf16, 2>(ta, tb, yp, nullptr, (int)M, (int)N, (int)K, (int)N, 0, errp, st, nullptr,
                                            0, nullptr, &tg, &ag);
  else
    launch_pair<false, false, kStoreBf16, 2>(ta, tb, yp, nullptr, (int)M, (int)N, (int)K, (int)N, 0, errp, st, nullptr,
                                             0, nullptr, &tg, &ag);
}

// Python entry: C (op)= A x B^T in the layouts described at the top of the file.
//   a: [M, K] (a_mn=false) or [K, M] (a_mn=true), bf16, inner stride 1
//   b: [N, K] (b_mn=false) or [K, N] (b_mn=true)
//   c: [M, N] bf16 (epi 0/3) or fp32 (epi 1/2)
//   residual: [M, N] bf16 for epi 3 (may be c itself)
void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool a_mn, bool b_mn, int64_t epi,
               c10::optional<torch::Tensor> residual, torch::Tensor err, bool streamk) {
  using namespace gemm;
  LIBRA_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm_bf16: CUDA tensors required");
  LIBRA_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 operands");
  LIBRA_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_bf16: 2-D tensors");
  LIBRA_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm_bf16: inner stride must be 1");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  LIBRA_CHECK(K == Kb, "gemm_bf16: K mismatch %lld vs %lld", (long long)K, (long long)Kb);
  LIBRA_CHECK(c.size(0) == M && c.size(1) == N, "gemm_bf16: output shape mismatch");
  // TMA needs 16-byte strides (leading dims % 8); the epilogue stores 16-byte
  // vectors (N % 8).  K and M may be anything: out-of-range rows/columns of a
  // box are zero-filled and the K loop steps in aligned 64-element blocks.
  LIBRA_CHECK(N % 8 == 0 && (a.stride(0) % 8) == 0 && (b.stride(0) % 8) == 0 && (c.stride(0) % 8) == 0,
              "gemm_bf16: N and every leading dimension must be multiples of 8 (16-byte TMA strides); "
              "got N=%lld lda=%lld ldb=%lld ldc=%lld", (long long)N, (long long)a.stride(0), (long long)b.stride(0),
              (long long)c.stride(0));
  LIBRA_CHECK(a.size(1) >= 1 && b.size(1) >= 1, "gemm_bf16: empty inner dimension");
  LIBRA_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) == 0,
              "gemm_bf16: 16-byte aligned base pointers required");
  const bool f32_out = (epi == kStoreF32 || epi == kAccumF32);
  LIBRA_CHECK(c.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm_bf16: output dtype does not match epilogue");
  const __nv_bfloat16* rptr = nullptr;
  int64_t ldr = 0;
  if (epi == kStoreBf16AddResidual) {
    LIBRA_CHECK(residual.has_value(), "gemm_bf16: residual required");
    LIBRA_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1 && residual->size(0) == M &&
                    residual->size(1) == N && residual->stride(0) % 8 == 0,
                "gemm_bf16: bad residual");
    rptr = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    ldr = residual->stride(0);
  }
  if (M == 0 || N == 0) return;
  if (K == 0) {
    if (epi != kAccumF32) {
      if (epi == kStoreBf16AddResidual) c.copy_(*residual); else c.zero_();
    }
    return;
  }
  static const bool trace = std::getenv("LIBRA_GEMM_TRACE") != nullptr;
  if (trace)
    fprintf(stderr, "[gemm] M=%ld N=%ld K=%ld a_mn=%d b_mn=%d epi=%ld lda=%ld ldb=%ld ldc=%ld a=%p b=%p c=%p\n",
            (long)M, (long)N, (long)K, (int)a_mn, (int)b_mn, (long)epi, (long)a.stride(0), (long)b.stride(0),
            (long)c.stride(0), a.data_ptr(), b.data_ptr(), c.data_ptr());
  const c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (trace) fprintf(stderr, "[gemm] stream=%p\n", (void*)st);
  LIBRA_CHECK(!streamk || epi == kAccumF32, "gemm_bf16: stream-K needs the accumulate epilogue");
  const bool paired = !streamk && use_pair(M, N);
  const int BN = (N <= 128) ? 128 : 256;
  CUtensorMap ta = a_mn ? make_map(a.data_ptr(), M, K, a.stride(0), 64, 64) : make_map(a.data_ptr(), K, M, a.stride(0), 64, BM);
  // a CTA of a pair loads 128 of the tile's 256 B rows
  CUtensorMap tb = b_mn ? make_map(b.data_ptr(), N, K, b.stride(0), 64, 64)
                        : make_map(b.data_ptr(), K, N, b.stride(0), 64, paired ? 128 : BN);
  if (trace) fprintf(stderr, "[gemm] tensor maps encoded\n");
  int* errp = err.data_ptr<int>();
  void* cp = c.data_ptr();
  const int ldc = (int)c.stride(0);
#define LIBRA_GEMM_EPI(E)                                                                                   \
  if (paired) dispatch_pair<E>(a_mn, b_mn, ta, tb, cp, rptr, M, N, K, ldc, (int)ldr, errp, st);          \
  else if (BN == 128) dispatch_major<128, E>(a_mn, b_mn, ta, tb, cp, rptr, M, N, K, ldc, (int)ldr, errp, st, streamk); \
  else dispatch_major<256, E>(a_mn, b_mn, ta, tb, cp, rptr, M, N, K, ldc, (int)ldr, errp, st, streamk);
  switch (epi) {
    case kStoreBf16: LIBRA_GEMM_EPI(kStoreBf16); break;
    case kStoreF32: LIBRA_GEMM_EPI(kStoreF32); break;
    case kAccumF32: LIBRA_GEMM_EPI(kAccumF32); break;
    case kStoreBf16AddResidual: LIBRA_GEMM_EPI(kStoreBf16AddResidual); break;
    default: LIBRA_CHECK(false, "gemm_bf16: unknown epilogue %lld", (long long)epi);
  }
#undef LIBRA_GEMM_EPI
  if (trace) fprintf(stderr, "[gemm] launched\n");
}


// Grouped (per-expert) GEMM with group boundaries in device memory.
//   mode 0 (rows): a [T, K] K-major; b [G, Nb, K] (b_mn false; Nb = N, or 2N for the SwiGLU epilogue whose
//          output has N = Nb / 2 columns) or [G, K, N] (b_mn true); c [T, N] bf16; c2 optional [T, 2N] gate/up
//   mode 1 (k):    a [T, M] and b [T, N] (both MN-major: rows are the reduction); c [G, M, N] fp32,
//          accumulated (epi 2) or stored (epi 1)
// offs [G + 1] int32 on the device: group g owns rows [offs[g], offs[g+1]); every offs[g] must be a
// multiple of 128 and rows past a group's real count must be zero (they take part in the products).
void grouped_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor offs, int64_t mode, bool b_mn,
                  int64_t epi, c10::optional<torch::Tensor> c2, torch::Tensor err) {
  using namespace gemm;
  LIBRA_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda() && offs.is_cuda(), "grouped_gemm: CUDA tensors required");
  LIBRA_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "grouped_gemm: bf16 operands");
  LIBRA_CHECK(a.is_contiguous() && b.is_contiguous() && c.is_contiguous(), "grouped_gemm: contiguous tensors");
  LIBRA_CHECK(offs.scalar_type() == at::kInt && offs.dim() == 1 && offs.numel() >= 2 && offs.numel() <= kMaxGroups + 1,
              "grouped_gemm: offs must be int32 [G + 1] with G <= %d", kMaxGroups);
  LIBRA_CHECK(a.dim() == 2 && b.dim() == 3, "grouped_gemm: a [T, *] and b [G, *, *]");
  const int G = (int)offs.numel() - 1;
  LIBRA_CHECK(b.size(0) == G, "grouped_gemm: b has %lld groups, offs %d", (long long)b.size(0), G);
  const int64_t T = a.size(0);
  const c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  int* errp = err.data_ptr<int>();
  const int* op = offs.data_ptr<int>();
  if (T == 0) return;
  static int sms = 0;
  if (!sms) sms = num_sms();
  if (mode == kGroupRows) {
    const int64_t K = a.size(1);
    const bool swiglu = epi == kSwiGLU;
    const int64_t N = b_mn ? b.size(2) : (swiglu ? b.size(1) / 2 : b.size(1));
    LIBRA_CHECK((b_mn ? b.size(1) : b.size(2)) == K, "grouped_gemm: K mismatch");
    LIBRA_CHECK(K % 64 == 0 && N % 128 == 0, "grouped_gemm: K must be a multiple of 64 and N of 128");
    LIBRA_CHECK(c.scalar_type() == at::kBFloat16 && c.dim() == 2 && c.size(0) == T && c.size(1) == N,
                "grouped_gemm: c must be bf16 [T, N]");
    LIBRA_CHECK(epi == kStoreBf16 || (swiglu && !b_mn), "grouped_gemm: row mode stores bf16 (or SwiGLU)");
    __nv_bfloat16* c2p = nullptr;
    if (c2.has_value()) {
      LIBRA_CHECK(swiglu && c2->scalar_type() == at::kBFloat16 && c2->is_contiguous() && c2->size(0) == T &&
                      c2->size(1) == 2 * N, "grouped_gemm: c2 is the SwiGLU gate/up output [T, 2N]");
      c2p = reinterpret_cast<__nv_bfloat16*>(c2->data_ptr());
    }
    CUtensorMap ta = make_map(a.data_ptr(), K, T, K, 64, BM);
    const int tiles_ub = (int)(((T + BM - 1) / BM) * (N / (swiglu ? 128 : 256)) + 1);
    const int grid = tiles_ub < sms ? tiles_ub : sms;
    constexpr int smem = Cfg<256>::kSmemBytes;
    if (swiglu) {
      CUtensorMap tb = make_map(b.data_ptr(), K, (int64_t)G * 2 * N, K, 64, 128);
      auto kern = grouped_gemm_kernel<256, false, false, kSwiGLU, kGroupRows>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<grid, kThreads, smem, st>>>(ta, tb, c.data_ptr(), op, G, 0, (int)N, (int)K, (int)N, errp, c2p,
                                         (int)(2 * N));
    } else if (b_mn) {
      CUtensorMap tb = make_map(b.data_ptr(), N, (int64_t)G * K, N, 64, 64);
      auto kern = grouped_gemm_kernel<256, false, true, kStoreBf16, kGroupRows>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<grid, kThreads, smem, st>>>(ta, tb, c.data_ptr(), op, G, 0, (int)N, (int)K, (int)N, errp, nullptr, 0);
    } else {
      CUtensorMap tb = make_map(b.data_ptr(), K, (int64_t)G * N, K, 64, 256);
      auto kern = grouped_gemm_kernel<256, false, false, kStoreBf16, kGroupRows>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<grid, kThreads, smem, st>>>(ta, tb, c.data_ptr(), op, G, 0, (int)N, (int)K, (int)N, errp, nullptr, 0);
    }
  } else {
    LIBRA_CHECK(mode == kGroupK && b.dim() == 3, "grouped_gemm: mode must be 0 (rows) or 1 (k)");
    LIBRA_CHECK(false, "grouped_gemm: use grouped_gemm_wgrad for mode 1");
  }
  LIBRA_LAUNCH_CHECK();
}

// Weight gradient of a grouped linear: c [G, M, N] fp32 (+)= per group, dy[rows]^T x[rows]
// with dy [T, M] and x [T, N] bf16 row-major (the rows are the reduction); offs as above, every group's
// row count a multiple of 64 (the padded layout gives 128).
void grouped_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor c, torch::Tensor offs, bool accumulate,
                        torch::Tensor err) {
  using namespace gemm;
  LIBRA_CHECK(dy.is_cuda() && x.is_cuda() && c.is_cuda() && offs.is_cuda(), "grouped_gemm_wgrad: CUDA tensors");
  LIBRA_CHECK(dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kFloat,
              "grouped_gemm_wgrad: bf16 inputs, fp32 output");
  LIBRA_CHECK(dy.is_contiguous() && x.is_contiguous() && c.is_contiguous() && dy.dim() == 2 && x.dim() == 2 &&
                  c.dim() == 3 && dy.size(0) == x.size(0),
              "grouped_gemm_wgrad: dy [T, M], x [T, N], c [G, M, N] contiguous");
  LIBRA_CHECK(offs.scalar_type() == at::kInt && offs.numel() == c.size(0) + 1 && offs.numel() <= kMaxGroups + 1,
              "grouped_gemm_wgrad: offs int32 [G + 1]");
  const int G = (int)c.size(0);
  const int64_t T = dy.size(0), M = dy.size(1), N = x.size(1);
  LIBRA_CHECK(c.size(1) == M && c.size(2) == N, "grouped_gemm_wgrad: c must be [G, M, N]");
  LIBRA_CHECK(M % 64 == 0 && N % 128 == 0, "grouped_gemm_wgrad: M a multiple of 64, N of 128");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(dy.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta = make_map(dy.data_ptr(), M, T, M, 64, 64);
  CUtensorMap tb = make_map(x.data_ptr(), N, T, N, 64, 64);
  static int sms = 0;
  if (!sms) sms = num_sms();
  const int tiles_ub = G * (int)((M + BM - 1) / BM) * (int)((N + 255) / 256);
  const int grid = tiles_ub < sms ? tiles_ub : sms;
  constexpr int smem = Cfg<256>::kSmemBytes;
  if (accumulate) {
    auto kern = grouped_gemm_kernel<256, true, true, kAccumF32, kGroupK>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kern<<<grid, kThreads, smem, st>>>(ta, tb, c.data_ptr(), offs.data_ptr<int>(), G, (int)M, (int)N, 0, (int)N,
                                       err.data_ptr<int>(), nullptr, 0);
  } else {
    auto kern = grouped_gemm_kernel<256, true, true, kStoreF32, kGroupK>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kern<<<grid, kThreads, smem, st>>>(ta, tb, c.data_ptr(), offs.data_ptr<int>(), G, (int)M, (int)N, 0, (int)N,
                                       err.data_ptr<int>(), nullptr, 0);
  }
  LIBRA_LAUNCH_CHECK();
}

}  // namespace libra

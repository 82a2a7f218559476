// Backward pass of the tcgen05 varlen GQA attention (forward: flash_attn.cu).
//
// Three launches, no atomics:
//   delta    one CTA per (q tile, q head): D = rowsum(dO * O) and lse * log2(e)
//            written to per-head padded arrays in which every 128-row q tile of
//            sequence b starts at pad_base(b) + 128 t, a 16-byte aligned
//            offset, so a block's 128 values arrive with one bulk copy.  Rows
//            past the sequence end are written as 0.
//   dkdv     per (kv tile, kv head): loop over the group's q heads and the
//            q tiles at or after the kv tile (causal);
//              S^T  = K Q^T           P^T  = 2^(S^T c - lse2_q)
//              dP^T = V dO^T          dS^T = P^T (dP^T - D_q) * scale
//              dV  += P^T dO          dK  += dS^T Q
//            TMEM: S^T [0,128) dP^T [128,256) dV [256,384) dK [384,512).
//            P^T and dS^T are written back as packed bf16 over the columns of
//            S^T / dP^T they were computed from and read from there as the A
//            operand of the dV / dK MMAs (tcgen05.mma executes in issue order,
//            so S^T of the next block, issued after dV, overwrites P^T only
//            after dV has read it).  Q, dO and the block's lse2 / D share a
//            2-stage ring; blocks are prefetched into L2 two ahead.
//   dq       per (q tile, q head): loop over kv tiles at or before it;
//              S = Q K^T   P s = 2^(S c - lse2 + log2 s)   dP = dO V^T
//              dS = P s (dP - D)      dQ += dS K
//            TMEM: S [0,128) dP [128,256) dQ [256,384) dS [384,448) [448,512).
//            dS (double-buffered, in TMEM) is the A operand of the dQ MMA;
//            S_{j+1} / dP_{j+1} are issued as soon as S_j / dP_j have been read.
//            K_j waits in a 3-stage ring (freed after dQ_j), V_j in a 2-stage
//            ring (freed after dP_j); blocks are prefetched into L2 three ahead.
// where c = scale * log2(e) and lse is the forward's natural-log denominator.
// The thread that owns a TMEM lane owns one row (kv row in dkdv, q row in dq);
// warps w and w+4 share a lane quarter and split the 128 columns in halves.
// Masks are applied only on blocks that cross the causal diagonal or a
// sequence end.  Same warp roles and bounded waits as the forward kernel.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_common.cuh"

namespace libra {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

// Start of sequence b (first token s0) in the padded per-head arrays: 4-float
// aligned, and 132 extra rows per sequence keep every sequence's last 128-row
// window clear of the next sequence.
__host__ __device__ __forceinline__ int pad_base(int s0, int b) { return ((s0 + 3) & ~3) + 132 * b; }
inline int64_t pad_rows(int64_t T, int64_t B) { return ((T + 3) & ~int64_t(3)) + 132 * B + 128; }

// ------------------------------------------------------------------ delta
__global__ void __launch_bounds__(256) attn_delta_kernel(const __nv_bfloat16* __restrict__ O,
                                                         const __nv_bfloat16* __restrict__ dO,
                                                         const float* __restrict__ lse, const int* __restrict__ cu,
                                                         const int2* __restrict__ q_tiles, int Hq, int T, int T_pad,
                                                         float* __restrict__ lse2p, float* __restrict__ dltp) {
  const int2 t = q_tiles[blockIdx.x];
  const int h = blockIdx.y;
  const int s0 = cu[t.x], L = cu[t.x + 1] - s0;
  const int base = pad_base(s0, t.x) + t.y * BQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, l16 = lane & 15;  // 16 lanes x 16 bytes per row, two rows per warp step
#pragma unroll 2
  for (int r = 2 * warp + half; r < BQ; r += 16) {
    const int qp = t.y * BQ + r;
    const bool valid = qp < L;
    float dsum = 0.f;
    if (valid) {
      const size_t w = (size_t)(s0 + qp) * Hq + h;
      const uint4 o = reinterpret_cast<const uint4*>(O + w * D)[l16];
      const uint4 g = reinterpret_cast<const uint4*>(dO + w * D)[l16];
      const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&g);
#pragma unroll
      for (int e = 0; e < 8; ++e) dsum += __bfloat162float(ob[e]) * __bfloat162float(gb[e]);
    }
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, m);  // within the 16-lane half
    if (l16 == 0) {
      dltp[(size_t)h * T_pad + base + r] = dsum;
      lse2p[(size_t)h * T_pad + base + r] = valid ? lse[(size_t)h * T + s0 + qp] * kLog2e : 0.f;
    }
  }
}

// Each row of a 128-column TMEM tile is handled by two warps (same TMEM lane
// quarter, warps w and w+4): `half` selects columns [64*half, 64*half + 64).
constexpr int kSoftmaxWarps = 8;
constexpr int kBwdThreads = 64 + 32 * kSoftmaxWarps;

__device__ __forceinline__ void ld_half64(uint32_t taddr, float (&v)[64]) {
#pragma unroll
  for (int c = 0; c < 2; ++c) tmem_ld_32x32b_x32(taddr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
  tmem_ld_wait();
}

__device__ __forceinline__ void store_acc_half(uint32_t taddr, __nv_bfloat16* dst, bool ok) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t o[32];
    tmem_ld_32x32b_x32(taddr + c * 32, o);
    tmem_ld_wait();
    if (ok) {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 pk;
        pk.x = pack_bf16x2(__uint_as_float(o[q4 * 8 + 0]), __uint_as_float(o[q4 * 8 + 1]));
        pk.y = pack_bf16x2(__uint_as_float(o[q4 * 8 + 2]), __uint_as_float(o[q4 * 8 + 3]));
        pk.z = pack_bf16x2(__uint_as_float(o[q4 * 8 + 4]), __uint_as_float(o[q4 * 8 + 5]));
        pk.w = pack_bf16x2(__uint_as_float(o[q4 * 8 + 6]), __uint_as_float(o[q4 * 8 + 7]));
        *reinterpret_cast<uint4*>(dst + c * 32 + q4 * 8) = pk;
      }
    }
  }
}

// 64 fp32 values of a row -> 32 packed bf16 pairs written to 32 TMEM columns.
__device__ __forceinline__ void store_packed_half(uint32_t taddr, const float (&v)[64]) {
  uint32_t w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  tmem_st_32x32b_x32(taddr, w);
  tmem_st_wait();
}

// TMEM column of K step kk (16 elements) of a 128-wide operand stored as two
// packed 64-element halves at col0 and col0 + 64.
__device__ __forceinline__ uint32_t split_half_col(uint32_t col0, int kk) {
  return col0 + (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
}

// ------------------------------------------------------------------ dq
namespace dqk {
constexpr int kKStages = 3, kVStages = 2, kPrefetch = 3;
constexpr int kOffQ = 0, kOffDO = kTile, kOffK = 2 * kTile, kOffV = kOffK + kKStages * kTile;
constexpr int kOffBar = kOffV + kVStages * kTile;
// q_full q_empty | k_full[3] k_empty[3] | v_full[2] v_empty[2] | s_full s_empty dp_full dp_empty
// | ds_full[2] ds_empty[2] | dq_full dq_empty done
constexpr int kNumBars = 2 + 2 * kKStages + 2 * kVStages + 4 + 4 + 3;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256, kColDS = 384;
}  // namespace dqk

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const int* __restrict__ cu, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv,
                        const float* __restrict__ lse2p, const float* __restrict__ dltp, int T_pad,
                        __nv_bfloat16* __restrict__ dQ, float scale, float scale_log2, int causal, int* err) {
  using namespace dqk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *q_full = bars, *q_empty = bars + 1, *k_full = bars + 2, *k_empty = k_full + kKStages,
           *v_full = k_empty + kKStages, *v_empty = v_full + kVStages, *s_full = v_empty + kVStages,
           *s_empty = s_full + 1, *dp_full = s_full + 2, *dp_empty = s_full + 3, *ds_full = s_full + 4,
           *ds_empty = ds_full + 2, *dq_full = ds_empty + 2, *dq_empty = dq_full + 1, *done = dq_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = n_tiles * Hq, group = Hq / Hkv;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, kSoftmaxWarps);
    mbar_init(dp_full, 1);
    mbar_init(dp_empty, kSoftmaxWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ds_full[b], kSoftmaxWarps);
      mbar_init(&ds_empty[b], 1);
    }
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, kSoftmaxWarps);
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint8_t *smQ = smem + kOffQ, *smDO = smem + kOffDO, *smK = smem + kOffK, *smV = smem + kOffV;

  auto decode = [&](int item, int& b, int& s0, int& L, int& q0, int& h, int& hk, int& nkv) {
    const int2 t = tiles[item / Hq];
    b = t.x;
    h = item % Hq;
    hk = h / group;
    s0 = cu[t.x];
    L = cu[t.x + 1] - s0;
    q0 = t.y * BQ;
    const int nall = (L + BKV - 1) / BKV;
    nkv = causal ? min(t.y + 1, nall) : nall;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0, item_it = 0, q_par = 0;  // g: K/V blocks loaded by this CTA
      bool ok = true, q_issued = false;
      uint32_t k_mask = 0, k_par = 0, v_mask = 0, v_par = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int b, s0, L, q0, h, hk, nkv;
        decode(item, b, s0, L, q0, h, hk, nkv);
        if (!mbar_wait(q_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        mbar_expect_tx(q_full, 2 * kTile);
        tma_load_2d(smQ, &tmQ, q_full, h * D, s0 + q0);
        tma_load_2d(smQ + kChunk, &tmQ, q_full, h * D + 64, s0 + q0);
        tma_load_2d(smDO, &tmDO, q_full, h * D, s0 + q0);
        tma_load_2d(smDO + kChunk, &tmDO, q_full, h * D + 64, s0 + q0);
        q_issued = true;
        q_par = item_it & 1u;
        auto prefetch = [&](int j) {
          const int y = s0 + j * BKV;
          tma_prefetch_l2_2d(&tmK, hk * D, y);
          tma_prefetch_l2_2d(&tmK, hk * D + 64, y);
          tma_prefetch_l2_2d(&tmV, hk * D, y);
          tma_prefetch_l2_2d(&tmV, hk * D + 64, y);
        };
        for (int j = 0; j < nkv && j < kPrefetch; ++j) prefetch(j);
        for (int j = 0; j < nkv; ++j, ++g) {
          if (j + kPrefetch < nkv) prefetch(j + kPrefetch);
          const int y = s0 + j * BKV;
          const int ks = g % kKStages, vs = g % kVStages;
          const uint32_t kph = (g / kKStages) & 1u, vph = (g / kVStages) & 1u;
          if (!mbar_wait(&k_empty[ks], kph ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          mbar_expect_tx(&k_full[ks], kTile);
          tma_load_2d(smK + ks * kTile, &tmK, &k_full[ks], hk * D, y);
          tma_load_2d(smK + ks * kTile + kChunk, &tmK, &k_full[ks], hk * D + 64, y);
          k_mask |= 1u << ks;
          k_par = (k_par & ~(1u << ks)) | (kph << ks);
          if (!mbar_wait(&v_empty[vs], vph ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          mbar_expect_tx(&v_full[vs], kTile);
          tma_load_2d(smV + vs * kTile, &tmV, &v_full[vs], hk * D, y);
          tma_load_2d(smV + vs * kTile + kChunk, &tmV, &v_full[vs], hk * D + 64, y);
          v_mask |= 1u << vs;
          v_par = (v_par & ~(1u << vs)) | (vph << vs);
        }
      }
      if (q_issued) mbar_wait(q_full, q_par, nullptr, 0);
      for (int s = 0; s < kKStages; ++s)
        if ((k_mask >> s) & 1u) mbar_wait(&k_full[s], (k_par >> s) & 1u, nullptr, 0);
      for (int s = 0; s < kVStages; ++s)
        if ((v_mask >> s) & 1u) mbar_wait(&v_full[s], (v_par >> s) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_kk = make_idesc_bf16(BQ, BKV, 0, 0);  // S, dP
      constexpr uint32_t idesc_dq = make_idesc_bf16(BQ, D, 0, 1);    // dQ = dS K (K read MN-major)
      const uint32_t aQ = smem_u32(smQ), aDO = smem_u32(smDO);
      uint32_t g = 0, item_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int b, s0, L, q0, h, hk, nkv;
        decode(item, b, s0, L, q0, h, hk, nkv);
        if (!mbar_wait(q_full, item_it & 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        tc_fence_after();
        // Per block j: S_{j+1} as soon as the softmax warps have read S_j,
        // dP_{j+1} as soon as they have read dP_j, then dQ_j once dS_j is in
        // TMEM, so the tensor core works on the next block while dS_j is built.
        const uint32_t g0 = g;
        auto issue_s = [&](uint32_t gj) -> bool {
          const int ks = gj % kKStages;
          if (!mbar_wait(&k_full[ks], (gj / kKStages) & 1u, err, kTimeoutAttnKV)) return false;
          if (!mbar_wait(s_empty, (gj & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aK = smem_u32(smK + ks * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColS, kmajor_desc(aQ, kk), kmajor_desc(aK, kk), idesc_kk, kk > 0);
          umma_commit(s_full);
          return true;
        };
        auto issue_dp = [&](uint32_t gj, bool last) -> bool {
          const int vs = gj % kVStages;
          if (!mbar_wait(&v_full[vs], (gj / kVStages) & 1u, err, kTimeoutAttnKV)) return false;
          if (!mbar_wait(dp_empty, (gj & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aV = smem_u32(smV + vs * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColDP, kmajor_desc(aDO, kk), kmajor_desc(aV, kk), idesc_kk, kk > 0);
          umma_commit(dp_full);
          umma_commit(&v_empty[vs]);
          if (last) umma_commit(q_empty);  // Q and dO are no longer read
          return true;
        };
        if (!issue_s(g0) || !issue_dp(g0, nkv == 1)) { ok = false; break; }
        for (int j = 0; j < nkv; ++j, ++g) {
          const int ks = g % kKStages, db = g & 1;
          if (j + 1 < nkv && !issue_s(g + 1)) { ok = false; break; }
          if (j + 1 < nkv && !issue_dp(g + 1, j + 2 == nkv)) { ok = false; break; }
          if (!mbar_wait(&ds_full[db], (g >> 1) & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (j == 0 && !mbar_wait(dq_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aK = smem_u32(smK + ks * kTile);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16_ts(tmem_base + kColDQ, tmem_base + kColDS + db * 64 + kk * 8, mnmajor_desc(aK, kk), idesc_dq,
                        (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&k_empty[ks]);
          umma_commit(&ds_empty[db]);
        }
        if (!ok) break;
        umma_commit(dq_full);
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, half = (warp - 2) >> 2;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;  // this thread's 64 columns of the row
    const float log2_scale = log2f(scale);
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
    };
    uint32_t g = 0, item_it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
      int b, s0, L, q0, h, hk, nkv;
      decode(item, b, s0, L, q0, h, hk, nkv);
      const int qp = q0 + row;
      const bool row_ok = qp < L;
      const size_t prow = (size_t)h * T_pad + pad_base(s0, b) + qp;  // rows past L hold 0
      const float lse2 = lse2p[prow] - log2_scale;  // folds the softmax scale into P
      const float dlt = dltp[prow];
      const int lim = causal ? min(qp + 1, L) : L;
      const int lim_tile = causal ? min(q0 + 1, L) : L;
      for (int j = 0; j < nkv; ++j, ++g) {
        float v[64];
        if (!wait_all(s_full, g & 1u, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        ld_half64(tmem_base + lane_addr + kColS + c0, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);
#pragma unroll
        for (int c = 0; c < 64; ++c) v[c] = ex2_approx(fmaf(v[c], scale_log2, -lse2));
        const int kb = j * BKV + c0;
        if ((j + 1) * BKV > lim_tile) {
#pragma unroll
          for (int c = 0; c < 64; ++c) v[c] = (kb + c < lim) ? v[c] : 0.f;
        }
        if (!wait_all(dp_full, g & 1u, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t d[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + kColDP + c0 + c * 32, d);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[c * 32 + e] *= __uint_as_float(d[e]) - dlt;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dp_empty);
        const int db = g & 1;
        if (g >= 2 && !wait_all(&ds_empty[db], ((g >> 1) & 1u) ^ 1u, kTimeoutAttnPV)) { ok = false; break; }
        tc_fence_after();
        store_packed_half(tmem_base + lane_addr + kColDS + db * 64 + half * 32, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ds_full[db]);
      }
      if (!ok) break;
      if (!wait_all(dq_full, item_it & 1u, kTimeoutAttnO)) break;
      tc_fence_after();
      store_acc_half(tmem_base + lane_addr + kColDQ + c0, dQ + ((size_t)(s0 + qp) * Hq + h) * D + c0, row_ok);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ dk, dv
namespace dkv {
constexpr int kStages = 2, kPrefetch = 2;
constexpr int kStageBytes = 2 * kTile + 1024;  // Q | dO | lse2[128] | delta[128]
constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile;
constexpr int kOffBar = kOffQ + kStages * kStageBytes;
// kv_full kv_empty | qd_full[2] qd_empty[2] | st_full dpt_full p_full ds_full | acc_full acc_empty done
constexpr int kNumBars = 2 + 2 * kStages + 4 + 3;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;
}  // namespace dkv

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                          const int* __restrict__ cu, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv,
                          const float* __restrict__ lse2p, const float* __restrict__ dltp, int T_pad,
                          __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV, float scale,
                          float scale_log2, int causal, int* err) {
  using namespace dkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *kv_full = bars, *kv_empty = bars + 1, *qd_full = bars + 2, *qd_empty = qd_full + kStages,
           *b0 = qd_empty + kStages;
  uint64_t *st_full = b0, *dpt_full = b0 + 1, *p_full = b0 + 2, *ds_full = b0 + 3, *acc_full = b0 + 4,
           *acc_empty = b0 + 5, *done = b0 + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = Hq / Hkv, n_items = n_tiles * Hkv;
  if (threadIdx.x == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(dpt_full, 1);
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(ds_full, kSoftmaxWarps);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kSoftmaxWarps);
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint8_t *smK = smem + kOffK, *smV = smem + kOffV, *smQD = smem + kOffQ;

  // item = (kv tile, kv head); blocks = group q heads x q tiles [jt, nq)
  auto decode = [&](int item, int& b, int& s0, int& L, int& jt, int& hk, int& nq, int& nblk) {
    const int2 t = tiles[item / Hkv];
    b = t.x;
    hk = item % Hkv;
    s0 = cu[t.x];
    L = cu[t.x + 1] - s0;
    jt = t.y;
    nq = (L + BQ - 1) / BQ;
    nblk = group * (causal ? nq - jt : nq);
  };
  auto block_q = [&](int blk, int jt, int nq, int hk, int& h, int& qi) {
    const int per = causal ? nq - jt : nq;
    h = hk * group + blk / per;
    qi = (causal ? jt : 0) + blk % per;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0, item_it = 0, kv_par = 0;  // g: q blocks loaded by this CTA
      bool ok = true, kv_issued = false;
      uint32_t mask = 0, par = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int b, s0, L, jt, hk, nq, nblk;
        decode(item, b, s0, L, jt, hk, nq, nblk);
        if (!mbar_wait(kv_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
        mbar_expect_tx(kv_full, 2 * kTile);
        tma_load_2d(smK, &tmK, kv_full, hk * D, s0 + jt * BKV);
        tma_load_2d(smK + kChunk, &tmK, kv_full, hk * D + 64, s0 + jt * BKV);
        tma_load_2d(smV, &tmV, kv_full, hk * D, s0 + jt * BKV);
        tma_load_2d(smV + kChunk, &tmV, kv_full, hk * D + 64, s0 + jt * BKV);
        kv_issued = true;
        kv_par = item_it & 1u;
        const int pbase = pad_base(s0, b);
        auto prefetch = [&](int blk) {
          int h, qi;
          block_q(blk, jt, nq, hk, h, qi);
          tma_prefetch_l2_2d(&tmQ, h * D, s0 + qi * BQ);
          tma_prefetch_l2_2d(&tmQ, h * D + 64, s0 + qi * BQ);
          tma_prefetch_l2_2d(&tmDO, h * D, s0 + qi * BQ);
          tma_prefetch_l2_2d(&tmDO, h * D + 64, s0 + qi * BQ);
        };
        for (int blk = 0; blk < nblk && blk < kPrefetch; ++blk) prefetch(blk);
        for (int blk = 0; blk < nblk; ++blk, ++g) {
          if (blk + kPrefetch < nblk) prefetch(blk + kPrefetch);
          int h, qi;
          block_q(blk, jt, nq, hk, h, qi);
          const int st = g % kStages;
          const uint32_t ph = (g / kStages) & 1u;
          if (!mbar_wait(&qd_empty[st], ph ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
          uint8_t* q = smQD + st * kStageBytes;
          mbar_expect_tx(&qd_full[st], 2 * kTile + 1024);
          tma_load_2d(q, &tmQ, &qd_full[st], h * D, s0 + qi * BQ);
          tma_load_2d(q + kChunk, &tmQ, &qd_full[st], h * D + 64, s0 + qi * BQ);
          tma_load_2d(q + kTile, &tmDO, &qd_full[st], h * D, s0 + qi * BQ);
          tma_load_2d(q + kTile + kChunk, &tmDO, &qd_full[st], h * D + 64, s0 + qi * BQ);
          const size_t prow = (size_t)h * T_pad + pbase + qi * BQ;
          bulk_load(q + 2 * kTile, lse2p + prow, 512, &qd_full[st]);
          bulk_load(q + 2 * kTile + 512, dltp + prow, 512, &qd_full[st]);
          mask |= 1u << st;
          par = (par & ~(1u << st)) | (ph << st);
        }
      }
      if (kv_issued) mbar_wait(kv_full, kv_par, nullptr, 0);
      for (int s = 0; s < kStages; ++s)
        if ((mask >> s) & 1u) mbar_wait(&qd_full[s], (par >> s) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BKV, BQ, 0, 0);  // S^T, dP^T
      constexpr uint32_t idesc_a = make_idesc_bf16(BKV, D, 0, 1);   // dV, dK (dO / Q read MN-major)
      const uint32_t aK = smem_u32(smK), aV = smem_u32(smV);
      uint32_t g = 0, item_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int b, s0, L, jt, hk, nq, nblk;
        decode(item, b, s0, L, jt, hk, nq, nblk);
        if (!mbar_wait(kv_full, item_it & 1u, err, kTimeoutAttnKV)) { ok = false; break; }
        tc_fence_after();
        // Order per block: dV_b, S^T_{b+1}, dK_b, dP^T_{b+1}.  S^T_{b+1} overwrites
        // P^T_b and dP^T_{b+1} overwrites dS^T_b after the MMAs that read them.
        auto issue_s = [&](uint32_t gb) -> bool {
          const int st = gb % kStages;
          if (!mbar_wait(&qd_full[st], (gb / kStages) & 1u, err, kTimeoutAttnQ)) return false;
          tc_fence_after();
          const uint32_t aQ = smem_u32(smQD + st * kStageBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColS, kmajor_desc(aK, kk), kmajor_desc(aQ, kk), idesc_s, kk > 0);
          umma_commit(st_full);
          return true;
        };
        auto issue_dp = [&](uint32_t gb) {
          const uint32_t aDO = smem_u32(smQD + (gb % kStages) * kStageBytes) + kTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColDP, kmajor_desc(aV, kk), kmajor_desc(aDO, kk), idesc_s, kk > 0);
          umma_commit(dpt_full);
        };
        if (!issue_s(g)) { ok = false; break; }
        issue_dp(g);
        for (int blk = 0; blk < nblk; ++blk, ++g) {
          const int st = g % kStages;
          const uint32_t aQ = smem_u32(smQD + st * kStageBytes), aDO = aQ + kTile;
          if (!mbar_wait(p_full, g & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (blk == 0 && !mbar_wait(acc_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem_base + kColDV, tmem_base + split_half_col(kColS, kk), mnmajor_desc(aDO, kk), idesc_a,
                        (blk > 0 || kk > 0) ? 1u : 0u);
          if (blk + 1 < nblk && !issue_s(g + 1)) { ok = false; break; }
          if (!mbar_wait(ds_full, g & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem_base + kColDK, tmem_base + split_half_col(kColDP, kk), mnmajor_desc(aQ, kk), idesc_a,
                        (blk > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&qd_empty[st]);
          if (blk + 1 < nblk) issue_dp(g + 1);
        }
        if (!ok) break;
        umma_commit(kv_empty);
        umma_commit(acc_full);
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, half = (warp - 2) >> 2;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;  // this thread's 64 q columns of the kv row
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
    };
    uint32_t g = 0, item_it = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
      int b, s0, L, jt, hk, nq, nblk;
      decode(item, b, s0, L, jt, hk, nq, nblk);
      const int kp = jt * BKV + row;
      const bool row_ok = kp < L;
      for (int blk = 0; blk < nblk; ++blk, ++g) {
        int h, qi;
        block_q(blk, jt, nq, hk, h, qi);
        const int st = g % kStages;
        const float* s_lse = reinterpret_cast<const float*>(smQD + st * kStageBytes + 2 * kTile) + c0;
        const float* s_dlt = s_lse + 128;
        // the stage's lse2 / delta (bulk copies) are visible once its barrier completed
        if (!wait_all(&qd_full[st], (g / kStages) & 1u, kTimeoutAttnQ)) { ok = false; break; }
        if (!wait_all(st_full, g & 1u, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        float v[64];
        ld_half64(tmem_base + lane_addr + kColS + c0, v);
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4) {
          const float4 l4 = reinterpret_cast<const float4*>(s_lse)[c4];
          v[4 * c4 + 0] = ex2_approx(fmaf(v[4 * c4 + 0], scale_log2, -l4.x));
          v[4 * c4 + 1] = ex2_approx(fmaf(v[4 * c4 + 1], scale_log2, -l4.y));
          v[4 * c4 + 2] = ex2_approx(fmaf(v[4 * c4 + 2], scale_log2, -l4.z));
          v[4 * c4 + 3] = ex2_approx(fmaf(v[4 * c4 + 3], scale_log2, -l4.w));
        }
        const int q0 = qi * BQ + c0;
        if ((causal && qi == jt) || (qi + 1) * BQ > L) {  // diagonal block or last q tile
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int qp = q0 + c;
            v[c] = (qp < L && (!causal || kp <= qp)) ? v[c] : 0.f;
          }
        }
        // P^T over the first 32 of this half's S^T columns (already read)
        store_packed_half(tmem_base + lane_addr + kColS + c0, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (!wait_all(dpt_full, g & 1u, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t d[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + kColDP + c0 + c * 32, d);
          tmem_ld_wait();
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 d4 = reinterpret_cast<const float4*>(s_dlt + c * 32)[e4];
            const int i = c * 32 + e4 * 4;
            v[i + 0] *= (__uint_as_float(d[e4 * 4 + 0]) - d4.x) * scale;
            v[i + 1] *= (__uint_as_float(d[e4 * 4 + 1]) - d4.y) * scale;
            v[i + 2] *= (__uint_as_float(d[e4 * 4 + 2]) - d4.z) * scale;
            v[i + 3] *= (__uint_as_float(d[e4 * 4 + 3]) - d4.w) * scale;
          }
        }
        // dS^T over the first 32 of this half's dP^T columns (already read)
        store_packed_half(tmem_base + lane_addr + kColDP + c0, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
      if (!ok) break;
      if (!wait_all(acc_full, item_it & 1u, kTimeoutAttnO)) break;
      tc_fence_after();
      store_acc_half(tmem_base + lane_addr + kColDV + c0, dV + ((size_t)(s0 + kp) * Hkv + hk) * D + c0, row_ok);
      store_acc_half(tmem_base + lane_addr + kColDK + c0, dK + ((size_t)(s0 + kp) * Hkv + hk) * D + c0, row_ok);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ host
// q_tiles: (sequence, q tile) table of the forward; kv_tiles: (sequence, kv tile)
// table ordered by decreasing backward work.
std::vector<torch::Tensor> flash_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                     torch::Tensor out, torch::Tensor lse, torch::Tensor cu_seqlens,
                                     torch::Tensor q_tiles, torch::Tensor kv_tiles, double scale, bool causal,
                                     torch::Tensor err) {
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_qkv(out, "out");
  check_qkv(dout, "dout");
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k.size(1);
  LIBRA_CHECK(out.sizes() == q.sizes() && dout.sizes() == q.sizes() && Hq % Hkv == 0,
              "flash_bwd: out/dout must match q and Hq must be a multiple of Hkv");
  LIBRA_CHECK(k.size(0) == T && v.size(0) == T, "flash_bwd: q, k and v must have the same token count");
  LIBRA_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.size(0) == Hq &&
                  lse.size(1) == T,
              "flash_bwd: lse must be fp32 [Hq, T]");
  LIBRA_CHECK(cu_seqlens.is_cuda() && cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_contiguous(),
              "flash_bwd: cu_seqlens must be a contiguous CUDA int32 tensor");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  const int nkv = (int)kv_tiles.size(0), nq = (int)q_tiles.size(0);
  if (T == 0 || nq == 0) return {dq, dk, dv};
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t T_pad = pad_rows(T, cu_seqlens.numel() - 1);
  LIBRA_CHECK(T_pad * Hq < (int64_t)1 << 31, "flash_bwd: padded lse/delta arrays exceed 2^31 elements");
  auto lse2p = torch::empty({Hq, T_pad}, q.options().dtype(at::kFloat));
  auto dltp = torch::empty({Hq, T_pad}, q.options().dtype(at::kFloat));
  attn_delta_kernel<<<dim3(nq, Hq), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      lse.data_ptr<float>(), cu_seqlens.data_ptr<int>(), reinterpret_cast<const int2*>(q_tiles.data_ptr<int>()), Hq, T,
      (int)T_pad, lse2p.data_ptr<float>(), dltp.data_ptr<float>());
  LIBRA_LAUNCH_CHECK();
  const CUtensorMap mq = head_map(q), mk = head_map(k), mv = head_map(v), mdo = head_map(dout);
  static bool configured[kMaxDevices] = {};  // per device: the attributes are set on the current one
  if (!configured[current_device_index()]) {
    cudaFuncSetAttribute(flash_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dqk::kSmemBytes);
    cudaFuncSetAttribute(flash_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dkv::kSmemBytes);
    configured[current_device_index()] = true;
  }
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  if (nkv > 0) {
    const int items = nkv * Hkv;
    flash_bwd_dkdv_kernel<<<items < sms ? items : sms, kBwdThreads, dkv::kSmemBytes, stream>>>(
        mq, mk, mv, mdo, cu_seqlens.data_ptr<int>(), reinterpret_cast<const int2*>(kv_tiles.data_ptr<int>()), nkv, Hq,
        Hkv, lse2p.data_ptr<float>(), dltp.data_ptr<float>(), (int)T_pad,
        reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()),
        (float)scale, scale_log2, causal ? 1 : 0, err.data_ptr<int>());
    LIBRA_LAUNCH_CHECK();
  }
  const int items = nq * Hq;
  flash_bwd_dq_kernel<<<items < sms ? items : sms, kBwdThreads, dqk::kSmemBytes, stream>>>(
      mq, mk, mv, mdo, cu_seqlens.data_ptr<int>(), reinterpret_cast<const int2*>(q_tiles.data_ptr<int>()), nq, Hq,
      Hkv, lse2p.data_ptr<float>(), dltp.data_ptr<float>(), (int)T_pad,
      reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), (float)scale, scale_log2, causal ? 1 : 0, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
  return {dq, dk, dv};
}

}  // namespace attn
}  // namespace libra

// Backward pass of the tcgen05 varlen GQA attention (forward: flash_attn.cu).
//
// Three launches, no atomics:
//   delta    D[h, t]  = sum_d dO[t, h, d] * O[t, h, d]                (fp32)
//   dkdv     per (kv tile, kv head): loop over the group's q heads and the
//            q tiles at or after the kv tile (causal);
//              S^T  = K Q^T           P^T  = 2^(S^T c - lse_q)
//              dP^T = V dO^T          dS^T = P^T (dP^T - D_q) * scale
//              dV  += P^T dO          dK  += dS^T Q
//            TMEM: S^T [0,128) dP^T [128,256) dV [256,384) dK [384,512)
//   dq       per (q tile, q head): loop over kv tiles at or before it;
//              S = Q K^T   P = 2^(S c - lse)   dP = dO V^T
//              dS = P (dP - D) * scale         dQ += dS K
//            TMEM: S [0,128) dP [128,256) dQ [256,384)
// where c = scale * log2(e) and lse is the forward's natural-log denominator.
// The thread that owns a TMEM lane owns one row (kv row in dkdv, q row in dq);
// P^T / dS^T / dS go to a 128B-swizzled K-major smem tile that the next MMA
// reads (dS^T is also read MN-major as nothing else needs it).
// Same warp roles and bounded waits as the forward kernel.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_common.cuh"

namespace libra {
namespace attn {

// ------------------------------------------------------------------ delta
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ O, const __nv_bfloat16* __restrict__ dO,
                                  float* __restrict__ delta, int T, int H) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= T * H) return;
  const int t = w / H, h = w - t * H;
  const uint2 o = reinterpret_cast<const uint2*>(O + (size_t)w * D)[lane];
  const uint2 g = reinterpret_cast<const uint2*>(dO + (size_t)w * D)[lane];
  const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&o);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&g);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += __bfloat162float(ob[e]) * __bfloat162float(gb[e]);
  s = warp_sum(s);
  if (lane == 0) delta[(size_t)h * T + t] = s;
}

__device__ __forceinline__ void store_swizzled_row(uint8_t* tile, int row, const float* v, int vi0, int nvec) {
  // 8 bf16 per 16-byte unit; unit index XOR (row % 8) inside each 128-byte row
#pragma unroll
  for (int vi = 0; vi < 16; ++vi) {
    if (vi < vi0 || vi >= vi0 + nvec) continue;
    uint4 pk;
    pk.x = pack_bf16x2(v[vi * 8 + 0], v[vi * 8 + 1]);
    pk.y = pack_bf16x2(v[vi * 8 + 2], v[vi * 8 + 3]);
    pk.z = pack_bf16x2(v[vi * 8 + 4], v[vi * 8 + 5]);
    pk.w = pack_bf16x2(v[vi * 8 + 6], v[vi * 8 + 7]);
    const int unit = (vi & 7) ^ (row & 7);
    *reinterpret_cast<uint4*>(tile + (vi >> 3) * kChunk + row * 128 + unit * 16) = pk;
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

__device__ __forceinline__ void store_swizzled_half(uint8_t* tile, int row, const float (&v)[64], int half) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int vi = half * 8 + j;
    uint4 pk;
    pk.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
    pk.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
    pk.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
    pk.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
    const int unit = (vi & 7) ^ (row & 7);
    *reinterpret_cast<uint4*>(tile + (vi >> 3) * kChunk + row * 128 + unit * 16) = pk;
  }
}

// ------------------------------------------------------------------ dq
namespace dqk {
constexpr int kStages = 2;
constexpr int kOffQ = 0, kOffDO = kTile, kOffK = 2 * kTile, kOffV = kOffK + kStages * kTile;
constexpr int kOffDS = kOffV + kStages * kTile, kOffBar = kOffDS + kTile;
// q_full q_empty | k_full[2] v_full[2] kv_empty[2] | s_full s_empty dp_full dp_empty ds_full ds_free dq_full dq_empty done
constexpr int kNumBars = 2 + 3 * kStages + 9;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256;
}  // namespace dqk

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const int* __restrict__ cu, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv,
                        const float* __restrict__ lse, const float* __restrict__ delta,
                        __nv_bfloat16* __restrict__ dQ, int T, float scale, float scale_log2, int causal, int* err) {
  using namespace dqk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *q_full = bars, *q_empty = bars + 1, *k_full = bars + 2, *v_full = k_full + kStages,
           *kv_empty = v_full + kStages, *s_full = kv_empty + kStages, *s_empty = s_full + 1,
           *dp_full = s_full + 2, *dp_empty = s_full + 3, *ds_full = s_full + 4, *ds_free = s_full + 5,
           *dq_full = s_full + 6, *dq_empty = s_full + 7, *done = s_full + 8;
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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, kSoftmaxWarps);
    mbar_init(dp_full, 1);
    mbar_init(dp_empty, kSoftmaxWarps);
    mbar_init(ds_full, kSoftmaxWarps);
    mbar_init(ds_free, 1);
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
  uint8_t *smQ = smem + kOffQ, *smDO = smem + kOffDO, *smK = smem + kOffK, *smV = smem + kOffV,
          *smDS = smem + kOffDS;

  auto decode = [&](int item, int& s0, int& L, int& q0, int& h, int& hk, int& nkv) {
    const int2 t = tiles[item / Hq];
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
      uint32_t kv_it = 0, item_it = 0, q_par = 0;
      bool ok = true, q_issued = false, issued[kStages] = {false, false};
      uint32_t par[kStages] = {0, 0};
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int s0, L, q0, h, hk, nkv;
        decode(item, s0, L, q0, h, hk, nkv);
        if (!mbar_wait(q_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        mbar_expect_tx(q_full, 2 * kTile);
        tma_load_2d(smQ, &tmQ, q_full, h * D, s0 + q0);
        tma_load_2d(smQ + kChunk, &tmQ, q_full, h * D + 64, s0 + q0);
        tma_load_2d(smDO, &tmDO, q_full, h * D, s0 + q0);
        tma_load_2d(smDO + kChunk, &tmDO, q_full, h * D + 64, s0 + q0);
        q_issued = true;
        q_par = item_it & 1u;
        for (int j = 0; j < nkv; ++j, ++kv_it) {
          const int st = kv_it % kStages;
          const uint32_t ph = (kv_it / kStages) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          const int y = s0 + j * BKV;
          mbar_expect_tx(&k_full[st], kTile);
          tma_load_2d(smK + st * kTile, &tmK, &k_full[st], hk * D, y);
          tma_load_2d(smK + st * kTile + kChunk, &tmK, &k_full[st], hk * D + 64, y);
          mbar_expect_tx(&v_full[st], kTile);
          tma_load_2d(smV + st * kTile, &tmV, &v_full[st], hk * D, y);
          tma_load_2d(smV + st * kTile + kChunk, &tmV, &v_full[st], hk * D + 64, y);
          issued[st] = true;
          par[st] = ph;
        }
      }
      if (q_issued) mbar_wait(q_full, q_par, nullptr, 0);
      for (int s = 0; s < kStages; ++s)
        if (issued[s]) {
          mbar_wait(&k_full[s], par[s], nullptr, 0);
          mbar_wait(&v_full[s], par[s], nullptr, 0);
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_kk = make_idesc_bf16(BQ, BKV, 0, 0);  // S, dP
      constexpr uint32_t idesc_dq = make_idesc_bf16(BQ, D, 0, 1);    // dQ = dS K (K read MN-major)
      const uint32_t aQ = smem_u32(smQ), aDO = smem_u32(smDO), aDS = smem_u32(smDS);
      uint32_t kv_it = 0, blk = 0, item_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int s0, L, q0, h, hk, nkv;
        decode(item, s0, L, q0, h, hk, nkv);
        if (!mbar_wait(q_full, item_it & 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        tc_fence_after();
        // S_{j+1} and dP_{j+1} are issued before waiting for dS_j, so the tensor
        // core works on the next block while the softmax warps build dS_j.
        const uint32_t blk0 = blk;
        auto issue_sdp = [&](int j) -> bool {
          const uint32_t g = blk0 + j, idx = kv_it + j;
          const int st = idx % kStages;
          const uint32_t ph = (idx / kStages) & 1u;
          if (!mbar_wait(&k_full[st], ph, err, kTimeoutAttnKV)) return false;
          if (!mbar_wait(s_empty, (g & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aK = smem_u32(smK + st * kTile), aV = smem_u32(smV + st * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColS, kmajor_desc(aQ, kk), kmajor_desc(aK, kk), idesc_kk, kk > 0);
          umma_commit(s_full);
          if (!mbar_wait(&v_full[st], ph, err, kTimeoutAttnKV)) return false;
          if (!mbar_wait(dp_empty, (g & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColDP, kmajor_desc(aDO, kk), kmajor_desc(aV, kk), idesc_kk, kk > 0);
          umma_commit(dp_full);
          if (j + 1 == nkv) umma_commit(q_empty);  // Q and dO are no longer read
          return true;
        };
        if (!issue_sdp(0)) { ok = false; break; }
        for (int j = 0; j < nkv; ++j, ++blk) {
          if (j + 1 < nkv && !issue_sdp(j + 1)) { ok = false; break; }
          const uint32_t idx = kv_it + j;
          const int st = idx % kStages;
          const uint32_t aK = smem_u32(smK + st * kTile);
          if (!mbar_wait(ds_full, blk & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (j == 0 && !mbar_wait(dq_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16(tmem_base + kColDQ, kmajor_desc(aDS, kk), mnmajor_desc(aK, kk), idesc_dq,
                     (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&kv_empty[st]);
          umma_commit(ds_free);
        }
        if (!ok) break;
        umma_commit(dq_full);
        kv_it += nkv;
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    const int quarter = warp & 3, row = quarter * 32 + lane, half = (warp - 2) >> 2;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;  // this thread's 64 columns of the row
    uint32_t blk = 0, item_it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++item_it) {
      int s0, L, q0, h, hk, nkv;
      decode(item, s0, L, q0, h, hk, nkv);
      const int qp = q0 + row;
      const bool row_ok = qp < L;
      const float lse2 = row_ok ? lse[(size_t)h * T + s0 + qp] * 1.4426950408889634f : 0.f;
      const float dlt = row_ok ? delta[(size_t)h * T + s0 + qp] : 0.f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j, ++blk) {
        float v[64];
        if (!mbar_wait(s_full, blk & 1u, err, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        ld_half64(tmem_base + lane_addr + kColS + c0, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);
        const int kb = j * BKV + c0;
        const int lim = causal ? min(qp + 1, L) : L;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p = ex2_approx(v[c] * scale_log2 - lse2);
          v[c] = (row_ok && kb + c < lim) ? p : 0.f;
        }
        if (!mbar_wait(dp_full, blk & 1u, err, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t d[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + kColDP + c0 + c * 32, d);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[c * 32 + e] = v[c * 32 + e] * (__uint_as_float(d[e]) - dlt) * scale;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dp_empty);
        if (j > 0) {  // the previous dQ MMA has read the dS tile
          if (!mbar_wait(ds_free, (blk - 1) & 1u, err, kTimeoutAttnPV)) { ok = false; break; }
        }
        store_swizzled_half(smDS, row, v, half);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
      if (!ok) break;
      if (!mbar_wait(dq_full, item_it & 1u, err, kTimeoutAttnO)) break;
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
constexpr int kStages = 2;
constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile;           // Q stages at kOffQ + st * 2 * kTile
constexpr int kOffPDS = kOffQ + kStages * 2 * kTile;                 // (dO of a stage follows its Q)
constexpr int kOffLD = kOffPDS + kTile;                              // lse2[128], delta[128] fp32
constexpr int kOffBar = kOffLD + 2 * 128 * 4;
// kv_full kv_empty | qd_full[2] qd_empty[2] | st_full st_empty dpt_full dpt_empty p_full dv_done ds_full pds_free
// acc_full acc_empty done grp
constexpr int kNumBars = 2 + 2 * kStages + 12;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 384;
}  // namespace dkv

// Barrier of the 128 softmax threads through an mbarrier, so it is bounded like
// every other wait (a named hardware barrier would wait forever if one warp
// left on a timeout).
__device__ __forceinline__ bool softmax_group_sync(uint64_t* bar, uint32_t& n, int* err) {
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, n & 1u, err, kTimeoutAttnS);
  ++n;
  return ok;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                          const int* __restrict__ cu, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv,
                          const float* __restrict__ lse, const float* __restrict__ delta,
                          __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV, int T, float scale,
                          float scale_log2, int causal, int* err) {
  using namespace dkv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *kv_full = bars, *kv_empty = bars + 1, *qd_full = bars + 2, *qd_empty = qd_full + kStages,
           *b0 = qd_empty + kStages;
  uint64_t *st_full = b0, *st_empty = b0 + 1, *dpt_full = b0 + 2, *dpt_empty = b0 + 3, *p_full = b0 + 4,
           *dv_done = b0 + 5, *ds_full = b0 + 6, *pds_free = b0 + 7, *acc_full = b0 + 8, *acc_empty = b0 + 9,
           *done = b0 + 10, *grp = b0 + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(grp + 1);
  float* s_lse = reinterpret_cast<float*>(smem + kOffLD);  // [128]
  float* s_dlt = s_lse + 128;                              // [128]
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
    mbar_init(st_empty, kSoftmaxWarps);
    mbar_init(dpt_full, 1);
    mbar_init(dpt_empty, kSoftmaxWarps);
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(dv_done, 1);
    mbar_init(ds_full, kSoftmaxWarps);
    mbar_init(pds_free, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kSoftmaxWarps);
    mbar_init(done, 1);
    mbar_init(grp, 32 * kSoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint8_t *smK = smem + kOffK, *smV = smem + kOffV, *smQD = smem + kOffQ, *smPDS = smem + kOffPDS;

  // item = (kv tile, kv head); blocks = group q heads x q tiles [jt, nq)
  auto decode = [&](int item, int& s0, int& L, int& jt, int& hk, int& nq, int& nblk) {
    const int2 t = tiles[item / Hkv];
    hk = item % Hkv;
    s0 = cu[t.x];
    L = cu[t.x + 1] - s0;
    jt = t.y;
    nq = (L + BQ - 1) / BQ;
    nblk = group * (causal ? nq - jt : nq);
  };
  auto block_q = [&](int b, int jt, int nq, int hk, int& h, int& qi) {
    const int per = causal ? nq - jt : nq;
    h = hk * group + b / per;
    qi = (causal ? jt : 0) + b % per;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t qd_it = 0, item_it = 0, kv_par = 0;
      bool ok = true, kv_issued = false, issued[kStages] = {false, false};
      uint32_t par[kStages] = {0, 0};
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int s0, L, jt, hk, nq, nblk;
        decode(item, s0, L, jt, hk, nq, nblk);
        if (!mbar_wait(kv_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
        mbar_expect_tx(kv_full, 2 * kTile);
        tma_load_2d(smK, &tmK, kv_full, hk * D, s0 + jt * BKV);
        tma_load_2d(smK + kChunk, &tmK, kv_full, hk * D + 64, s0 + jt * BKV);
        tma_load_2d(smV, &tmV, kv_full, hk * D, s0 + jt * BKV);
        tma_load_2d(smV + kChunk, &tmV, kv_full, hk * D + 64, s0 + jt * BKV);
        kv_issued = true;
        kv_par = item_it & 1u;
        for (int b = 0; b < nblk; ++b, ++qd_it) {
          int h, qi;
          block_q(b, jt, nq, hk, h, qi);
          const int st = qd_it % kStages;
          const uint32_t ph = (qd_it / kStages) & 1u;
          if (!mbar_wait(&qd_empty[st], ph ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
          uint8_t* q = smQD + st * 2 * kTile;
          mbar_expect_tx(&qd_full[st], 2 * kTile);
          tma_load_2d(q, &tmQ, &qd_full[st], h * D, s0 + qi * BQ);
          tma_load_2d(q + kChunk, &tmQ, &qd_full[st], h * D + 64, s0 + qi * BQ);
          tma_load_2d(q + kTile, &tmDO, &qd_full[st], h * D, s0 + qi * BQ);
          tma_load_2d(q + kTile + kChunk, &tmDO, &qd_full[st], h * D + 64, s0 + qi * BQ);
          issued[st] = true;
          par[st] = ph;
        }
      }
      if (kv_issued) mbar_wait(kv_full, kv_par, nullptr, 0);
      for (int s = 0; s < kStages; ++s)
        if (issued[s]) mbar_wait(&qd_full[s], par[s], nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BKV, BQ, 0, 0);  // S^T, dP^T
      constexpr uint32_t idesc_a = make_idesc_bf16(BKV, D, 0, 1);   // dV, dK (dO / Q read MN-major)
      const uint32_t aK = smem_u32(smK), aV = smem_u32(smV), aPDS = smem_u32(smPDS);
      uint32_t qd_it = 0, item_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        int s0, L, jt, hk, nq, nblk;
        decode(item, s0, L, jt, hk, nq, nblk);
        if (!mbar_wait(kv_full, item_it & 1u, err, kTimeoutAttnKV)) { ok = false; break; }
        tc_fence_after();
        // S^T_{b+1} is issued between dV_b and dK_b, dP^T_{b+1} right after dK_b:
        // the tensor core works on the next block while the softmax warps build
        // P^T_b and dS^T_b.
        const uint32_t qd0 = qd_it;
        auto issue_s = [&](int b) -> bool {
          const uint32_t g = qd0 + b;
          const int st = g % kStages;
          if (!mbar_wait(&qd_full[st], (g / kStages) & 1u, err, kTimeoutAttnQ)) return false;
          if (!mbar_wait(st_empty, (g & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aQ = smem_u32(smQD + st * 2 * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColS, kmajor_desc(aK, kk), kmajor_desc(aQ, kk), idesc_s, kk > 0);
          umma_commit(st_full);
          return true;
        };
        auto issue_dp = [&](int b) -> bool {
          const uint32_t g = qd0 + b;
          const int st = g % kStages;
          if (!mbar_wait(dpt_empty, (g & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aDO = smem_u32(smQD + st * 2 * kTile) + kTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + kColDP, kmajor_desc(aV, kk), kmajor_desc(aDO, kk), idesc_s, kk > 0);
          umma_commit(dpt_full);
          return true;
        };
        if (!issue_s(0) || !issue_dp(0)) { ok = false; break; }
        for (int b = 0; b < nblk; ++b, ++qd_it) {
          const int st = qd_it % kStages;
          const uint32_t aQ = smem_u32(smQD + st * 2 * kTile), aDO = aQ + kTile;
          if (!mbar_wait(p_full, qd_it & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (b == 0 && !mbar_wait(acc_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16(tmem_base + kColDV, kmajor_desc(aPDS, kk), mnmajor_desc(aDO, kk), idesc_a,
                     (b > 0 || kk > 0) ? 1u : 0u);
          umma_commit(dv_done);
          if (b + 1 < nblk && !issue_s(b + 1)) { ok = false; break; }
          if (!mbar_wait(ds_full, qd_it & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16(tmem_base + kColDK, kmajor_desc(aPDS, kk), mnmajor_desc(aQ, kk), idesc_a,
                     (b > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&qd_empty[st]);
          umma_commit(pds_free);
          if (b + 1 < nblk && !issue_dp(b + 1)) { ok = false; break; }
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
    const int tid = threadIdx.x - 64;  // 0..255
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 64;  // this thread's 64 q columns of the kv row
    uint32_t qd_it = 0, item_it = 0, nsync = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++item_it) {
      int s0, L, jt, hk, nq, nblk;
      decode(item, s0, L, jt, hk, nq, nblk);
      const int kp = jt * BKV + row;
      const bool row_ok = kp < L;
      bool ok = true;
      for (int b = 0; b < nblk; ++b, ++qd_it) {
        int h, qi;
        block_q(b, jt, nq, hk, h, qi);
        // this block's lse (base 2) and delta for its 128 q rows, after every
        // thread has finished with the previous block's
        if (!softmax_group_sync(grp, nsync, err)) { ok = false; break; }
        if (tid < 128) {
          const int qp = qi * BQ + tid;
          const bool qok = qp < L;
          s_lse[tid] = qok ? lse[(size_t)h * T + s0 + qp] * 1.4426950408889634f : 0.f;
          s_dlt[tid] = qok ? delta[(size_t)h * T + s0 + qp] : 0.f;
        }
        if (!softmax_group_sync(grp, nsync, err)) { ok = false; break; }
        float v[64];
        if (!mbar_wait(st_full, qd_it & 1u, err, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        ld_half64(tmem_base + lane_addr + kColS + c0, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_empty);
        const int q0 = qi * BQ + c0;
        const float* lrow = s_lse + c0;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int qp = q0 + c;
          const float p = ex2_approx(v[c] * scale_log2 - lrow[c]);
          v[c] = (row_ok && qp < L && (!causal || kp <= qp)) ? p : 0.f;
        }
        if (b > 0) {  // previous dK MMA has read the P/dS tile
          if (!mbar_wait(pds_free, (qd_it - 1) & 1u, err, kTimeoutAttnPV)) { ok = false; break; }
        }
        store_swizzled_half(smPDS, row, v, half);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (!mbar_wait(dpt_full, qd_it & 1u, err, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        const float* drow = s_dlt + c0;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t d[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + kColDP + c0 + c * 32, d);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            v[c * 32 + e] = v[c * 32 + e] * (__uint_as_float(d[e]) - drow[c * 32 + e]) * scale;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dpt_empty);
        if (!mbar_wait(dv_done, qd_it & 1u, err, kTimeoutAttnPV)) { ok = false; break; }
        store_swizzled_half(smPDS, row, v, half);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
      if (!ok) break;
      if (!mbar_wait(acc_full, item_it & 1u, err, kTimeoutAttnO)) break;
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
  LIBRA_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.size(0) == Hq &&
                  lse.size(1) == T,
              "flash_bwd: lse must be fp32 [Hq, T]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  if (T == 0) return {dq, dk, dv};
  auto stream = at::cuda::getCurrentCUDAStream();
  auto delta = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  {
    const int warps = T * Hq, per_block = 8;
    attn_delta_kernel<<<(warps + per_block - 1) / per_block, per_block * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        delta.data_ptr<float>(), T, Hq);
    LIBRA_LAUNCH_CHECK();
  }
  const CUtensorMap mq = head_map(q), mk = head_map(k), mv = head_map(v), mdo = head_map(dout);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(flash_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dqk::kSmemBytes);
    cudaFuncSetAttribute(flash_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dkv::kSmemBytes);
    configured = true;
  }
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  const int nkv = (int)kv_tiles.size(0), nq = (int)q_tiles.size(0);
  if (nkv > 0) {
    const int items = nkv * Hkv;
    flash_bwd_dkdv_kernel<<<items < sms ? items : sms, kBwdThreads, dkv::kSmemBytes, stream>>>(
        mq, mk, mv, mdo, cu_seqlens.data_ptr<int>(), reinterpret_cast<const int2*>(kv_tiles.data_ptr<int>()), nkv, Hq,
        Hkv, lse.data_ptr<float>(), delta.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()), T, (float)scale, scale_log2, causal ? 1 : 0,
        err.data_ptr<int>());
    LIBRA_LAUNCH_CHECK();
  }
  if (nq > 0) {
    const int items = nq * Hq;
    flash_bwd_dq_kernel<<<items < sms ? items : sms, kBwdThreads, dqk::kSmemBytes, stream>>>(
        mq, mk, mv, mdo, cu_seqlens.data_ptr<int>(), reinterpret_cast<const int2*>(q_tiles.data_ptr<int>()), nq, Hq,
        Hkv, lse.data_ptr<float>(), delta.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), T,
        (float)scale, scale_log2, causal ? 1 : 0, err.data_ptr<int>());
    LIBRA_LAUNCH_CHECK();
  }
  return {dq, dk, dv};
}

}  // namespace attn
}  // namespace libra

// Causal (or full) GQA attention over packed variable-length sequences on the
// 5th-generation tensor cores: forward pass.
//
//   q [T, Hq, 128], k/v [T, Hkv, 128] bf16, cu_seqlens [B+1] int32
//   o [T, Hq, 128] bf16, lse [Hq, T] fp32 (natural log of the softmax denominator)
//
// Replaces the SDPA/flash call of the reference's attention adapter
// (engine/megatron_core_attention.py:447-456).
//
// Work item = (sequence, 128-row q tile, q head); a persistent grid walks a
// host-built tile table (heaviest causal tiles first, the Hq heads of a tile
// adjacent so the shared K/V of a kv head stay in L2).
//
// One CTA (192 threads) per SM:
//   warp 0      TMA producer: Q tile (32 KB), then K_j and V_j (32 KB each) into
//               a 2-stage ring.  K and V use the same [kv rows][64 dims] box;
//               K is read as a K-major B operand, V as an MN-major B operand.
//   warp 1      tcgen05.mma issuer: S_j = Q K_j^T into one of two TMEM S
//               buffers (issued one block ahead), O += P_j V_j into TMEM O.
//   warps 2-5   softmax: thread = q row = TMEM lane.  tcgen05.ld the S row,
//               mask, online max/sum in base 2, P_j as bf16 into a 128B-swizzled
//               smem tile (the A operand of the PV MMA).  The running max only
//               moves when it grows by more than 2^8, so O (in TMEM) is rescaled
//               rarely; the final O / l uses the same max and stays exact.
//               Epilogue: tcgen05.ld O, divide by l, store bf16 rows and lse.
// TMEM: S0 [0,128) S1 [128,256) O [256,384) (512 allocated).
// Every wait is bounded; on a timeout the kernel records an error code, drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_common.cuh"

namespace libra {
namespace attn {

constexpr int kStages = 2;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;
constexpr int kOffV = kOffK + kStages * kTile;
constexpr int kOffP = kOffV + kStages * kTile;
constexpr int kOffX = kOffP + kTile;  // row max / sum exchange between the two warps of a row: [2][2][128] fp32
constexpr int kOffBar = kOffX + 2 * 2 * 128 * 4;
// q_full q_empty | k_full[2] v_full[2] kv_empty[2] | s_full[2] s_empty[2] | p_full pv_done o_empty done grp
constexpr int kNumBars = 2 + 3 * kStages + 4 + 5;
// softmax: two warps per row (warps w and w+4 share a TMEM lane quarter), 64 columns each
constexpr int kFwdSoftmaxWarps = 8;
constexpr int kFwdThreads = 64 + 32 * kFwdSoftmaxWarps;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// One work item.  Queries may be the suffix of their sequence (prefix-cached
// extend): q rows [s0, s0 + L) of the packed q tensor are positions
// [off, off + L) of a key sequence stored at rows [k0, k0 + Lk) of k/v, with
// off = Lk - L (0 in training, where cu_k == cu_q).
struct Item {
  int s0, L, q0, h, hk, nkv, k0, Lk, off;
};

__device__ __forceinline__ Item decode(int item, const int* __restrict__ cu, const int* __restrict__ cu_k,
                                       const int2* __restrict__ tiles, int Hq, int group, int causal) {
  const int2 t = tiles[item / Hq];
  Item it;
  it.h = item % Hq;
  it.hk = it.h / group;
  it.s0 = cu[t.x];
  it.L = cu[t.x + 1] - it.s0;
  it.k0 = cu_k[t.x];
  it.Lk = cu_k[t.x + 1] - it.k0;
  it.off = it.Lk - it.L;
  it.q0 = t.y * BQ;
  const int nall = (it.Lk + BKV - 1) / BKV;
  // causal: key blocks up to the one holding the tile's last query position
  it.nkv = causal ? min((it.off + it.q0 + BQ - 1) / BKV + 1, nall) : nall;
  return it;
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const int* __restrict__ cu,
                     const int* __restrict__ cu_k, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv, __nv_bfloat16* __restrict__ O,
                     float* __restrict__ lse, int T, float scale_log2, int causal, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* o_empty = pv_done + 1;
  uint64_t* done = o_empty + 1;
  uint64_t* grp = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(grp + 1);
  float* xchg = reinterpret_cast<float*>(smem + kOffX);  // [parity][half][row]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = n_tiles * Hq;
  const int group = Hq / Hkv;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], kFwdSoftmaxWarps);
    }
    mbar_init(p_full, kFwdSoftmaxWarps);
    mbar_init(pv_done, 1);
    mbar_init(o_empty, kFwdSoftmaxWarps);
    mbar_init(done, 1);
    mbar_init(grp, 32 * kFwdSoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  uint8_t* smQ = smem + kOffQ;
  uint8_t* smK = smem + kOffK;
  uint8_t* smV = smem + kOffV;
  uint8_t* smP = smem + kOffP;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t kv_it = 0, item_it = 0;
      bool q_issued = false, ok = true;
      uint32_t q_par = 0;
      uint32_t last_k_par[kStages] = {0, 0}, last_v_par[kStages] = {0, 0};
      bool k_issued[kStages] = {false, false};
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
        if (!mbar_wait(q_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        mbar_expect_tx(q_full, kTile);
        tma_load_2d(smQ, &tmQ, q_full, it.h * D, it.s0 + it.q0);
        tma_load_2d(smQ + kChunk, &tmQ, q_full, it.h * D + 64, it.s0 + it.q0);
        q_issued = true;
        q_par = item_it & 1u;
        for (int j = 0; j < it.nkv; ++j, ++kv_it) {
          const int st = kv_it % kStages;
          const uint32_t ph = (kv_it / kStages) & 1u;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          const int y = it.k0 + j * BKV;
          mbar_expect_tx(&k_full[st], kTile);
          tma_load_2d(smK + st * kTile, &tmK, &k_full[st], it.hk * D, y);
          tma_load_2d(smK + st * kTile + kChunk, &tmK, &k_full[st], it.hk * D + 64, y);
          mbar_expect_tx(&v_full[st], kTile);
          tma_load_2d(smV + st * kTile, &tmV, &v_full[st], it.hk * D, y);
          tma_load_2d(smV + st * kTile + kChunk, &tmV, &v_full[st], it.hk * D + 64, y);
          k_issued[st] = true;
          last_k_par[st] = ph;
          last_v_par[st] = ph;
        }
      }
      // drain: every copy this thread issued must land before the CTA exits
      if (q_issued) mbar_wait(q_full, q_par, nullptr, 0);
      for (int s = 0; s < kStages; ++s)
        if (k_issued[s]) {
          mbar_wait(&k_full[s], last_k_par[s], nullptr, 0);
          mbar_wait(&v_full[s], last_v_par[s], nullptr, 0);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(BQ, D, 0, 1);
      const uint32_t aQ = smem_u32(smQ), aP = smem_u32(smP);
      uint32_t kv_it = 0, s_it = 0, pv_it = 0, item_it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
        if (!mbar_wait(q_full, item_it & 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        tc_fence_after();
        auto issue_s = [&](int j) -> bool {
          const uint32_t idx = kv_it + j;
          const int st = idx % kStages;
          if (!mbar_wait(&k_full[st], (idx / kStages) & 1u, err, kTimeoutAttnKV)) return false;
          const int sb = s_it & 1;
          if (!mbar_wait(&s_empty[sb], ((s_it >> 1) & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aK = smem_u32(smK + st * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + sb * BKV, kmajor_desc(aQ, kk), kmajor_desc(aK, kk), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[sb]);
          ++s_it;
          return true;
        };
        if (!issue_s(0)) { ok = false; break; }
        for (int j = 0; j < it.nkv && ok; ++j) {
          if (j + 1 < it.nkv) {
            if (!issue_s(j + 1)) { ok = false; break; }
          } else {
            umma_commit(q_empty);  // every S MMA of this item is issued: Q frees when they finish
          }
          const uint32_t idx = kv_it + j;
          const int st = idx % kStages;
          if (!mbar_wait(p_full, pv_it & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (!mbar_wait(&v_full[st], (idx / kStages) & 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          if (j == 0 && !mbar_wait(o_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aV = smem_u32(smV + st * kTile);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16(tmem_base + kColO, kmajor_desc(aP, kk), mnmajor_desc(aV, kk), idesc_o,
                     (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&kv_empty[st]);
          umma_commit(pv_done);
          ++pv_it;
        }
        kv_it += it.nkv;
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int half = (warp - 2) >> 2;  // which 64 of the 128 key columns (and of the 128 O columns)
    const int c0 = half * 64;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    uint32_t s_it = 0, pv_it = 0, item_it = 0, nsync = 0;
    // exchange a per-row value with the partner warp (other half of the same row)
    auto exchange = [&](float mine, float& theirs) -> bool {
      const int par = nsync & 1;
      xchg[(par * 2 + half) * 128 + row] = mine;
      mbar_arrive(grp);
      const bool okw = mbar_wait(grp, nsync & 1u, err, kTimeoutAttnS);
      ++nsync;
      theirs = xchg[(par * 2 + (half ^ 1)) * 128 + row];
      return okw;
    };
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++item_it) {
      const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
      const int qp = it.q0 + row;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < it.nkv; ++j) {
        const int sb = s_it & 1;
        if (!mbar_wait(&s_full[sb], (s_it >> 1) & 1u, err, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[64];
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tmem_ld_32x32b_x32(tmem_base + lane_addr + sb * BKV + c0 + c * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);
        ++s_it;
        // scale into log2 units and mask
        const int kb = j * BKV + c0;
        const int lim = causal ? min(it.off + qp + 1, it.Lk) : it.Lk;  // keys below lim are visible
        float bm = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          float v = __uint_as_float(r[c]) * scale_log2;
          v = (kb + c < lim) ? v : -INFINITY;
          r[c] = __float_as_uint(v);
          bm = fmaxf(bm, v);
        }
        float bm_other;
        if (!exchange(bm, bm_other)) { ok = false; break; }
        bm = fmaxf(bm, bm_other);  // both halves now hold the same block max
        const float m_new = fmaxf(m, bm);
        const bool rescale = (j > 0) && (m_new > m + kRescaleThreshold);
        if (j == 0) m = m_new;
        if (j > 0) {  // PV_{j-1} finished: O is stable and the P buffer is free
          if (!mbar_wait(pv_done, (pv_it - 1) & 1u, err, kTimeoutAttnPV)) { ok = false; break; }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {
          const float f = rescale ? ex2_approx(m - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tmem_base + lane_addr + kColO + c0 + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st_32x32b_x32(tmem_base + lane_addr + kColO + c0 + c * 32, o);
          }
          tmem_st_wait();
          if (rescale) {
            l *= f;
            m = m_new;
          }
        }
        // P = 2^(s - m) as bf16: this half's 64 columns of row `row` in the 128B-swizzled K-major tile
        float sum = 0.f;
#pragma unroll
        for (int j8 = 0; j8 < 8; ++j8) {
          float p[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            p[e] = ex2_approx(__uint_as_float(r[j8 * 8 + e]) - m);
            sum += p[e];
          }
          uint4 pk;
          pk.x = pack_bf16x2(p[0], p[1]);
          pk.y = pack_bf16x2(p[2], p[3]);
          pk.z = pack_bf16x2(p[4], p[5]);
          pk.w = pack_bf16x2(p[6], p[7]);
          const int vi = half * 8 + j8;
          const int unit = (vi & 7) ^ (row & 7);
          *reinterpret_cast<uint4*>(smP + (vi >> 3) * kChunk + row * 128 + unit * 16) = pk;
        }
        l += sum;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        ++pv_it;
      }
      if (!ok) break;
      // epilogue: row sum of both halves, then this half's 64 O columns
      float l_other;
      if (!exchange(l, l_other)) break;
      l += l_other;
      if (!mbar_wait(pv_done, (pv_it - 1) & 1u, err, kTimeoutAttnPV)) break;
      tc_fence_after();
      const bool row_ok = qp < it.L;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = O + ((size_t)(it.s0 + qp) * Hq + it.h) * D + c0;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + kColO + c0 + c * 32, o);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            pk.y = pack_bf16x2(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            pk.z = pack_bf16x2(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            pk.w = pack_bf16x2(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + q4 * 8) = pk;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      if (row_ok && half == 0) lse[(size_t)it.h * T + it.s0 + qp] = (m + lg2_approx(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// tiles: int32 [n, 2] = (sequence index, q tile index) on the device.
// cu_k: key offsets when the queries are the suffix of their sequences
// (prefix-cached extend); defaults to cu_seqlens (training, self-attention).
std::vector<torch::Tensor> flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor cu_seqlens,
                                     torch::Tensor tiles, double scale, bool causal, torch::Tensor err,
                                     c10::optional<torch::Tensor> cu_k) {
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hkv = (int)k.size(1);
  LIBRA_CHECK(v.size(0) == k.size(0) && v.size(1) == Hkv && Hkv > 0 && Hq % Hkv == 0,
              "flash_attn: k/v token counts must match and Hq must be a multiple of Hkv");
  LIBRA_CHECK(cu_seqlens.is_cuda() && cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_contiguous(),
              "flash_attn: cu_seqlens must be a contiguous CUDA int32 tensor");
  const torch::Tensor& cuk = cu_k.has_value() ? *cu_k : cu_seqlens;
  LIBRA_CHECK(cuk.is_cuda() && cuk.scalar_type() == at::kInt && cuk.is_contiguous() &&
                  cuk.numel() == cu_seqlens.numel(),
              "flash_attn: cu_k must be a contiguous CUDA int32 tensor shaped like cu_seqlens");
  LIBRA_CHECK(cu_k.has_value() || k.size(0) == T, "flash_attn: q and k token counts differ but no cu_k given");
  LIBRA_CHECK(tiles.is_cuda() && tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 2 &&
                  tiles.is_contiguous(),
              "flash_attn: tiles must be a contiguous CUDA int32 [n, 2] tensor");
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  const int n_tiles = (int)tiles.size(0);
  if (T == 0 || n_tiles == 0 || k.size(0) == 0) return {o, lse};
  const CUtensorMap mq = head_map(q), mk = head_map(k), mv = head_map(v);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    configured = true;
  }
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int items = n_tiles * Hq;
  const int grid = items < sms ? items : sms;
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  flash_fwd_kernel<<<grid, kFwdThreads, kSmemBytes, at::cuda::getCurrentCUDAStream()>>>(
      mq, mk, mv, cu_seqlens.data_ptr<int>(), cuk.data_ptr<int>(), reinterpret_cast<const int2*>(tiles.data_ptr<int>()),
      n_tiles, Hq, Hkv, reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), lse.data_ptr<float>(), T, scale_log2,
      causal ? 1 : 0, err.data_ptr<int>());
  LIBRA_LAUNCH_CHECK();
  return {o, lse};
}

}  // namespace attn
}  // namespace libra

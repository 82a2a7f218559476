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
// One CTA (320 threads) per SM:
//   warp 0      TMA producer: Q tile (32 KB), then K_j into a 3-stage ring (a
//               slot frees when S_j is computed) and V_j into a 2-stage ring
//               (frees after PV_j), K one block ahead of V; K/V blocks are
//               prefetched into L2 three blocks ahead of their loads.  K and V
//               use the same [kv rows][64 dims] box; K is read as a K-major B
//               operand, V as an MN-major B operand.
//   warp 1      tcgen05.mma issuer: S_j = Q K_j^T into one of two TMEM S
//               buffers (issued one block ahead), O += P_j V_j with P_j read
//               from TMEM (A operand in tensor memory).
//   warps 2-9   softmax: warps w and w+4 share a TMEM lane quarter, 16 rows
//               each; with the 16x256b load shape four threads hold one row
//               (32 of its 128 scores each), so row max / sum reduce with two
//               shuffles and no cross-warp synchronisation.  The mask is applied
//               only on blocks that cross the causal diagonal or the sequence
//               end; the scale folds into one FFMA per score.  P_j goes back to
//               TMEM as packed bf16 (16x128b shape), double-buffered so the next
//               block's P never waits for the PV MMA still reading the previous one.  The running max only
//               moves when it grows by more than 2^8, so O (in TMEM) is rescaled
//               rarely; the final O / l uses the same max and stays exact.
//               Epilogue: tcgen05.ld O, divide by l, stage bf16 rows in a
//               per-warp swizzled smem area and write them out coalesced, plus lse.
// TMEM: S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512).
// Every wait is bounded; on a timeout the kernel records an error code, drains
// its in-flight copies and MMAs, frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_common.cuh"

namespace libra {
namespace attn {

constexpr int kKStages = 3;  // K_j frees as soon as S_j is computed, so it can run further ahead
constexpr int kVStages = 2;  // V_j frees after PV_j
constexpr int kPrefetch = 3;  // K/V blocks brought into L2 this many blocks ahead of their load
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;
constexpr int kOffV = kOffK + kKStages * kTile;
constexpr int kOffStage = kOffV + kVStages * kTile;  // epilogue staging: 8 warps x 16 rows x 256 B
constexpr int kOffBar = kOffStage + kTile;
// q_full q_empty | k_full[3] k_empty[3] | v_full[2] v_empty[2] | s_full[2] s_empty[2] | p_full[2] p_empty[2]
// | o_empty done
constexpr int kNumBars = 2 + 2 * kKStages + 2 * kVStages + 4 + 4 + 2;
constexpr int kFwdSoftmaxWarps = 8;
constexpr int kFwdThreads = 64 + 32 * kFwdSoftmaxWarps;
constexpr int kSmemBytes = 1024 + kOffBar + 8 * kNumBars + 16;
constexpr uint32_t kColO = 256;
constexpr uint32_t kColP = 384;
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

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const int* __restrict__ cu,
                     const int* __restrict__ cu_k, const int2* __restrict__ tiles, int n_tiles, int Hq, int Hkv,
                     __nv_bfloat16* __restrict__ O, float* __restrict__ lse, int T, float scale_log2, int causal,
                     int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_full = v_empty + kVStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* o_empty = p_empty + 2;
  uint64_t* done = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

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
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], kFwdSoftmaxWarps);
      mbar_init(&p_full[b], kFwdSoftmaxWarps);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(o_empty, kFwdSoftmaxWarps);
    mbar_init(done, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t k_it = 0, v_it = 0, item_it = 0;
      bool q_issued = false, ok = true;
      uint32_t q_par = 0;
      uint32_t k_mask = 0, k_par = 0, v_mask = 0, v_par = 0;  // per stage: ever filled / parity of last fill
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
        if (!mbar_wait(q_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        mbar_expect_tx(q_full, kTile);
        tma_load_2d(smQ, &tmQ, q_full, it.h * D, it.s0 + it.q0);
        tma_load_2d(smQ + kChunk, &tmQ, q_full, it.h * D + 64, it.s0 + it.q0);
        q_issued = true;
        q_par = item_it & 1u;
        auto prefetch = [&](int j) {
          const int y = it.k0 + j * BKV;
          tma_prefetch_l2_2d(&tmK, it.hk * D, y);
          tma_prefetch_l2_2d(&tmK, it.hk * D + 64, y);
          tma_prefetch_l2_2d(&tmV, it.hk * D, y);
          tma_prefetch_l2_2d(&tmV, it.hk * D + 64, y);
        };
        auto load = [&](const CUtensorMap* map, uint8_t* ring, uint64_t* full, uint64_t* empty, int stages,
                        uint32_t& cnt, uint32_t& mask, uint32_t& par, int j) -> bool {
          const int st = cnt % stages;
          const uint32_t ph = (cnt / stages) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, err, kTimeoutAttnKV)) return false;
          const int y = it.k0 + j * BKV;
          mbar_expect_tx(&full[st], kTile);
          tma_load_2d(ring + st * kTile, map, &full[st], it.hk * D, y);
          tma_load_2d(ring + st * kTile + kChunk, map, &full[st], it.hk * D + 64, y);
          mask |= 1u << st;
          par = (par & ~(1u << st)) | (ph << st);
          ++cnt;
          return true;
        };
        for (int j = 0; j < it.nkv && j < kPrefetch; ++j) prefetch(j);
        if (item + (int)gridDim.x < n_items) {  // the next item's Q, so its load hits L2
          const Item nx = decode(item + gridDim.x, cu, cu_k, tiles, Hq, group, causal);
          tma_prefetch_l2_2d(&tmQ, nx.h * D, nx.s0 + nx.q0);
          tma_prefetch_l2_2d(&tmQ, nx.h * D + 64, nx.s0 + nx.q0);
        }
        // K runs one block ahead of V (the MMA order is S_{j+1} then PV_j)
        if (!load(&tmK, smK, k_full, k_empty, kKStages, k_it, k_mask, k_par, 0)) { ok = false; break; }
        for (int j = 0; j < it.nkv; ++j) {
          if (j + kPrefetch < it.nkv) prefetch(j + kPrefetch);
          if (j + 1 < it.nkv && !load(&tmK, smK, k_full, k_empty, kKStages, k_it, k_mask, k_par, j + 1)) {
            ok = false;
            break;
          }
          if (!load(&tmV, smV, v_full, v_empty, kVStages, v_it, v_mask, v_par, j)) { ok = false; break; }
        }
      }
      // drain: every copy this thread issued must land before the CTA exits
      if (q_issued) mbar_wait(q_full, q_par, nullptr, 0);
      for (int s = 0; s < kKStages; ++s)
        if ((k_mask >> s) & 1u) mbar_wait(&k_full[s], (k_par >> s) & 1u, nullptr, 0);
      for (int s = 0; s < kVStages; ++s)
        if ((v_mask >> s) & 1u) mbar_wait(&v_full[s], (v_par >> s) & 1u, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_bf16(BQ, D, 0, 1);
      const uint32_t aQ = smem_u32(smQ);
      uint32_t s_it = 0, pv_it = 0, item_it = 0;  // S MMAs = K loads, PV MMAs = V loads (CTA totals)
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++item_it) {
        const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
        if (!mbar_wait(q_full, item_it & 1u, err, kTimeoutAttnQ)) { ok = false; break; }
        tc_fence_after();
        auto issue_s = [&]() -> bool {
          const int ks = s_it % kKStages;
          if (!mbar_wait(&k_full[ks], (s_it / kKStages) & 1u, err, kTimeoutAttnKV)) return false;
          const int sb = s_it & 1;
          if (!mbar_wait(&s_empty[sb], ((s_it >> 1) & 1u) ^ 1u, err, kTimeoutAttnS)) return false;
          tc_fence_after();
          const uint32_t aK = smem_u32(smK + ks * kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16(tmem_base + sb * BKV, kmajor_desc(aQ, kk), kmajor_desc(aK, kk), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[sb]);
          umma_commit(&k_empty[ks]);
          ++s_it;
          return true;
        };
        if (!issue_s()) { ok = false; break; }
        for (int j = 0; j < it.nkv && ok; ++j) {
          if (j + 1 < it.nkv) {
            if (!issue_s()) { ok = false; break; }
          } else {
            umma_commit(q_empty);  // every S MMA of this item is issued: Q frees when they finish
          }
          const int vs = pv_it % kVStages;
          const int pb = pv_it & 1;
          if (!mbar_wait(&p_full[pb], (pv_it >> 1) & 1u, err, kTimeoutAttnP)) { ok = false; break; }
          if (!mbar_wait(&v_full[vs], (pv_it / kVStages) & 1u, err, kTimeoutAttnKV)) { ok = false; break; }
          if (j == 0 && !mbar_wait(o_empty, (item_it & 1u) ^ 1u, err, kTimeoutAttnO)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aV = smem_u32(smV + vs * kTile);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            umma_f16_ts(tmem_base + kColO, tmem_base + kColP + pb * 64 + kk * 8, mnmajor_desc(aV, kk), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&v_empty[vs]);
          umma_commit(&p_empty[pb]);
          ++pv_it;
        }
      }
      umma_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int sub = (warp - 2) >> 2;      // which 16 rows of the lane quarter
    const int rl = lane >> 2, cq = lane & 3;
    const int row0 = quarter * 32 + sub * 16 + rl;  // tile rows of this thread: row0, row0 + 8
    const uint32_t lane_addr = (uint32_t)(quarter * 32 + sub * 16) << 16;
    uint8_t* stage = smem + kOffStage + (warp - 2) * 4096;
    // Waits are made warp-uniform: the tcgen05 loads and stores that follow are
    // .sync.aligned, so either the whole warp goes on or the whole warp stops.
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
    };
    // wait until PV number g (global block count) has finished reading its P buffer
    auto pv_wait = [&](uint32_t g) -> bool { return wait_all(&p_empty[g & 1u], (g >> 1) & 1u, kTimeoutAttnPV); };
    uint32_t g = 0;  // blocks processed by this CTA (S and P buffer sequence)
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item it = decode(item, cu, cu_k, tiles, Hq, group, causal);
      const int qp0 = it.q0 + row0, qp1 = qp0 + 8;
      const int lim0 = causal ? min(it.off + qp0 + 1, it.Lk) : it.Lk;  // keys below lim are visible
      const int lim1 = causal ? min(it.off + qp1 + 1, it.Lk) : it.Lk;
      const int lim_tile = causal ? min(it.off + it.q0 + 1, it.Lk) : it.Lk;  // smallest limit in the tile
      float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
      for (int j = 0; j < it.nkv; ++j, ++g) {
        const int sb = g & 1;
        if (!wait_all(&s_full[sb], (g >> 1) & 1u, kTimeoutAttnS)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[64];
        tmem_ld_16x256b_x16(tmem_base + lane_addr + sb * BKV, r);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);
        const int kb = j * BKV + 2 * cq;
        if ((j + 1) * BKV > lim_tile) {  // block crosses the diagonal or the sequence end
#pragma unroll
          for (int i = 0; i < 16; ++i) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = kb + 8 * i + e;
              if (key >= lim0) r[4 * i + e] = __float_as_uint(-INFINITY);
              if (key >= lim1) r[4 * i + 2 + e] = __float_as_uint(-INFINITY);
            }
          }
        }
        // raw block max per row (scale > 0, so the scaled max is scale * raw max)
        float a0 = -INFINITY, a1 = -INFINITY, b0 = -INFINITY, b1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          a0 = fmaxf(a0, __uint_as_float(r[4 * i + 0]));
          b0 = fmaxf(b0, __uint_as_float(r[4 * i + 1]));
          a1 = fmaxf(a1, __uint_as_float(r[4 * i + 2]));
          b1 = fmaxf(b1, __uint_as_float(r[4 * i + 3]));
        }
        const float bm0 = quad_max(fmaxf(a0, b0)) * scale_log2;
        const float bm1 = quad_max(fmaxf(a1, b1)) * scale_log2;
        const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
        if (j == 0) {
          m0 = mn0;
          m1 = mn1;
        } else {
          const bool rs0 = mn0 > m0 + kRescaleThreshold, rs1 = mn1 > m1 + kRescaleThreshold;
          if (__any_sync(0xffffffffu, rs0 || rs1)) {
            if (!pv_wait(g - 1)) { ok = false; break; }  // O holds every earlier block
            tc_fence_after();
            const float f0 = rs0 ? ex2_approx(m0 - mn0) : 1.f;
            const float f1 = rs1 ? ex2_approx(m1 - mn1) : 1.f;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t o[32];
              tmem_ld_16x256b_x8(tmem_base + lane_addr + kColO + c * 64, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                o[4 * i + 0] = __float_as_uint(__uint_as_float(o[4 * i + 0]) * f0);
                o[4 * i + 1] = __float_as_uint(__uint_as_float(o[4 * i + 1]) * f0);
                o[4 * i + 2] = __float_as_uint(__uint_as_float(o[4 * i + 2]) * f1);
                o[4 * i + 3] = __float_as_uint(__uint_as_float(o[4 * i + 3]) * f1);
              }
              tmem_st_16x256b_x8(tmem_base + lane_addr + kColO + c * 64, o);
            }
            tmem_st_wait();
            if (rs0) {
              l0 *= f0;
              m0 = mn0;
            }
            if (rs1) {
              l1 *= f1;
              m1 = mn1;
            }
          }
        }
        // P = 2^(s * scale - m) packed to bf16 pairs, in place: r[2i] row0, r[2i+1] row1
        // (P column 4i + cq).  Group i is read before words 2i, 2i+1 are written.
        const float nm0 = -m0, nm1 = -m1;
        float s0a = 0.f, s0b = 0.f, s1a = 0.f, s1b = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            p[e] = ex2_approx(fmaf(__uint_as_float(r[4 * i + e]), scale_log2, (e < 2) ? nm0 : nm1));
          s0a += p[0];
          s0b += p[1];
          s1a += p[2];
          s1b += p[3];
          r[2 * i] = pack_bf16x2(p[0], p[1]);
          r[2 * i + 1] = pack_bf16x2(p[2], p[3]);
        }
        l0 += s0a + s0b;
        l1 += s1a + s1b;
        if (g >= 2 && !pv_wait(g - 2)) { ok = false; break; }  // P buffer sb is free again
        tc_fence_after();
        tmem_st_16x128b_x16(tmem_base + lane_addr + kColP + sb * 64, *reinterpret_cast<const uint32_t(*)[32]>(r));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      // epilogue: full row sums, then O / l through the staging area
      l0 = quad_sum(l0);
      l1 = quad_sum(l1);
      if (!pv_wait(g - 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t o[64];
      tmem_ld_16x256b_x16(tmem_base + lane_addr + kColO, o);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
      const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
      // row rl / rl + 8 of this warp's 16, 16-byte chunk i holds columns 8i..8i+7; word cq of the chunk
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t w0 = pack_bf16x2(__uint_as_float(o[4 * i + 0]) * inv0, __uint_as_float(o[4 * i + 1]) * inv0);
        const uint32_t w1 = pack_bf16x2(__uint_as_float(o[4 * i + 2]) * inv1, __uint_as_float(o[4 * i + 3]) * inv1);
        *reinterpret_cast<uint32_t*>(stage + rl * 256 + ((i ^ rl) << 4) + cq * 4) = w0;
        *reinterpret_cast<uint32_t*>(stage + (rl + 8) * 256 + ((i ^ rl) << 4) + cq * 4) = w1;
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int q = k * 32 + lane;
        const int rr = q >> 4, ch = q & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 256 + ((ch ^ (rr & 7)) << 4));
        const int qp = it.q0 + quarter * 32 + sub * 16 + rr;
        if (qp < it.L) *reinterpret_cast<uint4*>(O + ((size_t)(it.s0 + qp) * Hq + it.h) * D + ch * 8) = v;
      }
      __syncwarp();
      if (cq == 0) {
        if (qp0 < it.L) lse[(size_t)it.h * T + it.s0 + qp0] = (m0 + lg2_approx(l0)) * 0.6931471805599453f;
        if (qp1 < it.L) lse[(size_t)it.h * T + it.s0 + qp1] = (m1 + lg2_approx(l1)) * 0.6931471805599453f;
      }
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
  static bool configured[kMaxDevices] = {};  // per device: the attribute is set on the current one
  if (!configured[current_device_index()]) {
    cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    configured[current_device_index()] = true;
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

// Kernels of the rollout engine's fused decode step (one new token per
// running sequence, batch B <= a few hundred rows).
//
// At decode batch sizes every linear layer is a skinny GEMM whose cost is the
// weight read; the GEMMs run in the stream-K mode of the tcgen05 kernel
// (gemm_tcgen05.cu), which spreads the tiles x K-blocks iterations of every
// weight over all SMs and adds fp32 partial tiles into an accumulator with
// L2 reductions.  The kernels here consume those accumulators, fuse the
// elementwise work that follows each GEMM, and leave the accumulator zeroed
// for its next use (every consumer clears exactly what it read), so the step
// needs no memset:
//
//  * decode_qkv_post        acc [B, (nq + 2 nkv) D] -> bf16 round, q/k RMSNorm
//                           per head, RoPE, q -> q_out, k/v straight into the
//                           paged cache slot of the new token
//  * decode_residual_norm   x = bf16(x + acc); h = RMSNorm(x) * w
//  * decode_swiglu          a = silu(bf16(gate)) * bf16(up)
//  * decode_attention       paged decode attention, stream-K over KV blocks
//                           (see below)
//
// The bf16 rounding points match the training forward (GEMM epilogues round
// to bf16 before the norm / activation), so rollout logprobs follow the
// trainer's numerics.  Replaces the decode path inside the vLLM servers that
// the reference's rollout clients call (engine/rollout_engine.py:168-288).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.cuh"

namespace libra {
namespace decode {

constexpr int kD = 128;  // head dim

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ void ld_f32x8_zero(float* p, float (&v)[8]) {
  float4* q = reinterpret_cast<float4*>(p);
  const float4 a = __ldcg(q), b = __ldcg(q + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  __stcg(q, z);
  __stcg(q + 1, z);
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 p;
  p.x = pack_bf16x2(v[0], v[1]);
  p.y = pack_bf16x2(v[2], v[3]);
  p.z = pack_bf16x2(v[4], v[5]);
  p.w = pack_bf16x2(v[6], v[7]);
  return p;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ------------------------------------------------------------------ q/k norm + RoPE + KV write
// Same lane layout as the training kernel (norm_rope.cu): eight lanes per
// (row, head); lane j owns elements [8j, 8j+8) and [64+8j, 64+8j+8), so the
// rotate-half partner of every element is in the same thread.
__global__ void __launch_bounds__(256)
    qkv_post_kernel(float* __restrict__ acc, int ld, const __nv_bfloat16* __restrict__ qw,
                    const __nv_bfloat16* __restrict__ kw, const int* __restrict__ pos, const float* __restrict__ cos_t,
                    const float* __restrict__ sin_t, const int64_t* __restrict__ slot, __nv_bfloat16* __restrict__ q_out,
                    __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache, int B, int nq, int nkv,
                    float eps) {
  // the next kernel may start launching now: it waits for this one before reading what it writes
  pdl_launch_dependents();
  pdl_wait();
  const int heads = nq + nkv;
  const int lane = threadIdx.x & 31, grp = lane >> 3, j = lane & 7;
  const unsigned gmask = 0xFFu << (grp * 8);
  const int total = B * heads;
  const int step = gridDim.x * (blockDim.x >> 5) * 4;
  for (int item = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 + grp; item < total; item += step) {
    const int b = item / heads, h = item - b * heads;
    const bool is_q = h < nq;
    float* src = acc + (size_t)b * ld + (size_t)h * kD;
    const int i0 = 8 * j, i1 = kD / 2 + 8 * j;
    float x1[8], x2[8];
    ld_f32x8_zero(src + i0, x1);
    ld_f32x8_zero(src + i1, x2);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x1[e] = bf16_round(x1[e]);
      x2[e] = bf16_round(x2[e]);
      ss += x1[e] * x1[e] + x2[e] * x2[e];
    }
    ss += __shfl_xor_sync(gmask, ss, 4);
    ss += __shfl_xor_sync(gmask, ss, 2);
    ss += __shfl_xor_sync(gmask, ss, 1);
    const float r = rsqrtf(ss / (float)kD + eps);
    const __nv_bfloat16* wt = is_q ? qw : kw;
    float wa[8], wb[8];
    unpack8(*reinterpret_cast<const uint4*>(wt + i0), wa);
    unpack8(*reinterpret_cast<const uint4*>(wt + i1), wb);
    const int p = pos[b];
    const float4* ct = reinterpret_cast<const float4*>(cos_t + (size_t)p * (kD / 2) + i0);
    const float4* st = reinterpret_cast<const float4*>(sin_t + (size_t)p * (kD / 2) + i0);
    const float4 c0 = ct[0], c1 = ct[1], s0 = st[0], s1 = st[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // the training kernel rounds the normed value only at the end; so does this one
      const float y1 = x1[e] * r * wa[e], y2 = x2[e] * r * wb[e];
      o1[e] = y1 * c[e] - y2 * sn[e];
      o2[e] = y2 * c[e] + y1 * sn[e];
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = q_out + ((size_t)b * nq + h) * kD;
    } else {
      dst = k_cache + ((size_t)slot[b] * nkv + (h - nq)) * kD;
      float* vs = acc + (size_t)b * ld + (size_t)(nq + nkv + (h - nq)) * kD;
      float v1[8], v2[8];
      ld_f32x8_zero(vs + i0, v1);
      ld_f32x8_zero(vs + i1, v2);
      __nv_bfloat16* vd = v_cache + ((size_t)slot[b] * nkv + (h - nq)) * kD;
      *reinterpret_cast<uint4*>(vd + i0) = pack8(v1);
      *reinterpret_cast<uint4*>(vd + i1) = pack8(v2);
    }
    *reinterpret_cast<uint4*>(dst + i0) = pack8(o1);
    *reinterpret_cast<uint4*>(dst + i1) = pack8(o2);
  }
}

// ------------------------------------------------------------------ residual add + RMSNorm
// One CTA per row, 256 threads, the row in registers (H <= 256 * 8 * kVec).
constexpr int kRnThreads = 256;
constexpr int kRnVec = 4;

__global__ void __launch_bounds__(kRnThreads)
    residual_norm_kernel(__nv_bfloat16* __restrict__ x, float* __restrict__ acc, const __nv_bfloat16* __restrict__ w,
                         __nv_bfloat16* __restrict__ h_out, int H, float eps) {
  // the next kernel may start launching now: it waits for this one before reading what it writes
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  const int nvec = H >> 3;
  __nv_bfloat16* xr = x + (size_t)row * H;
  float* ar = acc + (size_t)row * H;
  float v[kRnVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRnVec; ++k) {
    const int vi = threadIdx.x + k * kRnThreads;
    if (vi < nvec) {
      float xs[8], a[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + vi * 8), xs);
      ld_f32x8_zero(ar + vi * 8, a);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[k][e] = bf16_round(a[e] + xs[e]);
        ss += v[k][e] * v[k][e];
      }
      *reinterpret_cast<uint4*>(xr + vi * 8) = pack8(v[k]);
    }
  }
  ss = warp_sum(ss);
  __shared__ float red[kRnThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRnThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int k = 0; k < kRnVec; ++k) {
    const int vi = threadIdx.x + k * kRnThreads;
    if (vi < nvec) {
      float wv[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(w + vi * 8), wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * r * wv[e];
      *reinterpret_cast<uint4*>(h_out + (size_t)row * H + vi * 8) = pack8(o);
    }
  }
}

// ------------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

__global__ void __launch_bounds__(256)
    swiglu_kernel(float* __restrict__ acc, __nv_bfloat16* __restrict__ a, int B, int F) {
  // the next kernel may start launching now: it waits for this one before reading what it writes
  pdl_launch_dependents();
  pdl_wait();
  const int per_row = F >> 3;
  const int total = B * per_row;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int b = i / per_row, c = (i - b * per_row) * 8;
    float g[8], u[8], o[8];
    ld_f32x8_zero(acc + (size_t)b * 2 * F + c, g);
    ld_f32x8_zero(acc + (size_t)b * 2 * F + F + c, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = silu_f(bf16_round(g[e])) * bf16_round(u[e]);
    *reinterpret_cast<uint4*>(a + (size_t)b * F + c) = pack8(o);
  }
}

// ------------------------------------------------------------------ paged decode attention
// Cache (per layer): k/v [num_blocks, 16, Hkv, 128] bf16.
//
// Work split (stream-K): the cache blocks of all B sequences, concatenated in
// batch order, are TB = sum_b ceil(len_b / 16) units; CTA c of the grid G
// (one per SM) takes units [c TB / G, (c + 1) TB / G).  Every CTA moves the
// same number of bytes however uneven the lengths are, and the grid does not
// depend on them, so one captured launch serves every step.  A CTA walks its
// units sequence by sequence ("segments"):
//  * a producer warp streams the K and V tiles of every block into an
//    S-stage shared-memory ring with TMA: per KV head and 64-dim half one
//    16-row x 128-byte box with the 128-byte swizzle, so the ldmatrix reads
//    below are free of bank conflicts.  A stage is refilled as soon as every
//    compute warp has arrived on its "empty" barrier; the compute warps never
//    wait for each other inside a segment;
//  * one warp per KV head runs the block on the tensor cores (mma.sync
//    m16n8k16, bf16 in, fp32 out): S = Q K^T with the head's G query rows
//    (padded to 16) as A and K as B, online softmax on the accumulator
//    fragments in the log2 domain, then O += P V with P taken straight from
//    the S fragments (the C layout of one m16n8 pair is the A layout of the
//    next m16n8k16).  Decode is bound by the KV read; the tensor cores keep
//    the arithmetic to a few instructions per 16 tokens, so the warps keep up
//    with HBM;
//  * at the end of a segment a sequence that lies inside one CTA is written
//    out directly; otherwise the CTA writes its partial (m, l, o) to
//    workspace slot c + b (unique: the CTA ranges are ordered like the
//    sequences) and bumps the sequence's counter; the CTA that brings the
//    counter to the sequence's segment count merges all partials, writes the
//    output and resets the counter for the next launch.
// Every wait is bounded; on a timeout the kernel records kTimeoutAttnKV,
// waits for its own copies in flight and returns.
constexpr int kBS = 16;
constexpr int kMaxB = 1024;
constexpr int kHalfTile = kBS * 128;  // bytes of one 16-row x 64-dim swizzled box

__device__ __forceinline__ int owner_cta(int x, int TB, int G) {
  return (int)(((long long)(x + 1) * G - 1) / TB);
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) . B(16x8, col) + D, bf16 inputs, fp32 accumulators
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Address of 16-byte chunk `c16` (0..15) of row `r` (0..15) of a head's K or V
// tile: two 64-dim boxes, each 16 rows x 128 B with the 128-byte swizzle.
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int r, int c16) {
  return base + (uint32_t)((c16 >> 3) * kHalfTile + r * 128 + (((c16 & 7) ^ (r & 7)) << 4));
}

// Named barrier over the compute warps (the producer warp does not take
// part); returns whether `pred` held in every participating thread.
__device__ __forceinline__ bool compute_bar_and(int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(nthreads)
      : "memory");
  return r != 0;
}

template <int G>
__global__ void __launch_bounds__(288, 1)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const __nv_bfloat16* __restrict__ q, const int* __restrict__ tables, int max_blocks,
                       const int* __restrict__ lens, int B, int Hkv, int S, __nv_bfloat16* __restrict__ out,
                       float* __restrict__ part_o, float* __restrict__ part_ml, int* __restrict__ counters,
                       float scale_log2, int* err) {
  static_assert(G >= 1 && G <= 8, "1 to 8 query heads per KV head");
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ncomp = 32 * Hkv;  // compute threads: one warp per KV head; warp Hkv is the producer
  const int Hq = Hkv * G;
  const uint32_t head_bytes = 2 * kHalfTile;             // one head's K (or V) tile of a block
  const uint32_t stage_bytes = 2 * Hkv * head_bytes;     // K tiles of every head, then V tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)S * stage_bytes);
  uint64_t* empty = full + 8;
  int* pre = reinterpret_cast<int*>(empty + 8);  // [B + 1]
  __shared__ int s_last;
  // the next kernel may start launching now: it waits for this one before reading what it writes
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {  // prefix sums of the per-sequence block counts
    int carry = 0;
    for (int base = 0; base < B; base += 32) {
      const int b = base + lane;
      const int nb = b < B ? (max(lens[b], 0) + kBS - 1) / kBS : 0;
      int v = nb;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (b < B) pre[b + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) pre[0] = 0;
  }
  if (tid == 0) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Hkv);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int TB = pre[B];
  const int c = blockIdx.x;
  if (c == 0) {  // sequences without any KV: zero output
    for (int b = 0; b < B; ++b)
      if (pre[b + 1] == pre[b])
        for (int i = tid; i < Hq * kD; i += blockDim.x) out[(size_t)b * Hq * kD + i] = __float2bfloat16(0.f);
  }
  // with fewer units than CTAs the extra CTAs sit out, so every working CTA has at least one unit
  const int NC = min((int)gridDim.x, TB);
  if (c >= NC) return;
  const int lo = (int)((long long)TB * c / NC), hi = (int)((long long)TB * (c + 1) / NC);
  int b0 = 0;
  {
    int l = 0, r = B - 1;
    while (l < r) {
      const int m = (l + r + 1) >> 1;
      if (pre[m] <= lo) l = m; else r = m - 1;
    }
    b0 = l;
    while (pre[b0 + 1] <= lo) ++b0;  // skip empty sequences
  }

  if (warp == Hkv) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int b = b0, it = lo;
      for (; it < hi; ++it) {
        const int st = (it - lo) % S;
        const uint32_t ph = ((it - lo) / S) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, err, kTimeoutAttnKV)) break;
        while (pre[b + 1] <= it) ++b;
        const int blk = tables[(size_t)b * max_blocks + (it - pre[b])];
        uint8_t* dst = sm + (size_t)st * stage_bytes;
        mbar_expect_tx(&full[st], stage_bytes);
        for (int hh = 0; hh < Hkv; ++hh) {
#pragma unroll
          for (int d = 0; d < 2; ++d) {
            tma_load_3d(dst + hh * head_bytes + d * kHalfTile, &tmK, &full[st], 64 * d, hh, blk * kBS);
            tma_load_3d(dst + (Hkv + hh) * head_bytes + d * kHalfTile, &tmV, &full[st], 64 * d, hh, blk * kBS);
          }
        }
      }
      // the copies of the last S units must land before the CTA exits
      for (int k = max(lo, it - S); k < it; ++k) mbar_wait(&full[(k - lo) % S], ((k - lo) / S) & 1u, nullptr, 0);
    }
    return;
  }

  // ------------------------------------------------------------ compute warps
  const int h = warp;             // this warp's KV head
  const int gid = lane >> 2, tig = lane & 3;
  const bool row_real = gid < G;  // this thread's query row (head h*G + gid) is a real head
  bool ok = true;
  int it = lo, cur_b = b0;
  while (it < hi) {
    while (pre[cur_b + 1] <= it) ++cur_b;
    const int seq_lo = pre[cur_b], seq_hi = pre[cur_b + 1];
    const int seg_end = min(hi, seq_hi);
    const int len = lens[cur_b];
    // Q fragments (A operand): row gid = query head h*G + gid, rows >= G (and 8..15) are zero
    uint32_t qa[8][2];
    {
      const __nv_bfloat16* qr = q + ((size_t)cur_b * Hq + h * G + (row_real ? gid : 0)) * kD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qa[ks][0] = row_real ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + 2 * tig) : 0u;
        qa[ks][1] = row_real ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + 8 + 2 * tig) : 0u;
      }
    }
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    for (; ok && it < seg_end; ++it) {
      const int st = (it - lo) % S;
      const uint32_t ph = ((it - lo) / S) & 1u;
      if (!mbar_wait(&full[st], ph, err, kTimeoutAttnKV)) {
        ok = false;
        break;
      }
      const uint32_t kbase = smem_u32(sm + (size_t)st * stage_bytes + h * head_bytes);
      const uint32_t vbase = kbase + Hkv * head_bytes;
      // ---- S = Q K^T: two n-tiles of 8 tokens, 8 k-steps of 16 dims
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {  // k-steps 2kp, 2kp+1
          const int mi = lane >> 3;
          uint32_t b00, b01, b10, b11;
          ldsm_x4(tile_addr(kbase, nt * 8 + (lane & 7), 4 * kp + mi), b00, b01, b10, b11);
          mma_bf16(s[nt], qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, b00, b01);
          mma_bf16(s[nt], qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, b10, b11);
        }
      }
      // ---- online softmax over this block's 16 tokens (row gid; rows 8..15 are padding)
      const int tok0 = (it - seq_lo) * kBS;
      float v[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pos = tok0 + nt * 8 + 2 * tig + e;
          v[nt * 2 + e] = pos < len ? s[nt][e] * scale_log2 : -INFINITY;
        }
      float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = v[e] == -INFINITY ? 0.f : exp2f(v[e] - m_new);
      l_run = l_run * alpha + (p[0] + p[1] + p[2] + p[3]);
      m_run = m_new;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= alpha;
        o[dt][1] *= alpha;
      }
      const uint32_t pa0 = pack_bf16x2(p[0], p[1]);  // P[gid][2tig..], tokens 0-7
      const uint32_t pa2 = pack_bf16x2(p[2], p[3]);  // tokens 8-15
      // ---- O += P V: 16 n-tiles of 8 dims
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // dim tiles 2dp, 2dp+1
        const int mi = lane >> 3;
        uint32_t b00, b01, b10, b11;
        ldsm_x4_t(tile_addr(vbase, (mi & 1) * 8 + (lane & 7), 2 * dp + (mi >> 1)), b00, b01, b10, b11);
        mma_bf16(o[2 * dp], pa0, 0u, pa2, 0u, b00, b01);
        mma_bf16(o[2 * dp + 1], pa0, 0u, pa2, 0u, b10, b11);
      }
      // this warp is done with the stage (its ldmatrix results are consumed above)
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // ---- segment end (every compute warp gets here for every segment, also after a timeout)
    if (!compute_bar_and(ncomp, ok)) break;
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    const bool whole = seq_lo >= lo && seq_hi <= hi;
    const int hq = h * G + gid;
    if (row_real) {
      if (whole) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = out + ((size_t)cur_b * Hq + hq) * kD + 2 * tig;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
          *reinterpret_cast<uint32_t*>(orow + dt * 8) = pack_bf16x2(o[dt][0] * inv, o[dt][1] * inv);
      } else {
        const size_t slot = (size_t)(c + cur_b) * Hq + hq;
        float* prow = part_o + slot * kD + 2 * tig;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt) __stcg(reinterpret_cast<float2*>(prow + dt * 8), make_float2(o[dt][0], o[dt][1]));
        if (tig == 0) __stcg(reinterpret_cast<float2*>(part_ml + slot * 2), make_float2(m_run, l_run));
      }
    }
    if (!whole) {
      __threadfence();
      compute_bar_and(ncomp, true);
      if (tid == 0) {
        const int nseg = owner_cta(seq_hi - 1, TB, NC) - owner_cta(seq_lo, TB, NC) + 1;
        const int old = atomicAdd(&counters[cur_b], 1);
        const int last = old == nseg - 1;
        if (last) counters[cur_b] = 0;
        s_last = last;
      }
      compute_bar_and(ncomp, true);
      if (s_last) {
        __threadfence();
        const int c0 = owner_cta(seq_lo, TB, NC), c1 = owner_cta(seq_hi - 1, TB, NC);
        // Merge: thread t owns items (head warp + k Hkv, dims 4 lane..) for k < G and walks the
        // partial slots CH at a time with every load of the chunk in flight before any is used
        constexpr int CH = G >= 8 ? 2 : (G >= 4 ? 4 : 8);
        float M[G], den[G];
        float4 num[G];
#pragma unroll
        for (int k = 0; k < G; ++k) {
          M[k] = -INFINITY;
          den[k] = 0.f;
          num[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        for (int cc = c0; cc <= c1; cc += CH) {
          float2 ml[G][CH];
          float4 ov[G][CH];
#pragma unroll
          for (int k = 0; k < G; ++k)
#pragma unroll
            for (int u = 0; u < CH; ++u) {
              if (cc + u <= c1) {
                const size_t slot = (size_t)(cc + u + cur_b) * Hq + warp + k * Hkv;
                ml[k][u] = __ldcg(reinterpret_cast<const float2*>(part_ml + slot * 2));
                ov[k][u] = __ldcg(reinterpret_cast<const float4*>(part_o + slot * kD) + lane);
              } else {
                ml[k][u] = make_float2(-INFINITY, 0.f);
                ov[k][u] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
#pragma unroll
          for (int k = 0; k < G; ++k) {
            float Mn = M[k];
#pragma unroll
            for (int u = 0; u < CH; ++u) Mn = fmaxf(Mn, ml[k][u].x);
            if (Mn == -INFINITY) continue;
            const float a = M[k] == -INFINITY ? 0.f : exp2f(M[k] - Mn);
            float4 acc = make_float4(num[k].x * a, num[k].y * a, num[k].z * a, num[k].w * a);
            float d = den[k] * a;
#pragma unroll
            for (int u = 0; u < CH; ++u) {
              const float w = ml[k][u].x == -INFINITY ? 0.f : exp2f(ml[k][u].x - Mn);
              acc.x = fmaf(w, ov[k][u].x, acc.x);
              acc.y = fmaf(w, ov[k][u].y, acc.y);
              acc.z = fmaf(w, ov[k][u].z, acc.z);
              acc.w = fmaf(w, ov[k][u].w, acc.w);
              d = fmaf(w, ml[k][u].y, d);
            }
            num[k] = acc;
            den[k] = d;
            M[k] = Mn;
          }
        }
#pragma unroll
        for (int k = 0; k < G; ++k) {
          const float inv = den[k] > 0.f ? 1.f / den[k] : 0.f;
          uint2 pk;
          pk.x = pack_bf16x2(num[k].x * inv, num[k].y * inv);
          pk.y = pack_bf16x2(num[k].z * inv, num[k].w * inv);
          *reinterpret_cast<uint2*>(out + ((size_t)cur_b * Hq + warp + k * Hkv) * kD + 4 * lane) = pk;
        }
      }
      compute_bar_and(ncomp, true);
    }
  }
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// 3-D map over one layer's cache [rows = blocks x 16, Hkv, 128]: box = 16 rows of one head, 64 dims
static CUtensorMap cache_map(const torch::Tensor& c) {
  const int64_t rows = c.size(0) * c.size(1), hkv = c.size(2);
  cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)hkv, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)(hkv * kD * 2)};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kBS};
  return tmap::make_bf16(c.data_ptr(), 3, dims, strides, box);
}

template <int G>
static void launch_attn(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                        const torch::Tensor& tables, const torch::Tensor& lens, int B, torch::Tensor& out,
                        torch::Tensor& part_o, torch::Tensor& part_ml, torch::Tensor& counters, int* err,
                        float scale_log2, cudaStream_t st, bool pdl) {
  const int Hkv = (int)kc.size(2);
  const int threads = 32 * (Hkv + 1);  // a warp per KV head + the producer warp
  const size_t stage_bytes = (size_t)2 * Hkv * 2 * kHalfTile;
  const size_t extra = 1024 /*alignment*/ + 128 + (size_t)(B + 1) * 4;
  // 227 KB per CTA, less a margin for the kernel's static shared memory
  constexpr size_t kMaxSmem = 226 * 1024;
  int S = (int)std::min<size_t>(8, (kMaxSmem - extra) / stage_bytes);
  LIBRA_CHECK(S >= 2, "decode_attention: %d KV heads leave room for %d pipeline stages", Hkv, S);
  const size_t smem = (size_t)S * stage_bytes + extra;
  auto kern = decode_attn_kernel<G>;
  static size_t configured_dev[kMaxDevices] = {};  // per instantiation and device: largest size set so far
  size_t& configured = configured_dev[current_device_index()];
  if (smem > configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    LIBRA_CHECK(e == cudaSuccess, "decode_attention: cannot reserve %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
    configured = smem;
  }
  const CUtensorMap tk = cache_map(kc), tv = cache_map(vc);
  launch_kernel(kern, dim3(sm_count()), dim3(threads), smem, st, pdl, tk, tv, (const __nv_bfloat16*)q.data_ptr(),
                tables.data_ptr<int>(), (int)tables.size(1), lens.data_ptr<int>(), B, Hkv, S,
                (__nv_bfloat16*)out.data_ptr(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                counters.data_ptr<int>(), scale_log2, err);
}

}  // namespace decode

// q [>=B, Hq, 128] bf16; caches [blocks, 16, Hkv, 128] bf16; block_tables [>=B, max_blocks] int32; seq_lens
// [>=B] int32 (tokens including the new one, whose KV is already in the cache); out [B, Hq, 128] bf16.
// Workspace (caller-owned, nothing is allocated, so the call can be captured in a CUDA graph):
// part_o [>= SMs + B, Hq, 128] fp32, part_ml [>= SMs + B, Hq, 2] fp32, counters [>= B] int32, zero
// before the first call (the kernel leaves them zero).  pdl: programmatic dependent launch (every
// kernel of the fused decode step waits for its predecessor with griddepcontrol.wait).
void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                      torch::Tensor counters, torch::Tensor err, double scale, bool pdl) {
  using namespace decode;
  LIBRA_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.dim() == 3 && q.is_contiguous() &&
                  q.size(2) == kD,
              "decode_attention: q must be contiguous bf16 [B, Hq, 128]");
  LIBRA_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4 && k_cache.size(1) == kBS &&
                  k_cache.size(3) == kD && k_cache.sizes() == v_cache.sizes() &&
                  k_cache.scalar_type() == at::kBFloat16 && v_cache.scalar_type() == at::kBFloat16,
              "decode_attention: contiguous bf16 caches [blocks, 16, kv_heads, 128]");
  const int B = (int)out.size(0), Hq = (int)q.size(1), Hkv = (int)k_cache.size(2);
  LIBRA_CHECK(Hkv >= 1 && Hkv <= 8 && Hq % Hkv == 0, "decode_attention: 1-8 KV heads dividing the query heads");
  LIBRA_CHECK(q.size(0) >= B && out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.dim() == 3 &&
                  out.size(1) == Hq && out.size(2) == kD,
              "decode_attention: out must be contiguous bf16 [B, Hq, 128] with B <= rows of q");
  LIBRA_CHECK(B <= kMaxB, "decode_attention: at most %d sequences per call", kMaxB);
  LIBRA_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous() && block_tables.dim() == 2 &&
                  block_tables.size(0) >= B && seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous() &&
                  seq_lens.numel() >= B,
              "decode_attention: int32 block tables [>=B, max_blocks] and lengths [>=B]");
  const int64_t slots = (int64_t)sm_count() + B;
  LIBRA_CHECK(part_o.is_contiguous() && part_o.scalar_type() == at::kFloat && part_o.numel() >= slots * Hq * kD &&
                  part_ml.is_contiguous() && part_ml.scalar_type() == at::kFloat && part_ml.numel() >= slots * Hq * 2,
              "decode_attention: workspace part_o [>= %lld, Hq, 128] / part_ml [>= %lld, Hq, 2] fp32",
              (long long)slots, (long long)slots);
  LIBRA_CHECK(counters.scalar_type() == at::kInt && counters.is_contiguous() && counters.numel() >= B,
              "decode_attention: counters int32 [>= B]");
  LIBRA_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "decode_attention: int32 error word");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const float sl2 = (float)(scale * 1.4426950408889634);  // log2(e)
  int* errp = err.data_ptr<int>();
  switch (Hq / Hkv) {
    case 1: launch_attn<1>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st, pdl); break;
    case 2: launch_attn<2>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st, pdl); break;
    case 4: launch_attn<4>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st, pdl); break;
    case 5: launch_attn<5>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st, pdl); break;
    case 8: launch_attn<8>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st, pdl); break;
    default: LIBRA_CHECK(false, "decode_attention: unsupported GQA group size %d", Hq / Hkv);
  }
}

// acc [>=B, (nq + 2 nkv) * 128] fp32 (row stride = stride(0)), read and zeroed; qw/kw [128] bf16; pos [>=B]
// int32; cos/sin [max_pos, 64] fp32; slot [>=B] int64 (cache row of the new token); q_out [B, nq, 128] bf16;
// caches [blocks, block_size, nkv, 128] bf16 receive the new token's normed+rotated K and its V.
void decode_qkv_post(torch::Tensor acc, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos, torch::Tensor cos_t,
                     torch::Tensor sin_t, torch::Tensor slot, torch::Tensor q_out, torch::Tensor k_cache,
                     torch::Tensor v_cache, double eps, bool pdl) {
  using namespace decode;
  const int B = (int)q_out.size(0), nq = (int)q_out.size(1), nkv = (int)k_cache.size(2);
  LIBRA_CHECK(q_out.is_contiguous() && q_out.scalar_type() == at::kBFloat16 && q_out.dim() == 3 && q_out.size(2) == kD,
              "decode_qkv_post: q_out bf16 [B, nq, 128]");
  LIBRA_CHECK(acc.scalar_type() == at::kFloat && acc.dim() == 2 && acc.stride(1) == 1 && acc.size(0) >= B &&
                  acc.size(1) == (int64_t)(nq + 2 * nkv) * kD && acc.stride(0) % 4 == 0,
              "decode_qkv_post: acc fp32 [>=B, (nq + 2 nkv) * 128]");
  LIBRA_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.sizes() == v_cache.sizes() &&
                  k_cache.dim() == 4 && k_cache.size(3) == kD && k_cache.scalar_type() == at::kBFloat16,
              "decode_qkv_post: contiguous bf16 caches [blocks, block_size, nkv, 128]");
  LIBRA_CHECK(pos.scalar_type() == at::kInt && pos.numel() >= B && slot.scalar_type() == at::kLong &&
                  slot.numel() >= B && cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat &&
                  cos_t.size(-1) == kD / 2 && qw.numel() == kD && kw.numel() == kD,
              "decode_qkv_post: bad pos/slot/rope/norm-weight arguments");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(acc.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int items = B * (nq + nkv);
  const int grid = (items + 31) / 32;
  launch_kernel(qkv_post_kernel, dim3(grid), dim3(256), 0, st, pdl, acc.data_ptr<float>(), (int)acc.stride(0),
                (const __nv_bfloat16*)qw.data_ptr(), (const __nv_bfloat16*)kw.data_ptr(), pos.data_ptr<int>(),
                cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), slot.data_ptr<int64_t>(),
                (__nv_bfloat16*)q_out.data_ptr(), (__nv_bfloat16*)k_cache.data_ptr(),
                (__nv_bfloat16*)v_cache.data_ptr(), B, nq, nkv, (float)eps);
}

// x [B, H] bf16 (updated in place: x = bf16(x + acc)); acc [>=B, H] fp32 read and zeroed; w [H] bf16;
// h_out [B, H] bf16 = RMSNorm(x) * w.  H % 8 == 0, H <= 8192.
void decode_residual_norm(torch::Tensor x, torch::Tensor acc, torch::Tensor w, torch::Tensor h_out, double eps,
                          bool pdl) {
  using namespace decode;
  const int B = (int)x.size(0), H = (int)x.size(1);
  LIBRA_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16 && h_out.is_contiguous() &&
                  h_out.scalar_type() == at::kBFloat16 && h_out.sizes() == x.sizes(),
              "decode_residual_norm: x / h_out contiguous bf16 [B, H]");
  LIBRA_CHECK(acc.is_contiguous() && acc.scalar_type() == at::kFloat && acc.size(0) >= B && acc.size(1) == H,
              "decode_residual_norm: acc contiguous fp32 [>=B, H]");
  LIBRA_CHECK(H % 8 == 0 && H <= kRnThreads * 8 * kRnVec && w.numel() == H,
              "decode_residual_norm: H must be a multiple of 8 and at most %d", kRnThreads * 8 * kRnVec);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  launch_kernel(residual_norm_kernel, dim3(B), dim3(kRnThreads), 0, st, pdl, (__nv_bfloat16*)x.data_ptr(),
                acc.data_ptr<float>(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)h_out.data_ptr(), H,
                (float)eps);
}

// acc [>=B, 2F] fp32 (gate columns then up columns), read and zeroed; a [B, F] bf16.
void decode_swiglu(torch::Tensor acc, torch::Tensor a, bool pdl) {
  using namespace decode;
  const int B = (int)a.size(0), F = (int)a.size(1);
  LIBRA_CHECK(a.is_contiguous() && a.scalar_type() == at::kBFloat16 && F % 8 == 0,
              "decode_swiglu: a contiguous bf16 [B, F], F % 8 == 0");
  LIBRA_CHECK(acc.is_contiguous() && acc.scalar_type() == at::kFloat && acc.size(0) >= B && acc.size(1) == 2 * F,
              "decode_swiglu: acc contiguous fp32 [>=B, 2F]");
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int total = B * (F / 8);
  const int grid = std::min((total + 255) / 256, sm_count() * 8);
  launch_kernel(swiglu_kernel, dim3(grid), dim3(256), 0, st, pdl, acc.data_ptr<float>(), (__nv_bfloat16*)a.data_ptr(),
                B, F);
}

}  // namespace libra

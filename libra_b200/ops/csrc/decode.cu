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
// Cache (per layer): k/v [num_blocks, 16, Hkv, 128] bf16, so one cache block
// of one layer is a contiguous 16 * Hkv * 256-byte run for K and one for V.
//
// Work split (stream-K): the cache blocks of all B sequences, concatenated in
// batch order, are TB = sum_b ceil(len_b / 16) units; CTA c of the grid G
// (one per SM) takes units [c TB / G, (c + 1) TB / G).  Every CTA moves the
// same number of bytes however uneven the lengths are, and the grid does not
// depend on them, so one captured launch serves every step.  A CTA walks its
// units sequence by sequence ("segments"):
//  * one thread streams whole K and V blocks into an S-stage shared-memory
//    ring with cp.async.bulk (mbarrier completion);
//  * two warps per KV head, each scoring 8 tokens of every block for the G
//    query heads of that KV head: lane l owns dims [4l, 4l+4), scores are
//    reduced across the warp with a reduce-scatter butterfly (each level
//    halves the values a lane holds), online softmax in the log2 domain;
//  * at the end of a segment the two warps of a head merge their states; a
//    sequence that lies inside one CTA is written out directly, otherwise the
//    CTA writes its partial (m, l, o) to workspace slot c + b (unique: the CTA
//    ranges are ordered like the sequences) and bumps the sequence's counter;
//    the CTA that brings the counter to the sequence's segment count merges
//    all partials, writes the output and resets the counter for the next
//    launch.
// Every wait is bounded; on a timeout the kernel records kTimeoutAttnKV,
// waits for its own copies in flight and returns.
constexpr int kBS = 16;
constexpr int kMaxB = 1024;
constexpr int kComb = 132;  // per (KV head, query head) merge record: m, l, 2 pad, o[128]; 16-byte multiple

template <int N, int O>
__device__ __forceinline__ void rs_level(float* v, int lane) {
  if constexpr (O >= 1) {
    if constexpr (N > 1) {
      const bool up = (lane & O) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        const float send = up ? v[i] : v[i + N / 2];
        const float keep = up ? v[i + N / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
      }
      rs_level<N / 2, O / 2>(v, lane);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
      rs_level<1, O / 2>(v, lane);
    }
  }
}

__device__ __forceinline__ int owner_cta(int x, int TB, int G) {
  return (int)(((long long)(x + 1) * G - 1) / TB);
}

template <int G>
__global__ void __launch_bounds__(512, 1)
    decode_attn_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, const int* __restrict__ tables, int max_blocks,
                       const int* __restrict__ lens, int B, int Hkv, int S, __nv_bfloat16* __restrict__ out,
                       float* __restrict__ part_o, float* __restrict__ part_ml, int* __restrict__ counters,
                       float scale_log2, int* err) {
  constexpr int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
  constexpr int NV = 8 * GP;                  // scores per lane before the reduction
  constexpr int V = NV >= 32 ? NV / 32 : 1;  // after it
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int Hq = Hkv * G;
  const int row_el = Hkv * kD;                  // elements per token row of the cache
  const uint32_t blk_bytes = kBS * row_el * 2;  // one K (or V) block
  const uint32_t stage_bytes = 2 * blk_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)S * stage_bytes);
  int* pre = reinterpret_cast<int*>(full + 8);                      // [B + 1]
  float* p_all = reinterpret_cast<float*>(pre + ((B + 1 + 3) & ~3));  // [warps][9][GP]
  __shared__ int s_last;

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
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int TB = pre[B];
  const int c = blockIdx.x;
  if (c == 0) {  // sequences without any KV: zero output
    for (int b = 0; b < B; ++b)
      if (pre[b + 1] == pre[b])
        for (int i = tid; i < Hq * kD; i += nthreads) out[(size_t)b * Hq * kD + i] = __float2bfloat16(0.f);
  }
  // with fewer units than CTAs the extra CTAs sit out, so every working CTA has at least one unit
  const int NC = min((int)gridDim.x, TB);
  if (c >= NC) return;
  const int lo = (int)((long long)TB * c / NC), hi = (int)((long long)TB * (c + 1) / NC);
  // first sequence of this range: the largest b with pre[b] <= lo
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
  // ---- producer state (thread 0)
  int ld_it = lo, ld_b = b0;
  auto issue = [&](int it) {
    while (pre[ld_b + 1] <= it) ++ld_b;
    const int j = it - pre[ld_b];
    const int blk = tables[(size_t)ld_b * max_blocks + j];
    const int st = (it - lo) % S;
    uint8_t* dst = sm + (size_t)st * stage_bytes;
    mbar_expect_tx(&full[st], stage_bytes);
    bulk_load(dst, kc + (size_t)blk * kBS * row_el, blk_bytes, &full[st]);
    bulk_load(dst + blk_bytes, vc + (size_t)blk * kBS * row_el, blk_bytes, &full[st]);
  };
  if (tid == 0)
    for (; ld_it < hi && ld_it < lo + S; ++ld_it) issue(ld_it);

  const int h = warp >> 1, half = warp & 1;
  float* p_s = p_all + warp * 9 * GP;
  bool aborted = false;
  int it = lo, cur_b = b0;
  while (it < hi) {
    while (pre[cur_b + 1] <= it) ++cur_b;
    const int seq_lo = pre[cur_b], seq_hi = pre[cur_b + 1];
    const int seg_end = min(hi, seq_hi);
    const int len = lens[cur_b];
    // this warp's query heads, this lane's four dims, in log2 units
    float qr[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint2 u = *reinterpret_cast<const uint2*>(q + ((size_t)cur_b * Hq + h * G + g) * kD + 4 * lane);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 bq = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      qr[g][0] = a.x * scale_log2;
      qr[g][1] = a.y * scale_log2;
      qr[g][2] = bq.x * scale_log2;
      qr[g][3] = bq.y * scale_log2;
    }
    float m_run[V], l_run[V], o[G][4];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      m_run[j] = -INFINITY;
      l_run[j] = 0.f;
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[g][e] = 0.f;
    for (; it < seg_end; ++it) {
      const int st = (it - lo) % S;
      const uint32_t ph = ((it - lo) / S) & 1u;
      const bool ok = mbar_wait(&full[st], ph, err, kTimeoutAttnKV);
      if (!__syncthreads_and(ok)) {
        aborted = true;
        break;
      }
      // every warp is done with block it-1: its stage takes block it-1+S
      if (tid == 0 && it > lo && ld_it < hi) issue(ld_it++);
      if (h < Hkv) {
        const __nv_bfloat16* Ks = reinterpret_cast<const __nv_bfloat16*>(sm + (size_t)st * stage_bytes) +
                                  (size_t)(half * 8) * row_el + h * kD + 4 * lane;
        const __nv_bfloat16* Vs = Ks + kBS * row_el;
        float sc[NV];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const uint2 u = *reinterpret_cast<const uint2*>(Ks + (size_t)t * row_el);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 bb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            if (g < G) {
              float acc = qr[g][0] * a.x;
              acc = fmaf(qr[g][1], a.y, acc);
              acc = fmaf(qr[g][2], bb.x, acc);
              acc = fmaf(qr[g][3], bb.y, acc);
              sc[t * GP + g] = acc;
            } else {
              sc[t * GP + g] = 0.f;
            }
          }
        }
        rs_level<NV, 16>(sc, lane);
        // lane holds token t = lane / 4 of this half; its values belong to heads gidx(j)
        const int t = lane >> 2;
        const int pos = (it - seq_lo) * kBS + half * 8 + t;
        const bool valid = pos < len;
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const int g = GP >= 4 ? (lane & 3) * (GP / 4) + j : (GP == 2 ? (lane >> 1) & 1 : 0);
          const float s = valid ? sc[j] : -INFINITY;
          float mx = s;
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m_run[j], mx);
          const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run[j] - m_new);
          const float p = s == -INFINITY ? 0.f : exp2f(s - m_new);
          float ps = p;
          ps += __shfl_xor_sync(0xffffffffu, ps, 4);
          ps += __shfl_xor_sync(0xffffffffu, ps, 8);
          ps += __shfl_xor_sync(0xffffffffu, ps, 16);
          l_run[j] = l_run[j] * alpha + ps;
          m_run[j] = m_new;
          p_s[t * GP + g] = p;
          if (t == 0) p_s[8 * GP + g] = alpha;
        }
        __syncwarp();
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float a = p_s[8 * GP + g];
#pragma unroll
          for (int e = 0; e < 4; ++e) o[g][e] *= a;
        }
#pragma unroll
        for (int tt = 0; tt < 8; ++tt) {
          const uint2 u = *reinterpret_cast<const uint2*>(Vs + (size_t)tt * row_el);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
          const float2 bb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
          float pr[GP];
#pragma unroll
          for (int g4 = 0; g4 < GP; g4 += (GP >= 4 ? 4 : GP)) {
            if constexpr (GP >= 4) {
              const float4 f = *reinterpret_cast<const float4*>(p_s + tt * GP + g4);
              pr[g4] = f.x;
              pr[g4 + 1] = f.y;
              pr[g4 + 2] = f.z;
              pr[g4 + 3] = f.w;
            } else {
#pragma unroll
              for (int g = 0; g < GP; ++g) pr[g] = p_s[tt * GP + g];
            }
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            o[g][0] = fmaf(pr[g], a.x, o[g][0]);
            o[g][1] = fmaf(pr[g], a.y, o[g][1]);
            o[g][2] = fmaf(pr[g], bb.x, o[g][2]);
            o[g][3] = fmaf(pr[g], bb.y, o[g][3]);
          }
        }
        __syncwarp();
      }
    }
    if (aborted) break;
    // ---- segment end: merge the two warps of every head through the stage of the last block
    __syncthreads();
    float* comb = reinterpret_cast<float*>(sm + (size_t)((it - 1 - lo) % S) * stage_bytes);  // [Hkv][G][kComb]
    float mh[G], lh[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int src = GP >= 4 ? g / (GP / 4) : (GP == 2 ? 2 * g : 0);
      const int j = GP >= 4 ? g % (GP / 4) : 0;
      float mv = 0.f, lv = 0.f;
#pragma unroll
      for (int jj = 0; jj < V; ++jj)
        if (jj == j) {
          mv = m_run[jj];
          lv = l_run[jj];
        }
      mh[g] = __shfl_sync(0xffffffffu, mv, src);
      lh[g] = __shfl_sync(0xffffffffu, lv, src);
    }
    if (h < Hkv && half == 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float* cg = comb + ((size_t)h * G + g) * kComb;
        *reinterpret_cast<float4*>(cg + 4 + 4 * lane) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
        if (lane == 0) {
          cg[0] = mh[g];
          cg[1] = lh[g];
        }
      }
    }
    __syncthreads();
    const bool whole = seq_lo >= lo && seq_hi <= hi;
    if (h < Hkv && half == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float* cg = comb + ((size_t)h * G + g) * kComb;
        const float m1 = cg[0], l1 = cg[1];
        const float4 o1 = *reinterpret_cast<const float4*>(cg + 4 + 4 * lane);
        const float M = fmaxf(mh[g], m1);
        const float a0 = mh[g] == -INFINITY ? 0.f : exp2f(mh[g] - M);
        const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - M);
        const float L = lh[g] * a0 + l1 * a1;
        float r[4] = {o[g][0] * a0 + o1.x * a1, o[g][1] * a0 + o1.y * a1, o[g][2] * a0 + o1.z * a1,
                      o[g][3] * a0 + o1.w * a1};
        const int hq = h * G + g;
        if (whole) {
          const float inv = L > 0.f ? 1.f / L : 0.f;
          uint2 pk;
          pk.x = pack_bf16x2(r[0] * inv, r[1] * inv);
          pk.y = pack_bf16x2(r[2] * inv, r[3] * inv);
          *reinterpret_cast<uint2*>(out + ((size_t)cur_b * Hq + hq) * kD + 4 * lane) = pk;
        } else {
          const size_t slot = (size_t)(c + cur_b) * Hq + hq;
          __stcg(reinterpret_cast<float4*>(part_o + slot * kD + 4 * lane), make_float4(r[0], r[1], r[2], r[3]));
          if (lane == 0) __stcg(reinterpret_cast<float2*>(part_ml + slot * 2), make_float2(M, L));
        }
      }
    }
    if (!whole) {
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const int nseg = owner_cta(seq_hi - 1, TB, NC) - owner_cta(seq_lo, TB, NC) + 1;
        const int old = atomicAdd(&counters[cur_b], 1);
        const int last = old == nseg - 1;
        if (last) counters[cur_b] = 0;
        s_last = last;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        const int c0 = owner_cta(seq_lo, TB, NC), c1 = owner_cta(seq_hi - 1, TB, NC);
        for (int i = tid; i < Hq * (kD / 4); i += nthreads) {
          const int hq = i / (kD / 4), d4 = i - hq * (kD / 4);
          float M = -INFINITY;
          for (int cc = c0; cc <= c1; ++cc)
            M = fmaxf(M, __ldcg(part_ml + ((size_t)(cc + cur_b) * Hq + hq) * 2));
          float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
          float den = 0.f;
          for (int cc = c0; cc <= c1; ++cc) {
            const size_t slot = (size_t)(cc + cur_b) * Hq + hq;
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml + slot * 2));
            if (ml.x == -INFINITY) continue;
            const float w = exp2f(ml.x - M);
            const float4 ov = __ldcg(reinterpret_cast<const float4*>(part_o + slot * kD) + d4);
            num.x = fmaf(w, ov.x, num.x);
            num.y = fmaf(w, ov.y, num.y);
            num.z = fmaf(w, ov.z, num.z);
            num.w = fmaf(w, ov.w, num.w);
            den = fmaf(w, ml.y, den);
          }
          const float inv = den > 0.f ? 1.f / den : 0.f;
          uint2 pk;
          pk.x = pack_bf16x2(num.x * inv, num.y * inv);
          pk.y = pack_bf16x2(num.z * inv, num.w * inv);
          *reinterpret_cast<uint2*>(out + ((size_t)cur_b * Hq + hq) * kD + 4 * d4) = pk;
        }
      }
    }
    __syncthreads();  // the merge area (a stage) and p_s are free again
  }
  if (aborted && tid == 0) {
    // copies issued for units [it, ld_it) may still be in flight
    for (int k = it; k < ld_it; ++k) mbar_wait(&full[(k - lo) % S], ((k - lo) / S) & 1u, nullptr, 0);
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

template <int G>
static void launch_attn(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                        const torch::Tensor& tables, const torch::Tensor& lens, int B, torch::Tensor& out,
                        torch::Tensor& part_o, torch::Tensor& part_ml, torch::Tensor& counters, int* err,
                        float scale_log2, cudaStream_t st) {
  constexpr int GP = G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8;
  const int Hkv = (int)kc.size(2);
  const int threads = 64 * Hkv;
  const size_t stage_bytes = (size_t)2 * kBS * Hkv * kD * 2;
  const size_t extra = 64 + (size_t)((B + 1 + 3) & ~3) * 4 + (size_t)(threads / 32) * 9 * GP * 4;
  // 227 KB per CTA, less a margin for the kernel's static shared memory
  constexpr size_t kMaxSmem = 226 * 1024;
  int S = (int)std::min<size_t>(8, (kMaxSmem - extra) / stage_bytes);
  LIBRA_CHECK(S >= 2, "decode_attention: %d KV heads leave room for %d pipeline stages", Hkv, S);
  const size_t smem = (size_t)S * stage_bytes + extra;
  auto kern = decode_attn_kernel<G>;
  static size_t configured = 0;  // one per instantiation: the largest dynamic size set so far
  if (smem > configured) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    LIBRA_CHECK(e == cudaSuccess, "decode_attention: cannot reserve %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
    configured = smem;
  }
  kern<<<sm_count(), threads, smem, st>>>(
      (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)kc.data_ptr(), (const __nv_bfloat16*)vc.data_ptr(),
      tables.data_ptr<int>(), (int)tables.size(1), lens.data_ptr<int>(), B, Hkv, S,
      (__nv_bfloat16*)out.data_ptr(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(), counters.data_ptr<int>(),
      scale_log2, err);
  LIBRA_LAUNCH_CHECK();
}

}  // namespace decode

// q [>=B, Hq, 128] bf16; caches [blocks, 16, Hkv, 128] bf16; block_tables [>=B, max_blocks] int32; seq_lens
// [>=B] int32 (tokens including the new one, whose KV is already in the cache); out [B, Hq, 128] bf16.
// Workspace (caller-owned, nothing is allocated, so the call can be captured in a CUDA graph):
// part_o [>= SMs + B, Hq, 128] fp32, part_ml [>= SMs + B, Hq, 2] fp32, counters [>= B] int32, zero
// before the first call (the kernel leaves them zero).
void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                      torch::Tensor counters, torch::Tensor err, double scale) {
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
    case 1: launch_attn<1>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st); break;
    case 2: launch_attn<2>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st); break;
    case 4: launch_attn<4>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st); break;
    case 5: launch_attn<5>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st); break;
    case 8: launch_attn<8>(q, k_cache, v_cache, block_tables, seq_lens, B, out, part_o, part_ml, counters, errp, sl2, st); break;
    default: LIBRA_CHECK(false, "decode_attention: unsupported GQA group size %d", Hq / Hkv);
  }
}

// acc [>=B, (nq + 2 nkv) * 128] fp32 (row stride = stride(0)), read and zeroed; qw/kw [128] bf16; pos [>=B]
// int32; cos/sin [max_pos, 64] fp32; slot [>=B] int64 (cache row of the new token); q_out [B, nq, 128] bf16;
// caches [blocks, block_size, nkv, 128] bf16 receive the new token's normed+rotated K and its V.
void decode_qkv_post(torch::Tensor acc, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos, torch::Tensor cos_t,
                     torch::Tensor sin_t, torch::Tensor slot, torch::Tensor q_out, torch::Tensor k_cache,
                     torch::Tensor v_cache, double eps) {
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
  qkv_post_kernel<<<grid, 256, 0, st>>>(acc.data_ptr<float>(), (int)acc.stride(0),
                                        (const __nv_bfloat16*)qw.data_ptr(), (const __nv_bfloat16*)kw.data_ptr(),
                                        pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                        slot.data_ptr<int64_t>(), (__nv_bfloat16*)q_out.data_ptr(),
                                        (__nv_bfloat16*)k_cache.data_ptr(), (__nv_bfloat16*)v_cache.data_ptr(), B, nq,
                                        nkv, (float)eps);
  LIBRA_LAUNCH_CHECK();
}

// x [B, H] bf16 (updated in place: x = bf16(x + acc)); acc [>=B, H] fp32 read and zeroed; w [H] bf16;
// h_out [B, H] bf16 = RMSNorm(x) * w.  H % 8 == 0, H <= 8192.
void decode_residual_norm(torch::Tensor x, torch::Tensor acc, torch::Tensor w, torch::Tensor h_out, double eps) {
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
  residual_norm_kernel<<<B, kRnThreads, 0, st>>>((__nv_bfloat16*)x.data_ptr(), acc.data_ptr<float>(),
                                                 (const __nv_bfloat16*)w.data_ptr(),
                                                 (__nv_bfloat16*)h_out.data_ptr(), H, (float)eps);
  LIBRA_LAUNCH_CHECK();
}

// acc [>=B, 2F] fp32 (gate columns then up columns), read and zeroed; a [B, F] bf16.
void decode_swiglu(torch::Tensor acc, torch::Tensor a) {
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
  swiglu_kernel<<<grid, 256, 0, st>>>(acc.data_ptr<float>(), (__nv_bfloat16*)a.data_ptr(), B, F);
  LIBRA_LAUNCH_CHECK();
}

}  // namespace libra

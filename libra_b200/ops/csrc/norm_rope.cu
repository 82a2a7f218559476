// RMSNorm (forward/backward) and the fused per-head q/k RMSNorm + rotary
// embedding of the Qwen3 attention block (reference call sites: Megatron-Core
// TorchSequenceParallelNorm and q/k layernorm + RoPE, engine/megatron_core_attention.py:461-489).
//
// Layout conventions (all row-major, bf16 activations, fp32 statistics):
//   x       [T, H]
//   qkv     [T, (nq + 2 nkv) * D]   (output of the fused QKV projection)
//   cos/sin [P, D/2] fp32 tables built on the host in double precision.
// Weight gradients are reduced in two stages: every CTA keeps fp32 partial
// sums in registers for the columns it owns and writes one row of a
// [grid, H] buffer; `colsum_kernel` folds those rows.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdio>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "libra_noalloc.h"

namespace libra {

// ------------------------------------------------------------------ RMSNorm fwd
// One warp per row; each lane walks 8-element (16-byte) vectors.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int T, int H, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  const int nvec = H >> 3;
  float ss = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    uint4 u = xr[v];
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float f = __bfloat162float(b[e]);
      ss += f * f;
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)H + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = rstd;
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * H);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  for (int v = lane; v < nvec; v += 32) {
    uint4 u = xr[v], wu = wr[v];
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
    const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __bfloat162float(b[e]) * rstd * __bfloat162float(wb[e]);
    uint4 pk;
    pk.x = pack_bf16x2(o[0], o[1]);
    pk.y = pack_bf16x2(o[2], o[3]);
    pk.z = pack_bf16x2(o[4], o[5]);
    pk.w = pack_bf16x2(o[6], o[7]);
    yr[v] = pk;
  }
}

// ------------------------------------------------------------------ RMSNorm bwd
// One warp per row (grid-stride over rows); lane l owns the 8-element vectors
// l, l+32, ...  The row is read twice: pass 1 forms sum(dy*w*xhat), pass 2
// (L1 hits) writes dx and adds dy*xhat into this warp's fp32 row of shared
// memory.  At the end the CTA folds its warps' rows into one row of the
// [grid, H] partial buffer, which `colsum_kernel` then reduces over CTAs.
// Every partial row is written by its CTA, so the buffer needs no zeroing.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int T, int H,
                                   int accumulate_dx) {
  extern __shared__ float s_dw[];  // [warps, H]
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = H >> 3;
  for (int i = threadIdx.x; i < warps * H; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  float* my = s_dw + (size_t)warp * H;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (int row = blockIdx.x * warps + warp; row < T; row += gridDim.x * warps) {
    const float r = rstd[row];
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * H);
    float dot = 0.f;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      uint4 xu = xr[v], gu = gr[v], wu = __ldg(wv + v);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xu);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gu);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += __bfloat162float(gb[e]) * __bfloat162float(wb[e]) * __bfloat162float(xb[e]);
    }
    const float mean = warp_sum(dot) * r / (float)H;
    uint4* dxr = reinterpret_cast<uint4*>(dx + (size_t)row * H);
#pragma unroll 2
    for (int v = lane; v < nvec; v += 32) {
      uint4 xu = xr[v], gu = gr[v], wu = __ldg(wv + v);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xu);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gu);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
      float o[8];
      float4* acc = reinterpret_cast<float4*>(my + v * 8);
      float4 a0 = acc[0], a1 = acc[1];
      float* af0 = reinterpret_cast<float*>(&a0);
      float* af1 = reinterpret_cast<float*>(&a1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xh = __bfloat162float(xb[e]) * r;
        const float g = __bfloat162float(gb[e]);
        o[e] = r * (g * __bfloat162float(wb[e]) - xh * mean);
        if (e < 4) af0[e] += g * xh; else af1[e - 4] += g * xh;
      }
      acc[0] = a0;
      acc[1] = a1;
      if (accumulate_dx) {
        uint4 prev = dxr[v];
        const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&prev);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] += __bfloat162float(pb[e]);
      }
      uint4 pk;
      pk.x = pack_bf16x2(o[0], o[1]);
      pk.y = pack_bf16x2(o[2], o[3]);
      pk.z = pack_bf16x2(o[4], o[5]);
      pk.w = pack_bf16x2(o[6], o[7]);
      dxr[v] = pk;
    }
  }
  __syncthreads();
  float* part = dw_part + (size_t)blockIdx.x * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float sum = 0.f;
    for (int k = 0; k < warps; ++k) sum += s_dw[(size_t)k * H + c];
    part[c] = sum;
  }
}

// Same contract as rmsnorm_bwd_kernel for rows of up to 32 * 8 * kVPL
// elements: the lane's kVPL vectors of x and dy (and of the dx being
// accumulated into) are loaded once, all in flight together, and both passes
// run from registers.
template <int kVPL>
__global__ void __launch_bounds__(256) rmsnorm_bwd_reg_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int T, int H,
    int accumulate_dx) {
  extern __shared__ float s_dw[];  // [warps, H]
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = H >> 3;
  for (int i = threadIdx.x; i < warps * H; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  float* my = s_dw + (size_t)warp * H;
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (int row = blockIdx.x * warps + warp; row < T; row += gridDim.x * warps) {
    const float r = rstd[row];
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (size_t)row * H);
    uint4* dxr = reinterpret_cast<uint4*>(dx + (size_t)row * H);
    uint4 xu[kVPL], gu[kVPL], pu[kVPL];
#pragma unroll
    for (int i = 0; i < kVPL; ++i) {
      const int v = lane + 32 * i;
      if (v < nvec) {
        xu[i] = xr[v];
        gu[i] = gr[v];
        if (accumulate_dx) pu[i] = dxr[v];
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kVPL; ++i) {
      const int v = lane + 32 * i;
      if (v >= nvec) break;
      const uint4 wu = __ldg(wv + v);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xu[i]);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gu[i]);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += __bfloat162float(gb[e]) * __bfloat162float(wb[e]) * __bfloat162float(xb[e]);
    }
    const float mean = warp_sum(dot) * r / (float)H;
#pragma unroll
    for (int i = 0; i < kVPL; ++i) {
      const int v = lane + 32 * i;
      if (v >= nvec) break;
      const uint4 wu = __ldg(wv + v);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xu[i]);
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gu[i]);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wu);
      const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&pu[i]);
      float o[8];
      float4* acc = reinterpret_cast<float4*>(my + v * 8);
      float4 a0 = acc[0], a1 = acc[1];
      float* af0 = reinterpret_cast<float*>(&a0);
      float* af1 = reinterpret_cast<float*>(&a1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xh = __bfloat162float(xb[e]) * r;
        const float g = __bfloat162float(gb[e]);
        o[e] = r * (g * __bfloat162float(wb[e]) - xh * mean);
        if (accumulate_dx) o[e] += __bfloat162float(pb[e]);
        if (e < 4) af0[e] += g * xh; else af1[e - 4] += g * xh;
      }
      acc[0] = a0;
      acc[1] = a1;
      uint4 pk;
      pk.x = pack_bf16x2(o[0], o[1]);
      pk.y = pack_bf16x2(o[2], o[3]);
      pk.z = pack_bf16x2(o[4], o[5]);
      pk.w = pack_bf16x2(o[6], o[7]);
      dxr[v] = pk;
    }
  }
  __syncthreads();
  float* part = dw_part + (size_t)blockIdx.x * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float sum = 0.f;
    for (int k = 0; k < warps; ++k) sum += s_dw[(size_t)k * H + c];
    part[c] = sum;
  }
}

// out[c] (+)= sum_r part[r, c].  Block (32 columns x 8 row groups); each
// thread keeps four independent partial sums, then the 8 groups are folded
// through shared memory.
constexpr int kColsumRowGroups = 8;
__global__ void colsum_kernel(const float* __restrict__ part, int rows, int cols, float* __restrict__ out,
                              int accumulate) {
  __shared__ float red[kColsumRowGroups][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (c < cols) {
    int r = threadIdx.y;
    const int step = kColsumRowGroups;
    for (; r + 3 * step < rows; r += 4 * step) {
      s0 += part[(size_t)r * cols + c];
      s1 += part[(size_t)(r + step) * cols + c];
      s2 += part[(size_t)(r + 2 * step) * cols + c];
      s3 += part[(size_t)(r + 3 * step) * cols + c];
    }
    for (; r < rows; r += step) s0 += part[(size_t)r * cols + c];
  }
  red[threadIdx.y][threadIdx.x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kColsumRowGroups; ++k) s += red[k][threadIdx.x];
    out[c] = accumulate ? out[c] + s : s;
  }
}

static inline void launch_colsum(const float* part, int rows, int cols, float* out, bool accumulate,
                                 cudaStream_t st) {
  colsum_kernel<<<(cols + 31) / 32, dim3(32, kColsumRowGroups), 0, st>>>(part, rows, cols, out, accumulate ? 1 : 0);
}

// ------------------------------------------------------------------ q/k norm + RoPE
// Eight lanes per (token, head), four heads per warp: lane j of a group owns
// elements [8j, 8j+8) and [64+8j, 64+8j+8) of the 128-wide head, so the
// rotate-half partner of every element sits in the same thread, every global
// access is 16 bytes, and the head's sum of squares reduces over the group
// with three shuffles.  Grid-stride over (token, head) items.
template <int D>
__global__ void __launch_bounds__(256)
    qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
                            const __nv_bfloat16* __restrict__ kw, const int* __restrict__ pos,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out,
                            __nv_bfloat16* __restrict__ v_out, float* __restrict__ rstd_out, int T, int nq, int nkv,
                            float eps) {
  static_assert(D == 128, "head_dim 128");
  const int heads = nq + nkv;
  const int lane = threadIdx.x & 31, grp = lane >> 3, j = lane & 7;
  const unsigned gmask = 0xFFu << (grp * 8);
  const int stride_row = (nq + 2 * nkv) * D;
  // Item counts stay below 2^31 (checked on the host), so the (token, head) split is a 32-bit division.
  const int total = T * heads;
  const int step = gridDim.x * (blockDim.x >> 5) * 4;
  for (int item = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 + grp; item < total; item += step) {
    const int t = item / heads, h = item - t * heads;
    const bool is_q = h < nq;
    const __nv_bfloat16* src = qkv + (size_t)t * stride_row + (size_t)h * D;
    const int i0 = 8 * j, i1 = D / 2 + 8 * j;
    const uint4 xa = *reinterpret_cast<const uint4*>(src + i0);
    const uint4 xb = *reinterpret_cast<const uint4*>(src + i1);
    const __nv_bfloat16* wt = is_q ? qw : kw;
    const uint4 wa = *reinterpret_cast<const uint4*>(wt + i0);
    const uint4 wb = *reinterpret_cast<const uint4*>(wt + i1);
    const int p = pos[t];
    const float4* ct = reinterpret_cast<const float4*>(cos_t + (size_t)p * (D / 2) + i0);
    const float4* st = reinterpret_cast<const float4*>(sin_t + (size_t)p * (D / 2) + i0);
    const float4 c0 = ct[0], c1 = ct[1], s0 = st[0], s1 = st[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const __nv_bfloat16* xav = reinterpret_cast<const __nv_bfloat16*>(&xa);
    const __nv_bfloat16* xbv = reinterpret_cast<const __nv_bfloat16*>(&xb);
    const __nv_bfloat16* wav = reinterpret_cast<const __nv_bfloat16*>(&wa);
    const __nv_bfloat16* wbv = reinterpret_cast<const __nv_bfloat16*>(&wb);
    float x1[8], x2[8], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x1[e] = __bfloat162float(xav[e]);
      x2[e] = __bfloat162float(xbv[e]);
      ss += x1[e] * x1[e] + x2[e] * x2[e];
    }
    ss += __shfl_xor_sync(gmask, ss, 4);
    ss += __shfl_xor_sync(gmask, ss, 2);
    ss += __shfl_xor_sync(gmask, ss, 1);
    const float r = rsqrtf(ss / (float)D + eps);
    if (j == 0) rstd_out[item] = r;
    float o1[8], o2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float y1 = x1[e] * r * __bfloat162float(wav[e]), y2 = x2[e] * r * __bfloat162float(wbv[e]);
      // rotate_half: first half gets -second*sin, second half gets +first*sin
      o1[e] = y1 * c[e] - y2 * sn[e];
      o2[e] = y2 * c[e] + y1 * sn[e];
    }
    uint4 pa, pb;
    pa.x = pack_bf16x2(o1[0], o1[1]); pa.y = pack_bf16x2(o1[2], o1[3]);
    pa.z = pack_bf16x2(o1[4], o1[5]); pa.w = pack_bf16x2(o1[6], o1[7]);
    pb.x = pack_bf16x2(o2[0], o2[1]); pb.y = pack_bf16x2(o2[2], o2[3]);
    pb.z = pack_bf16x2(o2[4], o2[5]); pb.w = pack_bf16x2(o2[6], o2[7]);
    __nv_bfloat16* dst = is_q ? q_out + ((size_t)t * nq + h) * D : k_out + ((size_t)t * nkv + (h - nq)) * D;
    *reinterpret_cast<uint4*>(dst + i0) = pa;
    *reinterpret_cast<uint4*>(dst + i1) = pb;
    if (!is_q) {
      const __nv_bfloat16* vs = qkv + (size_t)t * stride_row + (size_t)(nq + nkv + (h - nq)) * D;
      __nv_bfloat16* vd = v_out + ((size_t)t * nkv + (h - nq)) * D;
      *reinterpret_cast<uint4*>(vd + i0) = *reinterpret_cast<const uint4*>(vs + i0);
      *reinterpret_cast<uint4*>(vd + i1) = *reinterpret_cast<const uint4*>(vs + i1);
    }
  }
}

// Backward, same lane layout: per-lane q/k weight-gradient partials (16 each,
// for the lane's fixed elements) folded per CTA into a [gridDim.x, 2D] buffer.
template <int D>
__global__ void __launch_bounds__(256)
    qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
                            const __nv_bfloat16* __restrict__ kw, const int* __restrict__ pos,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dq,
                            const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv,
                            __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dw_part, int T, int nq, int nkv) {
  const int heads = nq + nkv;
  const int lane = threadIdx.x & 31, grp = lane >> 3, j = lane & 7;
  const unsigned gmask = 0xFFu << (grp * 8);
  const int stride_row = (nq + 2 * nkv) * D;
  const int i0 = 8 * j, i1 = D / 2 + 8 * j;
  __shared__ float s_w[2 * D];  // [q weights | k weights] in fp32
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) s_w[i] = __bfloat162float(i < D ? qw[i] : kw[i - D]);
  __syncthreads();
  float aq1[8] = {}, aq2[8] = {}, ak1[8] = {}, ak2[8] = {};
  // Item counts stay below 2^31 (checked on the host), so the (token, head) split is a 32-bit division.
  const int total = T * heads;
  const int step = gridDim.x * (blockDim.x >> 5) * 4;
  for (int item = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 + grp; item < total; item += step) {
    const int t = item / heads, h = item - t * heads;
    const bool is_q = h < nq;
    const __nv_bfloat16* g = is_q ? dq + ((size_t)t * nq + h) * D : dk + ((size_t)t * nkv + (h - nq)) * D;
    const uint4 ga = *reinterpret_cast<const uint4*>(g + i0);
    const uint4 gb = *reinterpret_cast<const uint4*>(g + i1);
    const __nv_bfloat16* src = qkv + (size_t)t * stride_row + (size_t)h * D;
    const uint4 xa = *reinterpret_cast<const uint4*>(src + i0);
    const uint4 xb = *reinterpret_cast<const uint4*>(src + i1);
    const int p = pos[t];
    const float4* ct = reinterpret_cast<const float4*>(cos_t + (size_t)p * (D / 2) + i0);
    const float4* st = reinterpret_cast<const float4*>(sin_t + (size_t)p * (D / 2) + i0);
    const float4 c0 = ct[0], c1 = ct[1], s0 = st[0], s1 = st[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const float r = rstd[item];
    const __nv_bfloat16* gav = reinterpret_cast<const __nv_bfloat16*>(&ga);
    const __nv_bfloat16* gbv = reinterpret_cast<const __nv_bfloat16*>(&gb);
    const __nv_bfloat16* xav = reinterpret_cast<const __nv_bfloat16*>(&xa);
    const __nv_bfloat16* xbv = reinterpret_cast<const __nv_bfloat16*>(&xb);
    const float* w = s_w + (is_q ? 0 : D);
    float dy1[8], dy2[8], xh1[8], xh2[8], dot = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float g1 = __bfloat162float(gav[e]), g2 = __bfloat162float(gbv[e]);
      // transpose of the rotation
      dy1[e] = g1 * c[e] + g2 * sn[e];
      dy2[e] = g2 * c[e] - g1 * sn[e];
      xh1[e] = __bfloat162float(xav[e]) * r;
      xh2[e] = __bfloat162float(xbv[e]) * r;
      dot += dy1[e] * w[i0 + e] * xh1[e] + dy2[e] * w[i1 + e] * xh2[e];
    }
    dot += __shfl_xor_sync(gmask, dot, 4);
    dot += __shfl_xor_sync(gmask, dot, 2);
    dot += __shfl_xor_sync(gmask, dot, 1);
    dot /= (float)D;
    float dx1[8], dx2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      dx1[e] = r * (dy1[e] * w[i0 + e] - xh1[e] * dot);
      dx2[e] = r * (dy2[e] * w[i1 + e] - xh2[e] * dot);
      if (is_q) {
        aq1[e] += dy1[e] * xh1[e];
        aq2[e] += dy2[e] * xh2[e];
      } else {
        ak1[e] += dy1[e] * xh1[e];
        ak2[e] += dy2[e] * xh2[e];
      }
    }
    uint4 pa, pb;
    pa.x = pack_bf16x2(dx1[0], dx1[1]); pa.y = pack_bf16x2(dx1[2], dx1[3]);
    pa.z = pack_bf16x2(dx1[4], dx1[5]); pa.w = pack_bf16x2(dx1[6], dx1[7]);
    pb.x = pack_bf16x2(dx2[0], dx2[1]); pb.y = pack_bf16x2(dx2[2], dx2[3]);
    pb.z = pack_bf16x2(dx2[4], dx2[5]); pb.w = pack_bf16x2(dx2[6], dx2[7]);
    __nv_bfloat16* dst = dqkv + (size_t)t * stride_row + (size_t)h * D;
    *reinterpret_cast<uint4*>(dst + i0) = pa;
    *reinterpret_cast<uint4*>(dst + i1) = pb;
    if (!is_q) {
      const __nv_bfloat16* vg = dv + ((size_t)t * nkv + (h - nq)) * D;
      __nv_bfloat16* vd = dqkv + (size_t)t * stride_row + (size_t)(nq + nkv + (h - nq)) * D;
      *reinterpret_cast<uint4*>(vd + i0) = *reinterpret_cast<const uint4*>(vg + i0);
      *reinterpret_cast<uint4*>(vd + i1) = *reinterpret_cast<const uint4*>(vg + i1);
    }
  }
  // fold the lanes' partials in shared memory, then write this CTA's row of
  // the [gridDim.x, 2D] partial buffer: [q weights (D) | k weights (D)]
  __shared__ float s_acc[2 * D];
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) s_acc[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    atomicAdd(&s_acc[i0 + e], aq1[e]);
    atomicAdd(&s_acc[i1 + e], aq2[e]);
    atomicAdd(&s_acc[D + i0 + e], ak1[e]);
    atomicAdd(&s_acc[D + i1 + e], ak2[e]);
  }
  __syncthreads();
  float* part = dw_part + (size_t)blockIdx.x * 2 * D;
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) part[i] = s_acc[i];
}

// ------------------------------------------------------------------ host wrappers
static int sm_count_nr() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static void check_bf16_rowmajor(const torch::Tensor& t, const char* name) {
  LIBRA_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(),
              "%s: contiguous CUDA bf16 tensor required", name);
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  check_bf16_rowmajor(x, "rmsnorm_fwd x");
  check_bf16_rowmajor(w, "rmsnorm_fwd w");
  const int H = (int)x.size(-1);
  const int T = (int)(x.numel() / H);
  LIBRA_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm_fwd: H must be a multiple of 8 and match w");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, rstd};
  const int warps = 8;
  rmsnorm_fwd_kernel<<<(T + warps - 1) / warps, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
      rstd.data_ptr<float>(), T, H, (float)eps);
  LIBRA_LAUNCH_CHECK();
  return {y, rstd};
}

// Warps per CTA for rmsnorm_bwd: each warp keeps an fp32 [H] row in shared
// memory, so wide rows get fewer warps.
static int rmsnorm_bwd_warps(int H) {
  int w = (int)((200 * 1024) / ((size_t)H * 4));
  return w < 1 ? 1 : (w > 8 ? 8 : w);
}

// CTAs for rmsnorm_bwd: all co-resident CTAs of one wave, but no more than the
// rows need.
using RmsnormBwdKernel = void (*)(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*, const float*,
                                  __nv_bfloat16*, float*, int, int, int);

// The register-resident kernel for rows of up to 4096 elements, else the
// two-pass one.
static RmsnormBwdKernel rmsnorm_bwd_pick(int H) {
  const int vpl = (H / 8 + 31) / 32;
  if (vpl <= 4) return rmsnorm_bwd_reg_kernel<4>;
  if (vpl <= 8) return rmsnorm_bwd_reg_kernel<8>;
  if (vpl <= 10) return rmsnorm_bwd_reg_kernel<10>;  // H = 2560
  if (vpl <= 12) return rmsnorm_bwd_reg_kernel<12>;
  if (vpl <= 16) return rmsnorm_bwd_reg_kernel<16>;
  return rmsnorm_bwd_kernel;
}

static int rmsnorm_bwd_grid(int T, int H, int warps, RmsnormBwdKernel kern) {
  int dev, sms, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = (size_t)warps * H * 4;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, warps * 32, smem);
  if (per_sm < 1) per_sm = 1;
  const int need = (T + warps - 1) / warps;
  int g = sms * per_sm;
  if (need < g) g = need;
  return g < 1 ? 1 : g;
}

static constexpr int kRmsnormBwdMaxH = 51200;  // one warp's fp32 row fits in 200 KB of shared memory

// Returns dx (bf16).  dw (fp32, [H]) is written or accumulated in place.
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                          bool accumulate_dw, c10::optional<torch::Tensor> dx_accum) {
  check_bf16_rowmajor(dy, "rmsnorm_bwd dy");
  check_bf16_rowmajor(x, "rmsnorm_bwd x");
  const int H = (int)x.size(-1);
  const int T = (int)(x.numel() / H);
  LIBRA_CHECK(H % 8 == 0 && H <= kRmsnormBwdMaxH, "rmsnorm_bwd: unsupported H=%d", H);
  LIBRA_CHECK(dw.scalar_type() == at::kFloat && dw.numel() == H && dw.is_contiguous(), "rmsnorm_bwd: dw fp32 [H]");
  const c10::cuda::CUDAGuard guard(x.device());
  torch::Tensor dx;
  int acc_dx = 0;
  if (dx_accum.has_value()) {
    dx = *dx_accum;
    check_bf16_rowmajor(dx, "rmsnorm_bwd dx_accum");
    acc_dx = 1;
  } else {
    dx = torch::empty_like(x);
  }
  auto st = at::cuda::getCurrentCUDAStream();
  if (T == 0) {
    if (!accumulate_dw) dw.zero_();
    return dx;
  }
  const int warps = rmsnorm_bwd_warps(H);
  const RmsnormBwdKernel kern = rmsnorm_bwd_pick(H);
  const int grid = rmsnorm_bwd_grid(T, H, warps, kern);
  auto part = torch::empty({grid, H}, x.options().dtype(at::kFloat));
  kern<<<grid, warps * 32, (size_t)warps * H * 4, st>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(),
      rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(), part.data_ptr<float>(), T, H, acc_dx);
  LIBRA_LAUNCH_CHECK();
  launch_colsum(part.data_ptr<float>(), grid, H, dw.data_ptr<float>(), accumulate_dw, st);
  LIBRA_LAUNCH_CHECK();
  return dx;
}

std::vector<torch::Tensor> qk_norm_rope_fwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                                            torch::Tensor cos_t, torch::Tensor sin_t, int64_t nq, int64_t nkv,
                                            double eps) {
  check_bf16_rowmajor(qkv, "qk_norm_rope qkv");
  const int D = 128;
  LIBRA_CHECK(qkv.size(-1) == (nq + 2 * nkv) * D, "qk_norm_rope: qkv width mismatch (head_dim must be 128)");
  LIBRA_CHECK(pos.scalar_type() == at::kInt && cos_t.scalar_type() == at::kFloat, "qk_norm_rope: int32 pos, fp32 tables");
  const int T = (int)(qkv.numel() / qkv.size(-1));
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto q = torch::empty({T, nq, D}, qkv.options());
  auto k = torch::empty({T, nkv, D}, qkv.options());
  auto v = torch::empty({T, nkv, D}, qkv.options());
  auto rstd = torch::empty({T * (nq + nkv)}, qkv.options().dtype(at::kFloat));
  LIBRA_CHECK((int64_t)T * (nq + nkv) < ((int64_t)1 << 31), "qk_norm_rope: more than 2^31 (token, head) items");
  const int total = T * (int)(nq + nkv);
  if (total == 0) return {q, k, v, rstd};
  LIBRA_CHECK(pos.is_contiguous() && cos_t.is_contiguous() && sin_t.is_contiguous() && qw.is_contiguous() &&
                  kw.is_contiguous() && (reinterpret_cast<uintptr_t>(cos_t.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sin_t.data_ptr()) & 15) == 0,
              "qk_norm_rope: contiguous, 16-byte aligned weights and tables");
  const int warps = 8;  // 32 (token, head) items per CTA
  int blocks = (total + warps * 4 - 1) / (warps * 4);
  const int cap = sm_count_nr() * 16;
  if (blocks > cap) blocks = cap;
  qk_norm_rope_fwd_kernel<128><<<blocks, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)qkv.data_ptr(), (const __nv_bfloat16*)qw.data_ptr(), (const __nv_bfloat16*)kw.data_ptr(),
      pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), (__nv_bfloat16*)q.data_ptr(),
      (__nv_bfloat16*)k.data_ptr(), (__nv_bfloat16*)v.data_ptr(), rstd.data_ptr<float>(), T, (int)nq, (int)nkv,
      (float)eps);
  LIBRA_LAUNCH_CHECK();
  return {q, k, v, rstd};
}

// Returns dqkv; dqw/dkw (fp32 [128]) are accumulated in place.
torch::Tensor qk_norm_rope_bwd(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw, torch::Tensor pos,
                               torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor rstd, torch::Tensor dq,
                               torch::Tensor dk, torch::Tensor dv, torch::Tensor dqw, torch::Tensor dkw, int64_t nq,
                               int64_t nkv) {
  const int D = 128;
  const int T = (int)(qkv.numel() / qkv.size(-1));
  LIBRA_CHECK(dq.is_contiguous() && dk.is_contiguous() && dv.is_contiguous(), "qk_norm_rope_bwd: contiguous grads");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto dqkv = torch::empty_like(qkv);
  const int warps = 8;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  LIBRA_CHECK((int64_t)T * (nq + nkv) < ((int64_t)1 << 31), "qk_norm_rope_bwd: more than 2^31 (token, head) items");
  const int total = T * (int)(nq + nkv);
  int blocks = sms * 8;
  if (blocks * warps * 4 > total) blocks = (total + warps * 4 - 1) / (warps * 4);
  if (blocks < 1) blocks = 1;
  auto part = torch::empty({blocks, 2 * D}, qkv.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  if (total > 0) {
    qk_norm_rope_bwd_kernel<128><<<blocks, warps * 32, 0, st>>>(
        (const __nv_bfloat16*)qkv.data_ptr(), (const __nv_bfloat16*)qw.data_ptr(), (const __nv_bfloat16*)kw.data_ptr(),
        pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rstd.data_ptr<float>(),
        (const __nv_bfloat16*)dq.data_ptr(), (const __nv_bfloat16*)dk.data_ptr(), (const __nv_bfloat16*)dv.data_ptr(),
        (__nv_bfloat16*)dqkv.data_ptr(), part.data_ptr<float>(), T, (int)nq, (int)nkv);
    LIBRA_LAUNCH_CHECK();
  }
  auto sums = torch::empty({2 * D}, qkv.options().dtype(at::kFloat));
  launch_colsum(part.data_ptr<float>(), total > 0 ? blocks : 0, 2 * D, sums.data_ptr<float>(), false, st);
  LIBRA_LAUNCH_CHECK();
  dqw.add_(sums.narrow(0, 0, D));
  dkw.add_(sums.narrow(0, D, D));
  return dqkv;
}

}  // namespace libra

// ------------------------------------------------------------------ RMSNorm bwd without allocation
// C entry point declared in libra_noalloc.h.  Same math and kernels as
// libra::rmsnorm_bwd; the [grid, H] weight-gradient partials live in the
// file-scope device array below instead of a torch allocation, and the grid is
// capped so that grid * H fits in it.
namespace {

constexpr size_t kNoAllocScratchFloats = 512 * 1024;  // 2 MiB of fp32 partials per device
__device__ __align__(256) float g_rmsnorm_bwd_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {};
thread_local char g_noalloc_error[256] = "";

int noalloc_fail(int code, const char* msg) {
  std::snprintf(g_noalloc_error, sizeof(g_noalloc_error), "%s", msg);
  return code;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* libra_rmsnorm_bwd_noalloc_error(void) {
  return g_noalloc_error;
}

extern "C" __attribute__((visibility("default"))) int libra_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw, int T, int H,
    int accumulate_dx, int accumulate_dw, cudaStream_t stream) {
  using namespace libra;
  g_noalloc_error[0] = 0;
  if (T < 0 || H <= 0 || H % 8 != 0) return noalloc_fail(1, "libra_rmsnorm_bwd_noalloc: need T >= 0 and H a positive multiple of 8");
  if ((size_t)H > kNoAllocScratchFloats || H > kRmsnormBwdMaxH)
    return noalloc_fail(2, "libra_rmsnorm_bwd_noalloc: H exceeds the no-alloc limit (H <= 51200)");
  if (!dw || (T > 0 && (!dy || !x || !w || !rstd || !dx)))
    return noalloc_fail(1, "libra_rmsnorm_bwd_noalloc: null pointer argument");
  const uintptr_t align_or = (uintptr_t)dy | (uintptr_t)x | (uintptr_t)w | (uintptr_t)dx;
  if (T > 0 && (align_or & 15u)) return noalloc_fail(1, "libra_rmsnorm_bwd_noalloc: dy/x/w/dx must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(3, "libra_rmsnorm_bwd_noalloc: no usable current CUDA device");
  float* scratch = nullptr;
  {
    // first call on each device: resolve the scratch array's address once,
    // with that device current
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_scratch_ptr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);
      if (e != cudaSuccess || !p) {
        char msg[200];
        std::snprintf(msg, sizeof(msg), "libra_rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(e));
        return noalloc_fail(3, msg);
      }
      g_noalloc_scratch_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_scratch_ptr[dev];
  }
  if (T == 0) {
    colsum_kernel<<<(H + 31) / 32, dim3(32, kColsumRowGroups), 0, stream>>>(scratch, 0, H, dw, accumulate_dw ? 1 : 0);
  } else {
    const int warps = rmsnorm_bwd_warps(H);
    const RmsnormBwdKernel kern = rmsnorm_bwd_pick(H);
    int grid = rmsnorm_bwd_grid(T, H, warps, kern);
    const int cap = (int)(kNoAllocScratchFloats / (size_t)H);
    if (grid > cap) grid = cap;
    kern<<<grid, warps * 32, (size_t)warps * H * 4, stream>>>(
        (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, rstd, (__nv_bfloat16*)dx, scratch,
        T, H, accumulate_dx ? 1 : 0);
    colsum_kernel<<<(H + 31) / 32, dim3(32, kColsumRowGroups), 0, stream>>>(scratch, grid, H, dw, accumulate_dw ? 1 : 0);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[200];
    std::snprintf(msg, sizeof(msg), "libra_rmsnorm_bwd_noalloc: launch failed: %s", cudaGetErrorString(e));
    return noalloc_fail(4, msg);
  }
  return 0;
}

// quantize.cuh — per-tensor e4m3 quantisation kernels (bandwidth bound).
//
// Semantics restated from the reference (diffusion/fp8_kernels.py):
//   amax      = max |x|                                   (:54-64, partial_amax_kernel)
//   scale     = amax > 0 ? amax / 448 : 1.0   (fp32)      (:90-102, finalize_amax_kernel)
//   q         = e4m3(max(-448, min(x / scale, 448)))      (:105-120, quantize_fp8_kernel)
// The clamp uses min-then-max with non-NaN-propagating fminf/fmaxf (the
// reference's tl.minimum / tl.maximum defaults), so x/0 = NaN clamps to +448.
// The division is IEEE round-to-nearest (__fdiv_rn) and the cast is
// cvt.rn.satfinite.e4m3x2.f32, which makes the bytes reproducible on the CPU.
//
// Current scaling (quantize_fp8, :559-601) is two launches:
//   amax_partials_kernel : grid-stride |x| max, one fp32 partial per CTA
//   quantize_cast_kernel<kCurrent> : every CTA folds the partials into amax and
//                          the scale (the reference's separate finalize launch
//                          disappears), CTA 0 publishes the scale, then casts.
// Delayed scaling (quantize_fp8_delayed, :518-556) is one pass plus a 1-CTA fold:
//   quantize_cast_kernel<kDelayed> : cast with the previous scale and emit amax partials
//   finalize_scale_kernel          : partials -> current scale
#pragma once

#include "sm100_common.cuh"

namespace fp8b {

constexpr int kQuantThreads = 256;
constexpr float kE4M3Max = 448.0f;

enum QuantMode : int { kCurrent = 0, kDelayed = 1 };

// Two floats -> two e4m3 bytes; `lo` lands in the low byte.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float scale_and_clamp(float v, float s) {
  float t = __fdiv_rn(v, s);
  t = fminf(t, kE4M3Max);   // tl.minimum(scaled, FP8_MAX)
  return fmaxf(-kE4M3Max, t);  // tl.maximum(-FP8_MAX, .)
}

__device__ __forceinline__ float absmax_word(float m, uint32_t w) {
  return fmaxf(m, fmaxf(fabsf(bf16_lo_f(w)), fabsf(bf16_hi_f(w))));
}

// Block-wide max of a non-negative value; result valid in every thread.
__device__ __forceinline__ float block_max(float v) {
  __shared__ float red[kQuantThreads / 32];
  __shared__ float result;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < (kQuantThreads / 32) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) result = w;
  }
  __syncthreads();
  return result;
}

__device__ __forceinline__ float scale_from_amax(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, kE4M3Max) : 1.0f;
}

// Fold `count` partial maxima into the tensor scale (every CTA does this; the
// partials are a few KB and L2 resident).
__device__ __forceinline__ float fold_partials_to_scale(const float* __restrict__ partials, int count) {
  float m = 0.0f;
  for (int i = threadIdx.x; i < count; i += blockDim.x) m = fmaxf(m, partials[i]);
  return scale_from_amax(block_max(m));
}

__device__ __forceinline__ float absmax_pair(uint32_t w) { return fmaxf(fabsf(bf16_lo_f(w)), fabsf(bf16_hi_f(w))); }

// max |.| of the 8 bf16 of a 16-byte vector folded into m (a depth-3 tree, so
// consecutive vectors do not serialise on one accumulator).
__device__ __forceinline__ float absmax_vec(float m, const uint4& a) {
  return fmaxf(m, fmaxf(fmaxf(absmax_pair(a.x), absmax_pair(a.y)), fmaxf(absmax_pair(a.z), absmax_pair(a.w))));
}

// Pass 1 of current scaling: |x| max per CTA.  Each thread keeps V 16-byte
// loads in flight per iteration (coalesced: vector i + v*T).  VEC: x is
// 16-byte aligned.
template <bool VEC, int V>
__global__ void __launch_bounds__(kQuantThreads) amax_partials_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                      float* __restrict__ partials) {
  float m = 0.0f;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (VEC) {
    const int64_t nvec = n >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    int64_t i = tid;
    for (; i + (V - 1) * nthreads < nvec; i += V * nthreads) {
      uint4 a[V];
#pragma unroll
      for (int v = 0; v < V; ++v) a[v] = __ldg(xv + i + v * nthreads);
      float mv[V];
#pragma unroll
      for (int v = 0; v < V; ++v) mv[v] = absmax_vec(0.0f, a[v]);
#pragma unroll
      for (int w = 1; w < V; w *= 2) {
#pragma unroll
        for (int v = 0; v + w < V; v += 2 * w) mv[v] = fmaxf(mv[v], mv[v + w]);
      }
      m = fmaxf(m, mv[0]);
    }
    for (; i < nvec; i += nthreads) m = absmax_vec(m, __ldg(xv + i));
    done = nvec << 3;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) m = fmaxf(m, fabsf(__uint_as_float(uint32_t(x[i]) << 16)));
  m = block_max(m);
  if (threadIdx.x == 0) partials[blockIdx.x] = m;
}

__device__ __forceinline__ uint32_t cast4(uint32_t w0, uint32_t w1, float s) {
  const uint32_t lo = cvt_e4m3x2(scale_and_clamp(bf16_lo_f(w0), s), scale_and_clamp(bf16_hi_f(w0), s));
  const uint32_t hi = cvt_e4m3x2(scale_and_clamp(bf16_lo_f(w1), s), scale_and_clamp(bf16_hi_f(w1), s));
  return lo | (hi << 16);
}

__device__ __forceinline__ uint2 cast_vec(const uint4& a, float s) {
  return make_uint2(cast4(a.x, a.y, s), cast4(a.z, a.w, s));
}

// Cast pass.  kCurrent: scale = fold(partials_in); CTA 0 stores it to scale_out.
//             kDelayed: scale = *prev_scale; each CTA also writes its |x| max
//                       to partials_out[blockIdx.x].
// V 16-byte loads in flight per thread and iteration.  In current mode x was
// just read by the amax pass, so the loads here are its last use (streaming
// hint); the e4m3 output is stored normally (its consumer follows).
// VEC: x 16-byte aligned and q 8-byte aligned.
template <int MODE, bool VEC, int V>
__global__ void __launch_bounds__(kQuantThreads) quantize_cast_kernel(
    const uint16_t* __restrict__ x, uint8_t* __restrict__ q, int64_t n, const float* __restrict__ partials_in,
    int n_partials, const float* __restrict__ prev_scale, float* __restrict__ scale_out,
    float* __restrict__ partials_out) {
  float s;
  if (MODE == kCurrent) {
    s = fold_partials_to_scale(partials_in, n_partials);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  } else {
    s = *prev_scale;
  }
  float m = 0.0f;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (VEC) {
    const int64_t nvec = n >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint2* qv = reinterpret_cast<uint2*>(q);
    int64_t i = tid;
    for (; i + (V - 1) * nthreads < nvec; i += V * nthreads) {
      uint4 a[V];
#pragma unroll
      for (int v = 0; v < V; ++v) a[v] = MODE == kCurrent ? __ldcs(xv + i + v * nthreads) : __ldg(xv + i + v * nthreads);
      if (MODE == kDelayed) {
#pragma unroll
        for (int v = 0; v < V; ++v) m = absmax_vec(m, a[v]);
      }
#pragma unroll
      for (int v = 0; v < V; ++v) qv[i + v * nthreads] = cast_vec(a[v], s);
    }
    for (; i < nvec; i += nthreads) {
      const uint4 a = __ldg(xv + i);
      if (MODE == kDelayed) m = absmax_vec(m, a);
      qv[i] = cast_vec(a, s);
    }
    done = nvec << 3;
  }
  for (int64_t i = done + tid; i < n; i += nthreads) {
    const float v = __uint_as_float(uint32_t(x[i]) << 16);
    if (MODE == kDelayed) m = fmaxf(m, fabsf(v));
    q[i] = static_cast<uint8_t>(cvt_e4m3x2(scale_and_clamp(v, s), 0.0f) & 0xFFu);
  }
  if (MODE == kDelayed) {
    m = block_max(m);
    if (threadIdx.x == 0) partials_out[blockIdx.x] = m;
  }
}

__global__ void __launch_bounds__(kQuantThreads) finalize_scale_kernel(const float* __restrict__ partials,
                                                                       int n_partials, float* __restrict__ scale_out) {
  const float s = fold_partials_to_scale(partials, n_partials);
  if (threadIdx.x == 0) *scale_out = s;
}

// ---------------------------------------------------------------- byte transposes
// dst[b][c][r] = src[b][r][c] for a batch of R x C byte matrices with arbitrary
// leading dimensions.  Used for the conv weight re-layout
// [Cout][3][3][Cin] -> [Cin][3][3][Cout] (batch = the 9 taps) and for the plain
// 2-D transpose the reference applies to dY (fp8_kernels.py:321-337).
constexpr int kTransTile = 64;

__global__ void __launch_bounds__(256) transpose_u8_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                           int64_t rows, int64_t cols, int64_t src_ld,
                                                           int64_t dst_ld, int64_t src_bstride,
                                                           int64_t dst_bstride) {
  __shared__ uint8_t tile[kTransTile][kTransTile + 4];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kTransTile;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kTransTile;
  const uint8_t* s = src + static_cast<int64_t>(blockIdx.z) * src_bstride;
  uint8_t* d = dst + static_cast<int64_t>(blockIdx.z) * dst_bstride;
  for (int i = threadIdx.x; i < kTransTile * kTransTile; i += blockDim.x) {
    const int rr = i / kTransTile, cc = i % kTransTile;
    const int64_t r = r0 + rr, c = c0 + cc;
    if (r < rows && c < cols) tile[rr][cc] = s[r * src_ld + c];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kTransTile * kTransTile; i += blockDim.x) {
    const int cc = i / kTransTile, rr = i % kTransTile;
    const int64_t r = r0 + rr, c = c0 + cc;
    if (r < rows && c < cols) d[c * dst_ld + r] = tile[rr][cc];
  }
}

// Same transpose for whole 64x64 tiles with 16-byte aligned rows: one 16-byte
// load and one 16-byte store per thread (the weight re-layout of the
// data-grad runs on every backward pass, so it should cost a launch, not more).
__global__ void __launch_bounds__(256) transpose_u8_tiles16_kernel(const uint8_t* __restrict__ src,
                                                                   uint8_t* __restrict__ dst, int64_t src_ld,
                                                                   int64_t dst_ld, int64_t src_bstride,
                                                                   int64_t dst_bstride) {
  __shared__ __align__(16) uint8_t tile[kTransTile][kTransTile + 4];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kTransTile;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kTransTile;
  const uint8_t* s = src + static_cast<int64_t>(blockIdx.z) * src_bstride;
  uint8_t* d = dst + static_cast<int64_t>(blockIdx.z) * dst_bstride;
  const int row = threadIdx.x >> 2, seg = (threadIdx.x & 3) * 16;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(s + (r0 + row) * src_ld + c0 + seg));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 16; ++i) tile[row][seg + i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
  __syncthreads();
  // output row = input column `row`, output bytes = input rows seg .. seg+15
  uint32_t o[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i >> 2] |= static_cast<uint32_t>(tile[seg + i][row]) << (8 * (i & 3));
  *reinterpret_cast<uint4*>(d + (c0 + row) * dst_ld + r0 + seg) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace fp8b

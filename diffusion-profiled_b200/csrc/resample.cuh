// resample.cuh — the UNet's nearest-neighbour resampling and skip concatenation
// on NHWC activations, in the dtypes the reference produces under bf16 autocast
// (reference unet.py:368-383: F.interpolate(x, scale_factor=0.5 / 2.0,
// mode="nearest") runs in fp32 under autocast, so its output is fp32 whatever
// the input; torch.cat promotes to the widest input dtype).
//
//   down2      : y[n, h, w, c] = fp32(x[n, 2h, 2w, c])                  (scale 0.5)
//   down2 bwd  : dx[n, h, w, c] = (h, w even) ? dy[n, h/2, w/2, c] : 0   (in x's dtype)
//   up_cat     : y[n, h, w, 0:C1]      = a[n, h/f, w/f, :]               (f = 2, or 1: no resampling)
//                y[n, h, w, C1:C1+C2]  = s[n, h, w, :]
//   up_cat bwd : da[n, h, w, c] = sum over the f x f block of dy[.., c]  (fp32 sum, rounded to a's dtype)
//                ds[n, h, w, c] = dy[n, h, w, C1 + c]                    (in s's dtype)
//   pair       : up_cat with y fp32 and also y16 = bf16(y); its backward takes
//                dy + dy16 (fp32 sum) as the gradient of y
//
// One kernel per direction: the autocast casts, the separate resampling pass
// and the concatenation copy become one read and one write of each element.
// Each thread moves vectors of 8 channels (C1, C2 multiples of 8).
#pragma once

#include "groupnorm.cuh"

namespace fp8b {

constexpr int kResampleThreads = 256;

// 8 channels of type T at vector index vi (8 elements per vector) as fp32, and back.
template <typename T>
__device__ __forceinline__ void load8f(const T* __restrict__ p, int64_t vi, float (&f)[8]) {
  unpack_x8(load_x8(p, vi), f);
}

template <typename TX>
__global__ void __launch_bounds__(kResampleThreads) down2_kernel(const TX* __restrict__ x, int n, int h, int w,
                                                                 int c, float* __restrict__ y) {
  pdl_wait();
  const int ho = h / 2, wo = w / 2, vecs = c / 8;
  const int64_t total = static_cast<int64_t>(n) * ho * wo * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vecs);
    const int64_t pix = i / vecs;
    const int wq = static_cast<int>(pix % wo);
    const int64_t r = pix / wo;
    const int hq = static_cast<int>(r % ho);
    const int64_t img = r / ho;
    const int64_t src = ((img * h + 2 * hq) * w + 2 * wq) * vecs + v;
    float f[8];
    load8f(x, src, f);
    store_x8(y, i, f);
  }
}

template <typename TX>
__global__ void __launch_bounds__(kResampleThreads) down2_bwd_kernel(const float* __restrict__ dy, int n, int h,
                                                                     int w, int c, TX* __restrict__ dx) {
  pdl_wait();
  const int ho = h / 2, wo = w / 2, vecs = c / 8;
  const int64_t total = static_cast<int64_t>(n) * h * w * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vecs);
    const int64_t pix = i / vecs;
    const int wi = static_cast<int>(pix % w);
    const int64_t r = pix / w;
    const int hi = static_cast<int>(r % h);
    const int64_t img = r / h;
    float f[8];
    if (((hi | wi) & 1) == 0 && hi / 2 < ho && wi / 2 < wo) {
      load8f(dy, ((img * ho + hi / 2) * wo + wi / 2) * vecs + v, f);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = 0.0f;
    }
    store_x8(dx, i, f);
  }
}

// y has C1 + C2 channels at (h, w); a is (h / f, w / f) with C1 channels; s is (h, w) with C2.
// y16 (may be null): a second output, bf16(y) -- the copy bf16 autocast makes of
// an fp32 y for the 1x1 skip conv that reads it -- written in the same pass.
template <typename TA, typename TS, typename TO>
__global__ void __launch_bounds__(kResampleThreads) up_cat_kernel(const TA* __restrict__ a, const TS* __restrict__ s,
                                                                  int n, int h, int w, int c1, int c2, int f,
                                                                  TO* __restrict__ y, uint16_t* __restrict__ y16) {
  pdl_wait();
  const int v1 = c1 / 8, vecs = (c1 + c2) / 8;
  const int ha = h / f, wa = w / f;
  const int64_t total = static_cast<int64_t>(n) * h * w * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vecs);
    const int64_t pix = i / vecs;
    float e[8];
    if (v < v1) {
      const int wi = static_cast<int>(pix % w);
      const int64_t r = pix / w;
      const int hi = static_cast<int>(r % h);
      const int64_t img = r / h;
      load8f(a, ((img * ha + hi / f) * wa + wi / f) * v1 + v, e);
    } else {
      load8f(s, pix * (vecs - v1) + (v - v1), e);
    }
    store_x8(y, i, e);
    if (y16 != nullptr) store_x8(y16, i, e);
  }
}

// dy16 (may be null): the gradient of the y16 output, added to dy in fp32 first
// (the sum autograd forms for a tensor read twice), element by element.
template <typename TO>
__device__ __forceinline__ void load_dy8(const TO* __restrict__ dy, const uint16_t* __restrict__ dy16, int64_t vi,
                                         float (&e)[8]) {
  load8f(dy, vi, e);
  if (dy16 != nullptr) {
    float g[8];
    load8f(dy16, vi, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] += g[k];
  }
}

template <typename TA, typename TS, typename TO>
__global__ void __launch_bounds__(kResampleThreads) up_cat_bwd_kernel(const TO* __restrict__ dy,
                                                                      const uint16_t* __restrict__ dy16, int n, int h,
                                                                      int w, int c1, int c2, int f,
                                                                      TA* __restrict__ da, TS* __restrict__ ds) {
  pdl_wait();
  const int v1 = c1 / 8, v2 = c2 / 8, vecs = v1 + v2;
  const int ha = h / f, wa = w / f;
  const int64_t total_a = static_cast<int64_t>(n) * ha * wa * v1;
  const int64_t total_s = static_cast<int64_t>(n) * h * w * v2;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total_a + total_s;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < total_a) {
      const int v = static_cast<int>(i % v1);
      const int64_t pix = i / v1;
      const int wq = static_cast<int>(pix % wa);
      const int64_t r = pix / wa;
      const int hq = static_cast<int>(r % ha);
      const int64_t img = r / ha;
      float acc[8] = {};
      for (int di = 0; di < f; ++di)
        for (int dj = 0; dj < f; ++dj) {
          float e[8];
          load_dy8(dy, dy16, ((img * h + hq * f + di) * w + wq * f + dj) * vecs + v, e);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] += e[k];
        }
      store_x8(da, i, acc);
    } else {
      const int64_t j = i - total_a;
      const int v = static_cast<int>(j % v2);
      const int64_t pix = j / v2;
      float e[8];
      load_dy8(dy, dy16, pix * vecs + v1 + v, e);
      store_x8(ds, j, e);
    }
  }
}

// ---------------------------------------------------------------- residual joins
// y = (a + b) / sqrt(2) as the reference's bf16-autocast ops compute it
// (unet.py:161 and :203, `(skip + h) / math.sqrt(2.0)`): the sum rounded to the
// result dtype TO (the wider of the two), then multiplied by inv = RN32(1 / RN32(sqrt 2))
// -- torch divides a tensor by a host scalar as a multiplication by its
// reciprocal in fp32 -- and rounded to TO again.  Backward: g = RN_TO(dy * inv),
// handed to a and b in their own dtypes.  Element-wise on dense tensors of one
// memory layout, 8 elements per thread.
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  if constexpr (sizeof(T) == 2) return __uint_as_float(pack_bf16x2(v, 0.0f) << 16);
  return v;
}

template <typename TA, typename TB, typename TO>
__global__ void __launch_bounds__(kResampleThreads) add_scale_kernel(const TA* __restrict__ a, const TB* __restrict__ b,
                                                                     int64_t vecs, float inv, TO* __restrict__ y) {
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vecs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float fa[8], fb[8];
    load8f(a, i, fa);
    load8f(b, i, fb);
#pragma unroll
    for (int k = 0; k < 8; ++k) fa[k] = round_to<TO>(fa[k] + fb[k]) * inv;
    store_x8(y, i, fa);
  }
}

template <typename TA, typename TB, typename TO>
__global__ void __launch_bounds__(kResampleThreads) add_scale_bwd_kernel(const TO* __restrict__ dy, int64_t vecs,
                                                                         float inv, TA* __restrict__ da,
                                                                         TB* __restrict__ db) {
  pdl_wait();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vecs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float g[8];
    load8f(dy, i, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = round_to<TO>(g[k] * inv);
    store_x8(da, i, g);
    store_x8(db, i, g);
  }
}

// The join's backward when b is the bf16 output of a delayed-scaling FP8 conv:
// db is also written as e4m3, cast with max(window) exactly as that conv's
// backward would cast its output gradient (fp8_quantize_delayed_window with
// advance = 0, reference fp8_kernels.py:883-889), with one |db| max per CTA that
// the last CTA folds into db's scale (stored at window[*pos]; pos is kept).
// Fewer, longer-lived CTAs than the plain passes (each first reduces the scale
// history), with kJoinUnroll vectors of dy in flight per thread.
constexpr int kJoinUnroll = 4;

template <typename TA, typename TO, class Div>
__device__ __forceinline__ uint32_t add_scale_bwd_quant_loop(const TO* __restrict__ dy, int64_t vecs, float inv,
                                                             TA* __restrict__ da, uint16_t* __restrict__ db,
                                                             uint8_t* __restrict__ dbq, const Div& div) {
  uint32_t m2 = 0u;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < vecs;
       i0 += kJoinUnroll * stride) {
    XVec<TO> v[kJoinUnroll];
#pragma unroll
    for (int u = 0; u < kJoinUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      v[u] = i < vecs ? load_x8(dy, i) : zero_x8<TO>();
    }
#pragma unroll
    for (int u = 0; u < kJoinUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= vecs) break;
      float g[8];
      unpack_x8(v[u], g);
#pragma unroll
      for (int k = 0; k < 8; ++k) g[k] = round_to<TO>(g[k] * inv);
      store_x8(da, i, g);
      const uint4 h = pack8(g);
      reinterpret_cast<uint4*>(db)[i] = h;
      m2 = bf16x2_max(m2, absmax_vec2(h));
      reinterpret_cast<uint2*>(dbq)[i] = cast_vec(h, div);
    }
  }
  return m2;
}

template <typename TA, typename TO>
__global__ void __launch_bounds__(kResampleThreads) add_scale_bwd_quant_kernel(
    const TO* __restrict__ dy, int64_t vecs, float inv, TA* __restrict__ da, uint16_t* __restrict__ db,
    uint8_t* __restrict__ dbq, DelayedSource src, float* __restrict__ partials, ScaleFold fold) {
  pdl_wait();
  const float s = delayed_scale<kResampleThreads>(src);
  const uint32_t m2 = markstein_applies(s)  // s is uniform over the grid
                          ? add_scale_bwd_quant_loop(dy, vecs, inv, da, db, dbq, make_markstein(s))
                          : add_scale_bwd_quant_loop(dy, vecs, inv, da, db, dbq, DivF64(s));
  const float m = block_max<kResampleThreads>(unpack_max2(m2));
  if (threadIdx.x == 0) partials[blockIdx.x] = m;
  fold_scale_if_last<kResampleThreads>(partials, fold);
}

}  // namespace fp8b

// layernorm.cuh — LayerNorm over the channels of each token, forward and
// backward, for the attention blocks of the UNet (reference CHWAttention,
// unet.py:174 and :187: nn.LayerNorm(C) on the [B, HW, C] tokens of a
// channels_last feature map, run in fp32 under autocast and cast to bf16 by the
// qkv projection that consumes it).
//
//   y[t, c] = bf16( (x[t, c] - mean_t) * rstd_t * gamma_c + beta_c ),
//   rstd_t  = 1 / sqrt(var_t + eps)   (biased variance, as nn.LayerNorm)
//
// One warp per token: a lane holds VPL vectors of 8 channels (C <= 256 * VPL),
// so the mean and the variance (of the deviations, two passes over registers)
// are warp reductions and x is read once.  The backward reads x and dy once:
//   xhat = (x - mean) * rstd,  g = dy * gamma
//   dx   = rstd * (g - mean_c(g) - xhat * mean_c(g * xhat))
// and accumulates dgamma = sum_t dy * xhat, dbeta = sum_t dy per lane in
// registers; each CTA writes its partial sums, and a small kernel adds the
// partials of all CTAs in a fixed order (deterministic).
// x and dx are bf16 or fp32; y and dy are bf16.
#pragma once

#include "groupnorm.cuh"

namespace fp8b {

constexpr int kLnThreads = 256;
constexpr int kLnWarps = kLnThreads / 32;

template <typename TX, int VPL>
__global__ void __launch_bounds__(kLnThreads) ln_fwd_kernel(const TX* __restrict__ x,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, int64_t tokens, int c,
                                                            float eps, uint16_t* __restrict__ y,
                                                            float2* __restrict__ mean_rstd) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int vecs = c / 8;
  const float inv_c = 1.0f / static_cast<float>(c);
  float g[VPL][8], b[VPL][8];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int v = lane + 32 * j;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      g[j][k] = v < vecs ? gamma[v * 8 + k] : 0.0f;
      b[j][k] = v < vecs ? beta[v * 8 + k] : 0.0f;
    }
  }
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kLnWarps;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5); t < tokens; t += warps) {
    const TX* xt = x + t * c;
    float f[VPL][8];
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < vecs) {
        unpack_x8(load_x8(xt, v), f[j]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) f[j][k] = 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += f[j][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_c;
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < vecs) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = f[j][k] - mean;
          sq = fmaf(d, d, sq);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq * inv_c + eps);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < vecs) {
        float o8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o8[k] = fmaf((f[j][k] - mean) * rstd, g[j][k], b[j][k]);
        reinterpret_cast<uint4*>(y + t * c)[v] = pack8(o8);
      }
    }
    if (lane == 0) mean_rstd[t] = make_float2(mean, rstd);
  }
}

// part[blockIdx][0:C] = sum over this CTA's tokens of dy * xhat, part[..][C:2C] = sum of dy.
template <typename TX, int VPL>
__global__ void __launch_bounds__(kLnThreads) ln_bwd_kernel(const TX* __restrict__ x,
                                                            const uint16_t* __restrict__ dy,
                                                            const float* __restrict__ gamma,
                                                            const float2* __restrict__ mean_rstd, int64_t tokens,
                                                            int c, TX* __restrict__ dx, float* __restrict__ part) {
  extern __shared__ float ln_smem[];  // [kLnWarps][2C]
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vecs = c / 8;
  const float inv_c = 1.0f / static_cast<float>(c);
  float g[VPL][8], dgam[VPL][8], dbet[VPL][8];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int v = lane + 32 * j;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      g[j][k] = v < vecs ? gamma[v * 8 + k] : 0.0f;
      dgam[j][k] = 0.0f;
      dbet[j][k] = 0.0f;
    }
  }
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kLnWarps;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * kLnWarps + warp; t < tokens; t += warps) {
    const TX* xt = x + t * c;
    const uint4* dt = reinterpret_cast<const uint4*>(dy + t * c);
    const float2 mr = mean_rstd[t];
    float xh[VPL][8], gy[VPL][8];
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      float xf[8], df[8];
      if (v < vecs) {
        unpack_x8(load_x8(xt, v), xf);
        unpack8(__ldg(dt + v), df);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) xf[k] = df[k] = 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        xh[j][k] = (xf[k] - mr.x) * mr.y;
        gy[j][k] = df[k] * g[j][k];
        dgam[j][k] = fmaf(df[k], xh[j][k], dgam[j][k]);
        dbet[j][k] += df[k];
        s1 += gy[j][k];
        s2 = fmaf(gy[j][k], xh[j][k], s2);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const float m1 = s1 * inv_c, m2 = s2 * inv_c;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int v = lane + 32 * j;
      if (v < vecs) {
        float o8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o8[k] = mr.y * (gy[j][k] - m1 - xh[j][k] * m2);
        store_x8(dx + t * c, v, o8);
      }
    }
  }
  // per-CTA parameter-gradient partials, summed over the warps in a fixed order
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int v = lane + 32 * j;
    if (v < vecs)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        ln_smem[warp * 2 * c + v * 8 + k] = dgam[j][k];
        ln_smem[warp * 2 * c + c + v * 8 + k] = dbet[j][k];
      }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * c; i += blockDim.x) {
    float s = 0.0f;
    for (int w = 0; w < kLnWarps; ++w) s += ln_smem[w * 2 * c + i];
    part[static_cast<int64_t>(blockIdx.x) * 2 * c + i] = s;
  }
}

// dgamma[c] = sum_b part[b][c], dbeta[c] = sum_b part[b][C + c]: one warp per
// output, lanes striding over the partials, then a shuffle tree (fixed order).
__global__ void __launch_bounds__(kLnThreads) ln_param_reduce_kernel(const float* __restrict__ part, int parts, int c,
                                                                     float* __restrict__ dgamma,
                                                                     float* __restrict__ dbeta) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (i >= 2 * c) return;
  float s = 0.0f;
  for (int b = lane; b < parts; b += 32) s += part[static_cast<int64_t>(b) * 2 * c + i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    if (i < c)
      dgamma[i] = s;
    else
      dbeta[i - c] = s;
  }
}

}  // namespace fp8b

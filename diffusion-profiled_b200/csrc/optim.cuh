// optim.cuh — gradient clipping, AdamW and the EMA of the weights as one pass
// over the parameters (the training step's tail, reference train.py / ddpm.py:20-25:
// clip_grad_norm_(params, max_norm), AdamW, then ema = ema * beta + (1 - beta) * p).
//
//   coef   = min(1, max_norm / (||g||_2 + 1e-6))                  (clip_grad_norm_)
//   g'     = g * coef
//   p      = p * (1 - lr * wd)                                    (decoupled weight decay)
//   m      = m + (1 - b1) * (g' - m)                              (exp_avg.lerp_)
//   v      = v * b2 + (1 - b2) * g' * g'
//   p      = p - (lr / (1 - b1^t)) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
//   ema    = RN(ema * beta) + RN((1 - beta) * p)                  (the reference's two roundings)
//
// Three kernels for all parameters: per-chunk sums of g^2, one CTA for the norm,
// the clip factor and the step count (kept on the device, so a captured graph
// advances it every replay), and the update.  Each reads p, g, m, v, ema once and
// writes p, m, v, ema once: 36 bytes per parameter, where the separate clip,
// optimizer and EMA passes move about twice that.  Tensors are passed in groups
// of kOptTensors per launch (kernel parameter space).
#pragma once

#include "quantize.cuh"

namespace fp8b {

constexpr int kOptTensors = 40;
constexpr int kOptChunk = 8192;  // elements per CTA
constexpr int kOptThreads = 256;

struct OptGroup {
  float* p[kOptTensors];
  const float* g[kOptTensors];
  float* m[kOptTensors];
  float* v[kOptTensors];
  float* ema[kOptTensors];
  int64_t n[kOptTensors];
  int chunk_begin[kOptTensors + 1];
  int count;
};
static_assert(sizeof(OptGroup) < 4000, "kernel parameter size");

struct OptHyper {
  float lr, beta1, beta2, eps, weight_decay, ema_beta, max_norm;
  const float* coef;   // clip factor (device), from opt_norm_kernel
  const float* step;   // step count after this step (device)
};

__device__ __forceinline__ int opt_tensor_of(const OptGroup& b, int k) {
  int lo = 0, hi = b.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.chunk_begin[mid] <= k) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// partials[part0 + k] = sum of g^2 over chunk k of this group.
__global__ void __launch_bounds__(kOptThreads) opt_sumsq_kernel(OptGroup b, float* __restrict__ partials, int part0) {
  pdl_wait();
  __shared__ float red[kOptThreads / 32];
  const int k = blockIdx.x;
  const int t = opt_tensor_of(b, k);
  const int64_t begin = static_cast<int64_t>(k - b.chunk_begin[t]) * kOptChunk;
  const int64_t end = min(begin + kOptChunk, b.n[t]);
  const float* __restrict__ g = b.g[t];
  float s = 0.0f;
  for (int64_t i = begin + threadIdx.x; i < end; i += kOptThreads) s = fmaf(g[i], g[i], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.0f;
    for (int w = 0; w < kOptThreads / 32; ++w) tot += red[w];
    partials[part0 + k] = tot;
  }
}

// One CTA: coef = min(1, max_norm / (sqrt(sum partials) + 1e-6)) (1 when max_norm <= 0); step += 1.
__global__ void __launch_bounds__(kOptThreads) opt_norm_kernel(const float* __restrict__ partials, int n_parts,
                                                               float max_norm, float* __restrict__ coef,
                                                               float* __restrict__ step) {
  pdl_wait();
  __shared__ float red[kOptThreads];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n_parts; i += kOptThreads) s += partials[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = kOptThreads / 2; w > 0; w >>= 1) {  // fixed-order tree
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float c = 1.0f;
    if (max_norm > 0.0f) c = fminf(1.0f, max_norm / (sqrtf(red[0]) + 1e-6f));
    *coef = c;
    *step += 1.0f;
  }
}

__global__ void __launch_bounds__(kOptThreads) opt_update_kernel(OptGroup b, OptHyper h) {
  pdl_wait();
  const int k = blockIdx.x;
  const int t = opt_tensor_of(b, k);
  const int64_t begin = static_cast<int64_t>(k - b.chunk_begin[t]) * kOptChunk;
  const int64_t end = min(begin + kOptChunk, b.n[t]);
  const float coef = *h.coef;
  const float step = *h.step;
  const float bc1 = 1.0f - powf(h.beta1, step);
  const float bc2_sqrt = sqrtf(1.0f - powf(h.beta2, step));
  const float step_size = h.lr / bc1;
  const float decay = 1.0f - h.lr * h.weight_decay;
  const float one_m_ema = 1.0f - h.ema_beta;
  float* __restrict__ p = b.p[t];
  const float* __restrict__ g = b.g[t];
  float* __restrict__ m = b.m[t];
  float* __restrict__ v = b.v[t];
  float* __restrict__ e = b.ema[t];
  for (int64_t i = begin + threadIdx.x; i < end; i += kOptThreads) {
    const float gi = g[i] * coef;
    float pi = p[i] * decay;
    float mi = m[i];
    mi = fmaf(1.0f - h.beta1, gi - mi, mi);
    const float vi = fmaf(v[i], h.beta2, (1.0f - h.beta2) * gi * gi);
    pi -= step_size * mi / (sqrtf(vi) / bc2_sqrt + h.eps);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (e != nullptr) e[i] = __fadd_rn(__fmul_rn(e[i], h.ema_beta), __fmul_rn(one_m_ema, pi));
  }
}

}  // namespace fp8b

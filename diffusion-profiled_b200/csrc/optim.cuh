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

// Whether tensor t's chunks can move as float4 (every pointer 16-byte aligned;
// chunk starts are multiples of kOptChunk, so of 4 elements).
__device__ __forceinline__ bool opt_vec_ok(const OptGroup& b, int t) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(b.p[t]) | reinterpret_cast<uintptr_t>(b.g[t]) |
                         reinterpret_cast<uintptr_t>(b.m[t]) | reinterpret_cast<uintptr_t>(b.v[t]) |
                         reinterpret_cast<uintptr_t>(b.ema[t]);
  return (bits & 15u) == 0;
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
  int64_t tail = begin;
  if ((reinterpret_cast<uintptr_t>(g) & 15u) == 0) {
    const int64_t end4 = begin + ((end - begin) & ~int64_t(3));
    for (int64_t i = begin + 4 * threadIdx.x; i < end4; i += 4 * kOptThreads) {
      const float4 v = *reinterpret_cast<const float4*>(g + i);
      s = fmaf(v.x, v.x, s);
      s = fmaf(v.y, v.y, s);
      s = fmaf(v.z, v.z, s);
      s = fmaf(v.w, v.w, s);
    }
    tail = end4;
  }
  for (int64_t i = tail + threadIdx.x; i < end; i += kOptThreads) s = fmaf(g[i], g[i], s);
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

// The per-step constants of the update.
struct AdamConsts {
  float coef, bc2_sqrt, step_size, decay, one_m_b1, beta2, one_m_b2, eps, ema_beta, one_m_ema;
};

// One element: clip, decoupled decay, moments, step, then the EMA of the new weight.
__device__ __forceinline__ void adamw_ema_elem(const AdamConsts& k, float& p, float g, float& m, float& v, float* e) {
  const float gi = g * k.coef;
  float pi = p * k.decay;
  float mi = fmaf(k.one_m_b1, gi - m, m);
  const float vi = fmaf(v, k.beta2, k.one_m_b2 * gi * gi);
  pi -= k.step_size * mi / (sqrtf(vi) / k.bc2_sqrt + k.eps);
  p = pi;
  m = mi;
  v = vi;
  if (e != nullptr) *e = __fadd_rn(__fmul_rn(*e, k.ema_beta), __fmul_rn(k.one_m_ema, pi));
}

__global__ void __launch_bounds__(kOptThreads) opt_update_kernel(OptGroup b, OptHyper h) {
  pdl_wait();
  const int k = blockIdx.x;
  const int t = opt_tensor_of(b, k);
  const int64_t begin = static_cast<int64_t>(k - b.chunk_begin[t]) * kOptChunk;
  const int64_t end = min(begin + kOptChunk, b.n[t]);
  const float step = *h.step;
  AdamConsts c;
  c.coef = *h.coef;
  c.bc2_sqrt = sqrtf(1.0f - powf(h.beta2, step));
  c.step_size = h.lr / (1.0f - powf(h.beta1, step));
  c.decay = 1.0f - h.lr * h.weight_decay;
  c.one_m_b1 = 1.0f - h.beta1;
  c.beta2 = h.beta2;
  c.one_m_b2 = 1.0f - h.beta2;
  c.eps = h.eps;
  c.ema_beta = h.ema_beta;
  c.one_m_ema = 1.0f - h.ema_beta;
  float* __restrict__ p = b.p[t];
  const float* __restrict__ g = b.g[t];
  float* __restrict__ m = b.m[t];
  float* __restrict__ v = b.v[t];
  float* __restrict__ e = b.ema[t];
  int64_t tail = begin;
  if (opt_vec_ok(b, t)) {  // uniform over the CTA
    const int64_t end4 = begin + ((end - begin) & ~int64_t(3));
    for (int64_t i = begin + 4 * threadIdx.x; i < end4; i += 4 * kOptThreads) {
      float4 pv = *reinterpret_cast<const float4*>(p + i);
      const float4 gv = *reinterpret_cast<const float4*>(g + i);
      float4 mv = *reinterpret_cast<const float4*>(m + i);
      float4 vv = *reinterpret_cast<const float4*>(v + i);
      float4 ev = e != nullptr ? *reinterpret_cast<const float4*>(e + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      float* ep = e != nullptr ? &ev.x : nullptr;
      adamw_ema_elem(c, pv.x, gv.x, mv.x, vv.x, ep);
      adamw_ema_elem(c, pv.y, gv.y, mv.y, vv.y, ep ? &ev.y : nullptr);
      adamw_ema_elem(c, pv.z, gv.z, mv.z, vv.z, ep ? &ev.z : nullptr);
      adamw_ema_elem(c, pv.w, gv.w, mv.w, vv.w, ep ? &ev.w : nullptr);
      *reinterpret_cast<float4*>(p + i) = pv;
      *reinterpret_cast<float4*>(m + i) = mv;
      *reinterpret_cast<float4*>(v + i) = vv;
      if (e != nullptr) *reinterpret_cast<float4*>(e + i) = ev;
    }
    tail = end4;
  }
  for (int64_t i = tail + threadIdx.x; i < end; i += kOptThreads) {
    float pi = p[i], mi = m[i], vi = v[i];
    adamw_ema_elem(c, pi, g[i], mi, vi, e != nullptr ? e + i : nullptr);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
  }
}

}  // namespace fp8b

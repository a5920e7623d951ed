// groupnorm.cuh — GroupNorm + optional FiLM + SiLU + optional dropout, forward and
// backward, on NHWC bf16 activations (the UNet's norm -> activation chains that
// feed its 3x3 convs, reference unet.py:151 and :157-159).
//
// Forward, per sample n, channel c (group g = c / Cg, m = HW * Cg elements per group):
//   z = (x - mean_g) * rstd_g * gamma_c + beta_c          (nn.GroupNorm, eps inside rstd)
//   f = (s_nc + 1) * z + t_nc                             (FiLM, optional: s, t from the time embedding)
//   a = silu(f) * keep / (1 - p)                          (dropout, optional)
// which is one affine map per (n, c): f = A_nc * x + B_nc.
//
// Kernels (grid = samples x slices; a CTA owns a contiguous pixel range of one
// sample; thread (v, r) handles channel vector v (8 channels, 16 bytes) of
// pixels r, r + R, ...; C <= 512):
//   gn_stats_kernel     : per-channel sums of (x - x[n, 0, c]) and its square per slice
//   gn_act_fwd_kernel   : merges the slices' sums into per-group mean / rstd (Chan's
//                         pairwise update, so channels with different shifts combine
//                         without cancellation), writes them (slice 0) and applies the map
//   gn_act_bwd_reduce_kernel : recomputes f from x and the saved statistics; per-channel
//                         sums of df, df * z and df * xhat per slice (df = dL/df)
//   gn_act_bwd_apply_kernel  : dx = rstd * (gamma (s+1) df - mean_g[gamma (s+1) df]
//                              - xhat * mean_g[gamma (s+1) df xhat]),
//                         and the per-(n, c) totals the host turns into the parameter,
//                         scale and shift gradients.
// x (and dx) may be bf16 or fp32; the activation and its gradient are bf16.
// Dropout keeps element e when a 16-bit slice of splitmix64(seed, e / 4) is >= p * 65536
// (splitmix64: Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014); the seed is read from device memory so a captured
// graph draws a new mask each replay when the caller advances it.
#pragma once

#include "quantize.cuh"
#include "sm100_common.cuh"

namespace fp8b {

#ifndef FP8_GN_THREADS
#define FP8_GN_THREADS 512
#endif
#ifndef FP8_GN_UF
#define FP8_GN_UF 4
#endif
#ifndef FP8_GN_UB
#define FP8_GN_UB 2
#endif
#ifndef FP8_GN_MINB_BWD
#define FP8_GN_MINB_BWD 1
#endif
#ifndef FP8_GN_MINB_FWD
#define FP8_GN_MINB_FWD 1
#endif
constexpr int kGnThreads = FP8_GN_THREADS;
constexpr int kGnUnrollFwd = FP8_GN_UF;  // pixel rows per step, forward kernels
constexpr int kGnUnrollBwd = FP8_GN_UB;  // pixel rows per step, backward kernels

struct GnShape {
  int n, hw, c, groups;
  int slices;       // CTAs per sample of this kernel
  int part_slices;  // CTAs per sample of the kernel that wrote the partial sums this kernel reads
};

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Keep mask bits for the 8 elements starting at linear NHWC index e0 (e0 % 8 == 0).
__device__ __forceinline__ uint32_t dropout_keep8(uint64_t seed, int64_t e0, uint32_t thresh16) {
  uint32_t keep = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint64_t r = splitmix64(seed ^ (static_cast<uint64_t>(e0 / 4 + h) * 0xD1B54A32D192ED03ull));
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (static_cast<uint32_t>((r >> (16 * k)) & 0xFFFFu) >= thresh16) keep |= 1u << (h * 4 + k);
  }
  return keep;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_lo_f(w[i]);
    f[2 * i + 1] = bf16_hi_f(w[i]);
  }
}

// v rounded to the storage type TX (bf16: round to nearest even; fp32: unchanged).
template <typename TX>
__device__ __forceinline__ float round_to_x(float v) {
  if constexpr (sizeof(TX) == 2) return __uint_as_float(pack_bf16x2(v, 0.0f) << 16);
  return v;
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// Eight consecutive channels of x, stored as bf16 (uint16_t) or fp32: the
// reference runs GroupNorm on whatever its input is (fp32 after autocast's fp32
// resampling, bf16 after a conv), so both element types are accepted.
template <typename TX>
struct XVec;
template <>
struct XVec<uint16_t> {
  uint4 v;
};
template <>
struct XVec<float> {
  float4 a, b;
};

template <typename TX>
__device__ __forceinline__ XVec<TX> load_x8(const TX* __restrict__ x, int64_t vi) {
  XVec<TX> r;
  if constexpr (sizeof(TX) == 2) {
    r.v = __ldg(reinterpret_cast<const uint4*>(x) + vi);
  } else {
    r.a = __ldg(reinterpret_cast<const float4*>(x) + 2 * vi);
    r.b = __ldg(reinterpret_cast<const float4*>(x) + 2 * vi + 1);
  }
  return r;
}

template <typename TX>
__device__ __forceinline__ XVec<TX> zero_x8() {
  XVec<TX> r;
  if constexpr (sizeof(TX) == 2) {
    r.v = make_uint4(0u, 0u, 0u, 0u);
  } else {
    r.a = make_float4(0.f, 0.f, 0.f, 0.f);
    r.b = r.a;
  }
  return r;
}

template <typename TX>
__device__ __forceinline__ void unpack_x8(const XVec<TX>& r, float (&f)[8]) {
  if constexpr (sizeof(TX) == 2) {
    unpack8(r.v, f);
  } else {
    f[0] = r.a.x; f[1] = r.a.y; f[2] = r.a.z; f[3] = r.a.w;
    f[4] = r.b.x; f[5] = r.b.y; f[6] = r.b.z; f[7] = r.b.w;
  }
}

template <typename TX>
__device__ __forceinline__ void store_x8(TX* __restrict__ x, int64_t vi, const float (&f)[8]) {
  if constexpr (sizeof(TX) == 2) {
    reinterpret_cast<uint4*>(x)[vi] = pack8(f);
  } else {
    reinterpret_cast<float4*>(x)[2 * vi] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(x)[2 * vi + 1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

template <typename TX>
__device__ __forceinline__ float load_x1(const TX* __restrict__ x, int64_t i) {
  if constexpr (sizeof(TX) == 2) {
    return __uint_as_float(static_cast<uint32_t>(x[i]) << 16);
  } else {
    return x[i];
  }
}

// Thread layout shared by all four kernels.
struct GnThread {
  int vecs;   // C / 8 channel vectors per pixel
  int rows;   // pixel rows per CTA step (kGnThreads / vecs)
  int v, r;   // this thread's channel vector and row (r >= rows: idle in the streaming loops)
  int p0, p1; // pixel range of this CTA
  int n;      // sample
};

__device__ __forceinline__ GnThread gn_thread(const GnShape& s) {
  GnThread t;
  t.vecs = s.c / 8;
  t.rows = kGnThreads / t.vecs;
  t.v = threadIdx.x % t.vecs;
  t.r = threadIdx.x / t.vecs;
  t.n = blockIdx.x / s.slices;
  const int slice = blockIdx.x % s.slices;
  const int per = (s.hw + s.slices - 1) / s.slices;
  t.p0 = min(s.hw, slice * per);
  t.p1 = min(s.hw, t.p0 + per);
  return t;
}

// Sum `vals[j]` (j < NV) of every thread with the same channel vector into
// red[j * C + c], in a fixed order (deterministic).  buf: smem float[rows][NV][C];
// red: smem float[NV][C].  Ends with a __syncthreads.
template <int NV>
__device__ __forceinline__ void gn_reduce_rows(const GnThread& t, const GnShape& s, const float (*vals)[8],
                                               float* buf, float* red) {
  if (t.r < t.rows) {
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) buf[(t.r * NV + j) * s.c + t.v * 8 + k] = vals[j][k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NV * s.c; i += blockDim.x) {
    float v = 0.0f;
    for (int r = 0; r < t.rows; ++r) v += buf[r * NV * s.c + i];
    red[i] = v;
  }
  __syncthreads();
}

// Dynamic shared memory (bytes) of each kernel for C channels and G groups.
__host__ __device__ constexpr size_t gn_reduce_smem(int c, int nv) {
  return static_cast<size_t>(kGnThreads / (c / 8)) * nv * c * 4 + static_cast<size_t>(nv) * c * 4;
}
__host__ __device__ constexpr size_t gn_stats_smem(int c) { return gn_reduce_smem(c, 2); }
__host__ __device__ constexpr size_t gn_fwd_smem(int c, int g) { return (2 * static_cast<size_t>(g) + 4 * c) * 4; }
__host__ __device__ constexpr size_t gn_bwd_reduce_smem(int c, int g) {
  return (2 * static_cast<size_t>(c) + 2 * g) * 4 + gn_reduce_smem(c, 2);
}
__host__ __device__ constexpr size_t gn_bwd_apply_smem(int c, int g) {
  return (5 * static_cast<size_t>(c) + 4 * g) * 4;
}

// ------------------------------------------------------------------ statistics
// part[(n * slices + slice) * 2C + {0, C} + c] = sum (x - shift_c), sum (x - shift_c)^2
template <typename TX>
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(const TX* __restrict__ x, GnShape s,
                                                              float* __restrict__ part) {
  extern __shared__ float gn_smem[];
  pdl_wait();
  const GnThread t = gn_thread(s);
  float acc[2][8] = {};
  if (t.r < t.rows) {
    const TX* xs = x + static_cast<int64_t>(t.n) * s.hw * s.c;
    float sh[8];
    unpack_x8(load_x8(xs, t.v), sh);
    // Four pixel rows per step: their loads are in flight together.
    for (int p = t.p0 + t.r; p < t.p1; p += kGnUnrollFwd * t.rows) {
      XVec<TX> v[kGnUnrollFwd];
#pragma unroll
      for (int u = 0; u < kGnUnrollFwd; ++u) {
        const int pu = p + u * t.rows;
        v[u] = pu < t.p1 ? load_x8(xs, static_cast<int64_t>(pu) * t.vecs + t.v) : zero_x8<TX>();
      }
#pragma unroll
      for (int u = 0; u < kGnUnrollFwd; ++u) {
        if (p + u * t.rows >= t.p1) break;
        float f[8];
        unpack_x8(v[u], f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = f[k] - sh[k];
          acc[0][k] += d;
          acc[1][k] = fmaf(d, d, acc[1][k]);
        }
      }
    }
  }
  float* red = gn_smem + static_cast<size_t>(t.rows) * 2 * s.c;
  gn_reduce_rows<2>(t, s, acc, gn_smem, red);
  float* out = part + static_cast<int64_t>(blockIdx.x) * 2 * s.c;
  for (int i = threadIdx.x; i < 2 * s.c; i += blockDim.x) out[i] = red[i];
}

// Per-group mean / rstd of sample n from the slices' partial sums (all threads call;
// result in smem mean_g[G], rstd_g[G]).  shift_c = x[n, 0, c].
template <typename TX>
__device__ __forceinline__ void gn_group_stats(const TX* __restrict__ x, const float* __restrict__ part,
                                               const GnShape& s, int n, float eps, float* mean_g, float* rstd_g,
                                               float* ch_mean, float* ch_m2) {
  const float cnt = static_cast<float>(s.hw);
  for (int c = threadIdx.x; c < s.c; c += blockDim.x) {
    float s1 = 0.0f, s2 = 0.0f;
    for (int k = 0; k < s.part_slices; ++k) {
      const float* pp = part + (static_cast<int64_t>(n) * s.part_slices + k) * 2 * s.c;
      s1 += pp[c];
      s2 += pp[s.c + c];
    }
    const float shift = load_x1(x, static_cast<int64_t>(n) * s.hw * s.c + c);
    ch_mean[c] = shift + s1 / cnt;
    ch_m2[c] = fmaxf(s2 - s1 * s1 / cnt, 0.0f);
  }
  __syncthreads();
  const int cg = s.c / s.groups;
  for (int g = threadIdx.x; g < s.groups; g += blockDim.x) {
    float mean = 0.0f;
    for (int j = 0; j < cg; ++j) mean += ch_mean[g * cg + j];
    mean /= static_cast<float>(cg);
    float m2 = 0.0f;
    for (int j = 0; j < cg; ++j) {
      const float d = ch_mean[g * cg + j] - mean;
      m2 += ch_m2[g * cg + j] + cnt * d * d;
    }
    mean_g[g] = mean;
    rstd_g[g] = rsqrtf(m2 / (cnt * static_cast<float>(cg)) + eps);
  }
  __syncthreads();
}

struct GnActParams {
  const float* gamma;   // [C]
  const float* beta;    // [C]
  const uint16_t* film; // bf16 [N][film_ld]: scale at +0, shift at +C (nullptr: no FiLM)
  int film_ld;
  const int64_t* seed;  // device seed (nullptr: no dropout)
  float p;              // dropout probability
  float eps;
};

// Per-(n, c) affine map f = A x + B into smem A[C], B[C] (also z = a x + b for backward).
__device__ __forceinline__ void gn_coeffs(const GnShape& s, const GnActParams& q, int n, const float* mean_g,
                                          const float* rstd_g, float* A, float* B, float* a_z, float* b_z) {
  const int cg = s.c / s.groups;
  for (int c = threadIdx.x; c < s.c; c += blockDim.x) {
    const int g = c / cg;
    const float a = q.gamma[c] * rstd_g[g];
    const float b = q.beta[c] - mean_g[g] * a;
    float sc = 1.0f, sh = 0.0f;
    if (q.film != nullptr) {
      const uint16_t* fr = q.film + static_cast<int64_t>(n) * q.film_ld;
      sc += __uint_as_float(static_cast<uint32_t>(fr[c]) << 16);
      sh = __uint_as_float(static_cast<uint32_t>(fr[s.c + c]) << 16);
    }
    A[c] = sc * a;
    B[c] = fmaf(sc, b, sh);
    if (a_z != nullptr) {
      a_z[c] = a;
      b_z[c] = b;
    }
  }
  __syncthreads();
}

// stats[n * 2G + {0, G} + g] = mean, rstd (written by slice 0 of each sample).
// Output of the apply pass.  QUANT = false: the bf16 activations.  QUANT =
// true (the input of a delayed-scaling FP8 conv): their e4m3 bytes, cast with
// the previous scale exactly as the delayed quantize pass casts a bf16 tensor
// (reference quantize_fp8_delayed, fp8_kernels.py:518-556), and each CTA's max
// |bf16 activation| for the current scale; the bf16 tensor is never written.
struct GnOut {
  uint16_t* bf16;           // NHWC bf16 (QUANT = false)
  uint8_t* q;               // NHWC e4m3 (QUANT = true)
  DelayedSource prev_scale;  // the scale of the cast (QUANT = true)
  float* amax_part;         // [grid] per-CTA max |activation| (QUANT = true)
  ScaleFold fold;           // the last CTA folds amax_part into the current scale (QUANT = true)
};

// Plain bf16 stores: the Div of the non-quantizing instantiation.
struct NoCast {};

// The streaming loop of the apply pass over this thread's pixel rows; returns
// the packed max |bf16 activation| (QUANT) or 0.
template <typename TX, bool QUANT, bool DROP, class Div>
__device__ __forceinline__ uint32_t gn_apply_rows(const TX* __restrict__ xs, const GnThread& t, int64_t base,
                                                  const float (&a)[8], const float (&b)[8], uint64_t seed,
                                                  uint32_t thresh, float keep_scale, const GnOut& o, const Div& div) {
  uint32_t m2 = 0u;
  for (int p = t.p0 + t.r; p < t.p1; p += kGnUnrollFwd * t.rows) {
    XVec<TX> v[kGnUnrollFwd];
#pragma unroll
    for (int u = 0; u < kGnUnrollFwd; ++u) {
      const int pu = p + u * t.rows;
      v[u] = pu < t.p1 ? load_x8(xs, static_cast<int64_t>(pu) * t.vecs + t.v) : zero_x8<TX>();
    }
#pragma unroll
    for (int u = 0; u < kGnUnrollFwd; ++u) {
      const int pu = p + u * t.rows;
      if (pu >= t.p1) break;
      const int64_t vi = static_cast<int64_t>(pu) * t.vecs + t.v;
      float f[8];
      unpack_x8(v[u], f);
      const uint32_t keep = DROP ? dropout_keep8(seed, (base + vi) * 8, thresh) : 0xFFu;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float act = silu_f32(fmaf(a[k], f[k], b[k]));
        if constexpr (DROP)
          f[k] = (keep >> k) & 1u ? act * keep_scale : 0.0f;
        else
          f[k] = act;
      }
      const uint4 h = pack8(f);
      if constexpr (QUANT) {
        m2 = bf16x2_max(m2, absmax_vec2(h));
        reinterpret_cast<uint2*>(o.q)[base + vi] = cast_vec(h, div);
      } else {
        reinterpret_cast<uint4*>(o.bf16)[base + vi] = h;
      }
    }
  }
  return m2;
}

template <typename TX, bool QUANT, bool DROP>
__global__ void __launch_bounds__(kGnThreads, FP8_GN_MINB_FWD) gn_act_fwd_kernel(const TX* __restrict__ x, GnShape s,
                                                                const float* __restrict__ part, GnActParams q,
                                                                float* __restrict__ stats, GnOut o) {
  extern __shared__ float gn_smem[];
  pdl_wait();
  float* mean_g = gn_smem;
  float* rstd_g = mean_g + s.groups;
  float* A = rstd_g + s.groups;
  float* B = A + s.c;
  float* ch_mean = B + s.c;
  float* ch_m2 = ch_mean + s.c;
  const GnThread t = gn_thread(s);
  gn_group_stats(x, part, s, t.n, q.eps, mean_g, rstd_g, ch_mean, ch_m2);
  if (blockIdx.x % s.slices == 0)
    for (int g = threadIdx.x; g < s.groups; g += blockDim.x) {
      stats[static_cast<int64_t>(t.n) * 2 * s.groups + g] = mean_g[g];
      stats[static_cast<int64_t>(t.n) * 2 * s.groups + s.groups + g] = rstd_g[g];
    }
  // the delayed scale first: with a scale history every thread takes part in its max
  float sc = 1.0f;
  if constexpr (QUANT) sc = delayed_scale<kGnThreads>(o.prev_scale);
  gn_coeffs(s, q, t.n, mean_g, rstd_g, A, B, nullptr, nullptr);
  uint32_t m2 = 0u;
  if (t.r < t.rows) {
    float a[8], b[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      a[k] = A[t.v * 8 + k];
      b[k] = B[t.v * 8 + k];
    }
    const uint64_t seed = DROP ? static_cast<uint64_t>(*q.seed) : 0ull;
    const uint32_t thresh = static_cast<uint32_t>(q.p * 65536.0f);
    const float keep_scale = DROP ? 1.0f / (1.0f - q.p) : 1.0f;
    const int64_t base = static_cast<int64_t>(t.n) * s.hw * t.vecs;
    const TX* xs = x + base * 8;
    if constexpr (QUANT) {
      // the scale is uniform over the grid, so the choice never diverges
      m2 = markstein_applies(sc)
               ? gn_apply_rows<TX, true, DROP>(xs, t, base, a, b, seed, thresh, keep_scale, o, make_markstein(sc))
               : gn_apply_rows<TX, true, DROP>(xs, t, base, a, b, seed, thresh, keep_scale, o, DivF64(sc));
    } else {
      gn_apply_rows<TX, false, DROP>(xs, t, base, a, b, seed, thresh, keep_scale, o, NoCast{});
    }
  }
  if constexpr (QUANT) {
    const float m = block_max<kGnThreads>(unpack_max2(m2));
    if (threadIdx.x == 0) o.amax_part[blockIdx.x] = m;
    fold_scale_if_last<kGnThreads>(o.amax_part, o.fold);
  }
}

// Per-thread constants of the backward passes for its 8 channels: the affine
// map f = a x + b and xhat = rs x + nmr (nmr = -mean * rs).
struct GnBwdCoeffs {
  float a[8], b[8], rs[8], nmr[8];
};

__device__ __forceinline__ void gn_bwd_coeffs(const GnThread& t, const GnShape& s, const float* A, const float* B,
                                              const float* mean_g, const float* rstd_g, GnBwdCoeffs& k) {
  const int cg = s.c / s.groups;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = t.v * 8 + j;
    const int g = c / cg;
    k.a[j] = A[c];
    k.b[j] = B[c];
    k.rs[j] = rstd_g[g];
    k.nmr[j] = -mean_g[g] * rstd_g[g];
  }
}

// df = dL/df for one element: the activation's derivative (silu' = sg (1 + f (1 - sg)))
// times the incoming gradient, scaled by the dropout keep factor when DROP.
template <bool DROP>
__device__ __forceinline__ float gn_df(float f, float g, uint32_t keep, int k, float keep_scale) {
  const float sg = sigmoid_f32(f);
  float du = g;
  if constexpr (DROP) du = (keep >> k) & 1u ? g * keep_scale : 0.0f;
  return du * sg * fmaf(f, 1.0f - sg, 1.0f);
}

// part[(n * slices + slice) * 2C + {0, C} + c] = sum df, sum df * xhat.  (The FiLM
// scale gradient's sum of df * z follows from these: z = gamma xhat + beta.)
template <typename TX, bool DROP>
__global__ void __launch_bounds__(kGnThreads, FP8_GN_MINB_BWD) gn_act_bwd_reduce_kernel(
    const TX* __restrict__ x, const uint16_t* __restrict__ dy, GnShape s, const float* __restrict__ stats,
    GnActParams q, float* __restrict__ part) {
  extern __shared__ float gn_smem[];
  pdl_wait();
  float* A = gn_smem;
  float* B = A + s.c;
  float* mean_g = B + s.c;
  float* rstd_g = mean_g + s.groups;
  float* buf = rstd_g + s.groups;
  const GnThread t = gn_thread(s);
  float* red = buf + static_cast<size_t>(t.rows) * 2 * s.c;
  for (int g = threadIdx.x; g < s.groups; g += blockDim.x) {
    mean_g[g] = stats[static_cast<int64_t>(t.n) * 2 * s.groups + g];
    rstd_g[g] = stats[static_cast<int64_t>(t.n) * 2 * s.groups + s.groups + g];
  }
  __syncthreads();
  gn_coeffs(s, q, t.n, mean_g, rstd_g, A, B, nullptr, nullptr);
  float acc[2][8] = {};
  if (t.r < t.rows) {
    GnBwdCoeffs k;
    gn_bwd_coeffs(t, s, A, B, mean_g, rstd_g, k);
    const uint64_t seed = DROP ? static_cast<uint64_t>(*q.seed) : 0ull;
    const uint32_t thresh = static_cast<uint32_t>(q.p * 65536.0f);
    const float keep_scale = DROP ? 1.0f / (1.0f - q.p) : 1.0f;
    const int64_t base = static_cast<int64_t>(t.n) * s.hw * t.vecs;
    const TX* xs = x + base * 8;
    const uint4* ds = reinterpret_cast<const uint4*>(dy) + base;
    for (int p = t.p0 + t.r; p < t.p1; p += kGnUnrollBwd * t.rows) {
      XVec<TX> vx[kGnUnrollBwd];
      uint4 vd[kGnUnrollBwd];
#pragma unroll
      for (int u = 0; u < kGnUnrollBwd; ++u) {
        const int pu = p + u * t.rows;
        const int64_t vi = static_cast<int64_t>(pu) * t.vecs + t.v;
        vx[u] = pu < t.p1 ? load_x8(xs, vi) : zero_x8<TX>();
        vd[u] = pu < t.p1 ? __ldg(ds + vi) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kGnUnrollBwd; ++u) {
        const int pu = p + u * t.rows;
        if (pu >= t.p1) break;
        const int64_t vi = static_cast<int64_t>(pu) * t.vecs + t.v;
        float xf[8], gf[8];
        unpack_x8(vx[u], xf);
        unpack8(vd[u], gf);
        const uint32_t keep = DROP ? dropout_keep8(seed, (base + vi) * 8, thresh) : 0xFFu;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float df = gn_df<DROP>(fmaf(k.a[j], xf[j], k.b[j]), gf[j], keep, j, keep_scale);
          acc[0][j] += df;
          acc[1][j] = fmaf(df, fmaf(xf[j], k.rs[j], k.nmr[j]), acc[1][j]);
        }
      }
    }
  }
  gn_reduce_rows<2>(t, s, acc, buf, red);
  float* out = part + static_cast<int64_t>(blockIdx.x) * 2 * s.c;
  for (int i = threadIdx.x; i < 2 * s.c; i += blockDim.x) out[i] = red[i];
}

// Per-thread group terms of the backward apply for its 8 channels.
struct GnBwdGroup {
  float gk[8], m1[8], m2[8];
};

// The streaming loop of the backward apply over this thread's pixel rows.  QUANT:
// dx (bf16) is also cast to e4m3 with `div`; returns the packed max |dx|.
// dx_add (may be null): a second gradient of x, added to dx in x's dtype (the sum
// autograd forms when x has a second reader, e.g. the identity skip of a residual
// block): dx = RN(RN(dx_norm) + dx_add).
template <typename TX, bool DROP, bool QUANT, class Div>
__device__ __forceinline__ uint32_t gn_bwd_apply_rows(const TX* __restrict__ x, const uint16_t* __restrict__ dy,
                                                      const TX* __restrict__ dx_add, TX* __restrict__ dx,
                                                      const GnShape& s, const GnThread& t, const GnActParams& q,
                                                      const GnBwdCoeffs& k, const GnBwdGroup& gm, const GnOut& o,
                                                      const Div& div) {
  const uint64_t seed = DROP ? static_cast<uint64_t>(*q.seed) : 0ull;
  const uint32_t thresh = static_cast<uint32_t>(q.p * 65536.0f);
  const float keep_scale = DROP ? 1.0f / (1.0f - q.p) : 1.0f;
  const int64_t base = static_cast<int64_t>(t.n) * s.hw * t.vecs;
  const TX* xs = x + base * 8;
  const uint4* ds = reinterpret_cast<const uint4*>(dy) + base;
  const TX* as = dx_add != nullptr ? dx_add + base * 8 : nullptr;
  TX* os = dx + base * 8;
  uint32_t qm = 0u;
  for (int p = t.p0 + t.r; p < t.p1; p += kGnUnrollBwd * t.rows) {
    XVec<TX> vx[kGnUnrollBwd];
    uint4 vd[kGnUnrollBwd];
    XVec<TX> va[kGnUnrollBwd];
#pragma unroll
    for (int u = 0; u < kGnUnrollBwd; ++u) {
      const int pu = p + u * t.rows;
      const int64_t vi = static_cast<int64_t>(pu) * t.vecs + t.v;
      vx[u] = pu < t.p1 ? load_x8(xs, vi) : zero_x8<TX>();
      vd[u] = pu < t.p1 ? __ldg(ds + vi) : make_uint4(0u, 0u, 0u, 0u);
      va[u] = as != nullptr && pu < t.p1 ? load_x8(as, vi) : zero_x8<TX>();
    }
#pragma unroll
    for (int u = 0; u < kGnUnrollBwd; ++u) {
      const int pu = p + u * t.rows;
      if (pu >= t.p1) break;
      const int64_t vi = static_cast<int64_t>(pu) * t.vecs + t.v;
      float xf[8], gf[8], r[8];
      unpack_x8(vx[u], xf);
      unpack8(vd[u], gf);
      const uint32_t keep = DROP ? dropout_keep8(seed, (base + vi) * 8, thresh) : 0xFFu;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float df = gn_df<DROP>(fmaf(k.a[j], xf[j], k.b[j]), gf[j], keep, j, keep_scale);
        const float xhat = fmaf(xf[j], k.rs[j], k.nmr[j]);
        r[j] = k.rs[j] * (gm.gk[j] * df - gm.m1[j] - xhat * gm.m2[j]);
      }
      if (as != nullptr) {  // uniform over the grid
        float af[8];
        unpack_x8(va[u], af);
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = round_to_x<TX>(r[j]) + af[j];
      }
      if constexpr (QUANT) {
        const uint4 h = pack8(r);
        reinterpret_cast<uint4*>(os)[vi] = h;
        qm = bf16x2_max(qm, absmax_vec2(h));
        reinterpret_cast<uint2*>(o.q)[base + vi] = cast_vec(h, div);
      } else {
        store_x8(os, vi, r);
      }
    }
  }
  return qm;
}

// totals[n * 3C + {0, C, 2C} + c] = sum df, sum df z, sum df xhat over the sample
// (written by slice 0); dx = rstd * (gamma (s+1) df - mean_g[gamma (s+1) df]
// - xhat * mean_g[gamma (s+1) df xhat]).  QUANT (the input of a delayed-scaling
// FP8 conv's output gradient, x being that conv's bf16 output): dx is also cast to
// e4m3 with the delayed scale of o.prev_scale, exactly as the conv's backward
// quantize would cast it, and the last CTA folds the per-CTA max |dx| into dx's
// scale (o.fold).
template <typename TX, bool DROP, bool QUANT>
__global__ void __launch_bounds__(kGnThreads, FP8_GN_MINB_BWD) gn_act_bwd_apply_kernel(
    const TX* __restrict__ x, const uint16_t* __restrict__ dy, GnShape s, const float* __restrict__ stats,
    GnActParams q, const float* __restrict__ part, float* __restrict__ totals, TX* __restrict__ dx, GnOut o,
    const TX* __restrict__ dx_add) {
  static_assert(!QUANT || sizeof(TX) == 2, "the e4m3 dx is cast from a bf16 dx");
  extern __shared__ float gn_smem[];
  pdl_wait();
  // the delayed scale of the e4m3 dx first: with a scale history every thread takes part in its max
  float qs = 1.0f;
  if constexpr (QUANT) qs = delayed_scale<kGnThreads>(o.prev_scale);
  float* A = gn_smem;
  float* B = A + s.c;
  float* mean_g = B + s.c;
  float* rstd_g = mean_g + s.groups;
  float* tot = rstd_g + s.groups;  // [2][C]: sum df, sum df xhat
  float* g1 = tot + 2 * s.c;       // [G] mean over the group of gamma (s+1) df
  float* g2 = g1 + s.groups;       // [G] mean over the group of gamma (s+1) df xhat
  float* gs = g2 + s.groups;       // [C] gamma_c (s_nc + 1)
  const GnThread t = gn_thread(s);
  for (int g = threadIdx.x; g < s.groups; g += blockDim.x) {
    mean_g[g] = stats[static_cast<int64_t>(t.n) * 2 * s.groups + g];
    rstd_g[g] = stats[static_cast<int64_t>(t.n) * 2 * s.groups + s.groups + g];
  }
  __syncthreads();
  gn_coeffs(s, q, t.n, mean_g, rstd_g, A, B, nullptr, nullptr);
  const bool first = blockIdx.x % s.slices == 0;
  for (int i = threadIdx.x; i < 2 * s.c; i += blockDim.x) {
    float v = 0.0f;
    for (int k = 0; k < s.part_slices; ++k)
      v += part[(static_cast<int64_t>(t.n) * s.part_slices + k) * 2 * s.c + i];
    tot[i] = v;
  }
  for (int c = threadIdx.x; c < s.c; c += blockDim.x) {
    float sc = 1.0f;
    if (q.film != nullptr)
      sc += __uint_as_float(static_cast<uint32_t>(q.film[static_cast<int64_t>(t.n) * q.film_ld + c]) << 16);
    gs[c] = q.gamma[c] * sc;
  }
  __syncthreads();
  if (first)
    for (int c = threadIdx.x; c < s.c; c += blockDim.x) {
      float* tn = totals + static_cast<int64_t>(t.n) * 3 * s.c;
      tn[c] = tot[c];
      tn[s.c + c] = fmaf(q.gamma[c], tot[s.c + c], q.beta[c] * tot[c]);  // sum df z, z = gamma xhat + beta
      tn[2 * s.c + c] = tot[s.c + c];
    }
  const int cg = s.c / s.groups;
  const float inv_m = 1.0f / (static_cast<float>(s.hw) * static_cast<float>(cg));
  for (int g = threadIdx.x; g < s.groups; g += blockDim.x) {
    float s1 = 0.0f, s3 = 0.0f;
    for (int j = 0; j < cg; ++j) {
      const int c = g * cg + j;
      s1 = fmaf(gs[c], tot[c], s1);
      s3 = fmaf(gs[c], tot[s.c + c], s3);
    }
    g1[g] = s1 * inv_m;
    g2[g] = s3 * inv_m;
  }
  __syncthreads();
  uint32_t qm = 0u;
  if (t.r < t.rows) {
    GnBwdCoeffs k;
    gn_bwd_coeffs(t, s, A, B, mean_g, rstd_g, k);
    GnBwdGroup gm;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = t.v * 8 + j;
      const int g = c / cg;
      gm.gk[j] = gs[c];
      gm.m1[j] = g1[g];
      gm.m2[j] = g2[g];
    }
    if constexpr (QUANT) {
      qm = markstein_applies(qs)  // uniform over the grid
               ? gn_bwd_apply_rows<TX, DROP, true>(x, dy, dx_add, dx, s, t, q, k, gm, o, make_markstein(qs))
               : gn_bwd_apply_rows<TX, DROP, true>(x, dy, dx_add, dx, s, t, q, k, gm, o, DivF64(qs));
    } else {
      gn_bwd_apply_rows<TX, DROP, false>(x, dy, dx_add, dx, s, t, q, k, gm, o, NoCast{});
    }
  }
  if constexpr (QUANT) {
    const float m = block_max<kGnThreads>(unpack_max2(qm));
    if (threadIdx.x == 0) o.amax_part[blockIdx.x] = m;
    fold_scale_if_last<kGnThreads>(o.amax_part, o.fold);
  }
}

// Parameter gradients from the per-(n, c) totals of the backward:
//   dgamma_c = sum_n (s_nc + 1) * T[n][2C + c],  dbeta_c = sum_n (s_nc + 1) * T[n][c]
//   dfilm[n] = (T[n][C:2C], T[n][0:C]) as bf16     (the scale, then the shift gradient)
// with s = 0 and no dfilm without FiLM.  A CTA covers 32 channels with 32 lanes
// of samples (n = lane, lane + 32, ...; coalesced rows, four samples' loads in
// flight per thread), then two threads per channel sum the 32 lanes in order
// (deterministic).
constexpr int kGnParamLanes = 32;

__global__ void __launch_bounds__(32 * kGnParamLanes) gn_param_grads_kernel(
    const float* __restrict__ totals, const uint16_t* __restrict__ film, int film_ld, int n, int c,
    float* __restrict__ dgamma, float* __restrict__ dbeta, uint16_t* __restrict__ dfilm, int dfilm_ld) {
  __shared__ float red[2][kGnParamLanes][33];
  pdl_wait();
  const int cl = threadIdx.x & 31, lane = threadIdx.x >> 5;
  const int ch = blockIdx.x * 32 + cl;
  float g = 0.0f, b = 0.0f;
  if (ch < c) {
#pragma unroll 4
    for (int i = lane; i < n; i += kGnParamLanes) {
      const float* t = totals + static_cast<int64_t>(i) * 3 * c;
      const float t_df = t[ch], t_dfz = t[c + ch], t_dfx = t[2 * c + ch];
      float sc = 1.0f;
      if (film != nullptr) {
        sc += __uint_as_float(static_cast<uint32_t>(film[static_cast<int64_t>(i) * film_ld + ch]) << 16);
        uint16_t* d = dfilm + static_cast<int64_t>(i) * dfilm_ld;
        d[ch] = static_cast<uint16_t>(pack_bf16x2(t_dfz, 0.0f) & 0xFFFFu);
        d[c + ch] = static_cast<uint16_t>(pack_bf16x2(t_df, 0.0f) & 0xFFFFu);
      }
      g = fmaf(sc, t_dfx, g);
      b = fmaf(sc, t_df, b);
    }
  }
  red[0][lane][cl] = g;
  red[1][lane][cl] = b;
  __syncthreads();
  if (lane < 2 && ch < c) {  // lane 0: dgamma, lane 1: dbeta
    float sum = 0.0f;
#pragma unroll
    for (int l = 0; l < kGnParamLanes; ++l) sum += red[lane][l][cl];
    (lane == 0 ? dgamma : dbeta)[ch] = sum;
  }
}

}  // namespace fp8b

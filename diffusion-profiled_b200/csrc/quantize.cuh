// quantize.cuh — per-tensor e4m3 quantisation kernels (bandwidth bound).
//
// Semantics restated from the reference (diffusion/fp8_kernels.py):
//   amax      = max |x|                                   (:54-64, partial_amax_kernel)
//   scale     = amax > 0 ? amax / 448 : 1.0   (fp32)      (:90-102, finalize_amax_kernel)
//   q         = e4m3(max(-448, min(x / scale, 448)))      (:105-120, quantize_fp8_kernel)
// The clamp uses min-then-max with non-NaN-propagating fminf/fmaxf (the
// reference's tl.minimum / tl.maximum defaults), so x/0 = NaN clamps to +448.
// x / scale is the IEEE round-to-nearest fp32 quotient (computed exactly
// without a divide per element, see CastMarkstein and DivF64) and the cast is
// cvt.rn.satfinite.e4m3x2.f32, which makes the bytes reproducible on the CPU.
//
// Current scaling (quantize_fp8, :559-601) is two launches:
//   amax pass : |x| max, one fp32 partial per CTA
//   cast pass : every CTA folds the partials into amax and the scale (the
//               reference's separate finalize launch disappears), CTA 0
//               publishes the scale, then casts.
// Delayed scaling (quantize_fp8_delayed, :518-556) is one pass:
//   cast pass : cast with the previous scale, one amax partial per CTA; the
//               last CTA to finish folds the partials into the current scale
//               (fold_scale_if_last)
// Each pass exists twice: quant_stream_kernel (bulk copies through shared
// memory; 16-byte aligned x, 8-byte aligned q) and the scalar grid-stride
// amax_partials_kernel / quantize_cast_kernel for any other alignment.
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

// Two ways to get the e4m3 byte of x / s without an fp32 divide per element.
// Both give the byte of the IEEE round-to-nearest fp32 quotient for every bf16
// x; the kernel picks one per launch from s alone.
//
// DivF64 (any s).  With r = RN64(1/s) the double product RN64(x * r) is within
// about 2^-52 (relative) of the exact quotient.  x is a bf16 value (integer
// significand A < 2^8) and s an fp32 value (integer significand B < 2^24), so
// the exact quotient is either an fp32 number or stays away from every fp32
// rounding midpoint M = odd * 2^-p of its binade: |A/B - M| = |A*2^p - odd*B| /
// (B*2^p) has a non-zero integer numerator, so it is at least 1/(B*2^p), which
// is at least 2^-25/B > 2^-49 of M.  A double within 2^-52 of the quotient is
// thus on the same side of every midpoint and rounds to the same fp32 value:
// __double2float_rn(x * r) == IEEE x / s.  (Below 2^-126 the fp32 grid is
// coarser; such quotients become e4m3 zero either way.)  Scales of 0, inf and
// NaN behave as IEEE division does (r = inf, 0, NaN).  Costs two fp64
// conversions per element, which bound the cast kernel's throughput.
struct DivF64 {
  double r;
  __device__ __forceinline__ explicit DivF64(float s) : r(1.0 / static_cast<double>(s)) {}
  __device__ __forceinline__ float operator()(float x) const {
    return __double2float_rn(static_cast<double>(x) * r);
  }
  __device__ __forceinline__ uint32_t word(uint32_t w) const;
};

// Packed helpers: two bf16 in a 32-bit word (min/max return the other operand
// when one is NaN), two fp32 in one instruction (sm_100 f32x2 arithmetic).
__device__ __forceinline__ uint32_t bf16x2_min(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float2 f32x2_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f32x2_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// CastMarkstein (2^-60 <= s <= 2^100, i.e. every scale amax / 448 of a tensor
// whose amax lies in [2^-51, 2^108]).  Per pair of bf16:
//  1. clamp x to [-L, L] with bf16 min then max, where L is s * 1024 rounded up
//     to bf16.  Values beyond L have |x / s| > 1024 and saturate either way,
//     and a NaN x becomes L, so +448, as min(NaN / s, 448) does.  After this
//     the quotient is finite and below 2^11.
//  2. Markstein's correction step (P. Markstein, IBM J. Res. Dev. 34(1), 1990):
//     with r = RN32(1/s), q0 = RN32(x * r), e = fma(q0, -s, x) (exact),
//     q1 = RN32(q0 + e * r) is the correctly rounded quotient while
//     |q0| >= 2^-11, where e stays normal.
//  3. |q1| takes the sign of x: below 2^-11 the quotient becomes an e4m3 zero
//     whose sign is that of x (q1 alone can lose it: -0 / s gives q1 = +0).
//  4. cvt.rn.satfinite saturates |q1| >= 448 to +-448, as the clamp does.
// The sequence is checked against IEEE division and the reference clamp on the
// CPU: every (bf16 significand, fp32 significand) pair, exponents at the edges
// of the scale range, and all 65,536 bf16 bit patterns against sampled scales.
struct CastMarkstein {
  float2 r2, ns2;      // (r, r), (-s, -s)
  uint32_t lb2, nlb2;  // (L, L), (-L, -L) as bf16x2
  // Two bf16 -> two e4m3 bytes in the low 16 bits.
  __device__ __forceinline__ uint32_t word(uint32_t w) const {
    const uint32_t c = bf16x2_max(bf16x2_min(w, lb2), nlb2);
    const uint32_t lo = c << 16, hi = c & 0xFFFF0000u;
    const float2 x = make_float2(__uint_as_float(lo), __uint_as_float(hi));
    const float2 q0 = f32x2_mul(x, r2);
    const float2 e = f32x2_fma(q0, ns2, x);
    const float2 q1 = f32x2_fma(e, r2, q0);
    const float t0 = __uint_as_float((__float_as_uint(q1.x) & 0x7FFFFFFFu) | (lo & 0x80000000u));
    const float t1 = __uint_as_float((__float_as_uint(q1.y) & 0x7FFFFFFFu) | (hi & 0x80000000u));
    return cvt_e4m3x2(t0, t1);
  }
};

__device__ __forceinline__ bool markstein_applies(float s) { return s >= 0x1p-60f && s <= 0x1p100f; }
__device__ __forceinline__ CastMarkstein make_markstein(float s) {
  CastMarkstein c;
  const float r = __fdiv_rn(1.0f, s);
  c.r2 = make_float2(r, r);
  c.ns2 = make_float2(-s, -s);
  const uint32_t lb = ((__float_as_uint(s * 1024.0f) + 0xFFFFu) >> 16) & 0xFFFFu;  // round up to bf16
  c.lb2 = lb | (lb << 16);
  c.nlb2 = c.lb2 | 0x80008000u;
  return c;
}

__device__ __forceinline__ float scale_and_clamp(float v, const DivF64& div) {
  float t = div(v);
  t = fminf(t, kE4M3Max);      // tl.minimum(scaled, FP8_MAX)
  return fmaxf(-kE4M3Max, t);  // tl.maximum(-FP8_MAX, .)
}

__device__ __forceinline__ uint32_t DivF64::word(uint32_t w) const {
  return cvt_e4m3x2(scale_and_clamp(bf16_lo_f(w), *this), scale_and_clamp(bf16_hi_f(w), *this));
}

// Max of a non-negative value over threads 0 .. NT-1; result valid in each of them.
// BAR = 0: all NT threads of the block (__syncthreads); BAR > 0: named barrier BAR over
// the first NT threads only (the others may be busy elsewhere, e.g. a producer warp).
template <int NT = kQuantThreads, int BAR = 0>
__device__ __forceinline__ float block_max(float v) {
  static_assert(NT % 32 == 0 && NT <= 1024, "block size");
  __shared__ float red[NT / 32];
  __shared__ float result;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  if (BAR == 0) __syncthreads(); else named_barrier_sync(BAR, NT);
  if (warp == 0) {
    float w = lane < (NT / 32) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) result = w;
  }
  if (BAR == 0) __syncthreads(); else named_barrier_sync(BAR, NT);
  return result;
}

__device__ __forceinline__ float scale_from_amax(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, kE4M3Max) : 1.0f;
}

// The scale a delayed cast divides by: *prev, or -- when window != nullptr --
// the max of window[0 .. len), the reference's torch.max over a module's scale
// history (unet.py:69-91, fp8_kernels.py:841-853), which CTA 0 also writes to
// *used (the dequantisation scale of the cast bytes, read by the contraction
// that consumes them).  Every thread of the CTA must call delayed_scale().
struct DelayedSource {
  const float* prev;
  const float* window;
  int len;
  float* used;
};

// The history update after a delayed cast: window[*pos] = this tensor's scale,
// then (advance) *pos = (*pos + 1) % len -- the scatter and the position step of
// the reference module (unet.py:80-91), done by the CTA that folds the scale.
struct WindowUpdate {
  float* window;
  int64_t* pos;
  int len;
  int advance;
  // 0: the reference's entry for an all-zero tensor (its scale, 1.0); 1: 0.0,
  // so that such a tensor adds nothing to the history's max
  int empty_zero;
};

// The history entry of a tensor with this amax.
__device__ __forceinline__ float history_entry(float amax, int empty_zero) {
  return (empty_zero && !(amax > 0.0f)) ? 0.0f : scale_from_amax(amax);
}

// Fold `count` partial maxima into the tensor scale (every CTA does this; the
// partials are a few KB and L2 resident).
template <int NT = kQuantThreads, int BAR = 0>
__device__ __forceinline__ float fold_partials_to_scale(const float* __restrict__ partials, int count) {
  float m = 0.0f;
  for (int i = threadIdx.x; i < count; i += NT) m = fmaxf(m, partials[i]);
  return scale_from_amax(block_max<NT, BAR>(m));
}

template <int NT = kQuantThreads, int BAR = 0>
__device__ __forceinline__ float delayed_scale(const DelayedSource& d) {
  if (d.window == nullptr) return *d.prev;  // uniform over the grid
  float m = 0.0f;
  for (int i = threadIdx.x; i < d.len; i += NT) m = fmaxf(m, d.window[i]);
  m = block_max<NT, BAR>(m);
  if (d.used != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *d.used = m;
  return m;
}

// |x| maxima kept packed: two running bf16 maxima per 32-bit word (clearing
// the sign bits is |.|; bf16x2 max skips NaN like fmaxf).  Exact: a max of
// bf16 values is one of them.
constexpr uint32_t kAbsMask2 = 0x7FFF7FFFu;

// max |.| of the 8 bf16 of a 16-byte vector (a depth-2 tree).
__device__ __forceinline__ uint32_t absmax_vec2(const uint4& a) {
  return bf16x2_max(bf16x2_max(a.x & kAbsMask2, a.y & kAbsMask2), bf16x2_max(a.z & kAbsMask2, a.w & kAbsMask2));
}

__device__ __forceinline__ float unpack_max2(uint32_t m2) { return fmaxf(bf16_lo_f(m2), bf16_hi_f(m2)); }

template <class Div>
__device__ __forceinline__ uint32_t cast4(uint32_t w0, uint32_t w1, const Div& d) {
  return d.word(w0) | (d.word(w1) << 16);
}

template <class Div>
__device__ __forceinline__ uint2 cast_vec(const uint4& a, const Div& d) {
  return make_uint2(cast4(a.x, a.y, d), cast4(a.z, a.w, d));
}

// The tensor's own scale, folded by the last CTA of the launch that wrote the
// partial maxima (no separate one-CTA launch).  Every CTA stores its partial,
// fences, and takes a ticket from `counter`; the CTA with the last ticket sees
// every partial (each was fenced before its ticket), folds them into the scale,
// stores it to *scale_out and into the history (`wu`), and sets the counter back
// to zero for the next launch that is given it.  No CTA waits for another.
struct ScaleFold {
  unsigned int* counter;  // zero when the launch starts; zero again when it ends
  float* scale_out;       // may be null
  WindowUpdate wu;        // window == null: no history update
};

__device__ __forceinline__ void store_scale(float amax, float* scale_out, const WindowUpdate& wu) {
  if (scale_out != nullptr) *scale_out = scale_from_amax(amax);
  if (wu.window != nullptr) {
    const int64_t p = *wu.pos;
    wu.window[p] = history_entry(amax, wu.empty_zero);
    if (wu.advance) *wu.pos = (p + 1) % wu.len;
  }
}

// Every thread of every CTA, after thread 0 stored partials[blockIdx.x].
template <int NT>
__device__ __forceinline__ void fold_scale_if_last(const float* partials, const ScaleFold& f) {
  __shared__ unsigned int ticket;
  if (threadIdx.x == 0) {
    __threadfence();
    ticket = atomicAdd(f.counter, 1u);
  }
  __syncthreads();
  if (ticket != gridDim.x - 1) return;  // uniform over the CTA
  __threadfence();
  float m = 0.0f;
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += NT) m = fmaxf(m, __ldcg(partials + i));
  const float amax = block_max<NT>(m);
  if (threadIdx.x == 0) {
    store_scale(amax, f.scale_out, f.wu);
    *f.counter = 0u;
  }
}

// ---------------------------------------------------------------- scalar passes
// Grid-stride, one element per thread and step: the path for x that is not
// 16-byte aligned or q that is not 8-byte aligned (views with an odd offset).
// Aligned tensors take the streaming passes below.

// Pass 1 of current scaling: |x| max per CTA.
__global__ void __launch_bounds__(kQuantThreads) amax_partials_kernel(const uint16_t* __restrict__ x, int64_t n,
                                                                      float* __restrict__ partials) {
  pdl_wait();
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  float m = 0.0f;
  for (int64_t i = tid; i < n; i += nthreads) m = fmaxf(m, fabsf(__uint_as_float(uint32_t(x[i]) << 16)));
  m = block_max(m);
  if (threadIdx.x == 0) partials[blockIdx.x] = m;
}

template <int MODE, class Div>
__device__ __forceinline__ float cast_loop(const uint16_t* __restrict__ x, uint8_t* __restrict__ q, int64_t n,
                                           const Div& div) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  float m = 0.0f;
  for (int64_t i = tid; i < n; i += nthreads) {
    const uint32_t w = x[i];
    if (MODE == kDelayed) m = fmaxf(m, fabsf(__uint_as_float(w << 16)));
    q[i] = static_cast<uint8_t>(div.word(w) & 0xFFu);
  }
  return m;
}

// Cast pass.  kCurrent: scale = fold(partials_in); CTA 0 stores it to scale_out.
//             kDelayed: scale = *prev_scale; each CTA also writes its |x| max
//                       to partials_out[blockIdx.x].
template <int MODE>
__global__ void __launch_bounds__(kQuantThreads) quantize_cast_kernel(
    const uint16_t* __restrict__ x, uint8_t* __restrict__ q, int64_t n, const float* __restrict__ partials_in,
    int n_partials, DelayedSource prev_scale, float* __restrict__ scale_out, float* __restrict__ partials_out,
    ScaleFold fold) {
  pdl_wait();
  float s;
  if (MODE == kCurrent) {
    s = fold_partials_to_scale(partials_in, n_partials);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  } else {
    s = delayed_scale(prev_scale);
  }
  // s is uniform over the grid, so the branch never diverges.
  const float m = markstein_applies(s) ? cast_loop<MODE>(x, q, n, make_markstein(s))
                                       : cast_loop<MODE>(x, q, n, DivF64(s));
  if (MODE == kDelayed) {
    const float bm = block_max(m);
    if (threadIdx.x == 0) partials_out[blockIdx.x] = bm;
    if (fold.counter != nullptr) fold_scale_if_last<kQuantThreads>(partials_out, fold);
  }
}

// ---------------------------------------------------------------- streaming passes
// The 16-byte aligned bulk of x (all but the last n % 8 elements) moves through
// shared memory in chunks of kStreamChunkBytes: one producer thread keeps
// kStreamStages untiled bulk copies (cp.async.bulk, no multicast) in flight per
// CTA, paced by full/empty mbarriers, and eight consumer warps read each chunk
// from shared memory.  The copy engine keeps the loads in flight, so the
// threads only spend instructions on the bytes themselves.  CTA c takes chunks
// c, c + grid, ...; the last chunk may be short (a multiple of 16 bytes) and
// CTA 0 also handles the n % 8 tail elements with plain loads.
//   kStreamAmax        : |x| max per CTA                         -> partials_out
//   kStreamCastCurrent : scale = fold(partials_in), cast; CTA 0 -> scale_out
//   kStreamCastDelayed : cast with *prev_scale, |x| max per CTA  -> partials_out,
//                        folded into the current scale by the last CTA
enum StreamKind : int { kStreamAmax = 0, kStreamCastCurrent = 1, kStreamCastDelayed = 2 };

#ifndef FP8_STREAM_CHUNK_BYTES
#define FP8_STREAM_CHUNK_BYTES 16384
#endif
#ifndef FP8_STREAM_STAGES
#define FP8_STREAM_STAGES 4
#endif
#ifndef FP8_STREAM_CONSUMER_WARPS
#define FP8_STREAM_CONSUMER_WARPS 8
#endif
constexpr int kStreamChunkBytes = FP8_STREAM_CHUNK_BYTES;
constexpr int kStreamStages = FP8_STREAM_STAGES;
constexpr int kStreamConsumerWarps = FP8_STREAM_CONSUMER_WARPS;
constexpr int kStreamConsumers = kStreamConsumerWarps * 32;
constexpr int kStreamThreads = kStreamConsumers + 32;  // + the producer warp
constexpr int kStreamVecPerThread = kStreamChunkBytes / 16 / kStreamConsumers;
constexpr size_t kStreamSmemBytes = static_cast<size_t>(kStreamStages) * kStreamChunkBytes + 2 * kStreamStages * 8;
static_assert(kStreamChunkBytes % (16 * kStreamConsumers) == 0, "chunk must split evenly over the consumers");

struct StreamShape {
  int64_t main_bytes;  // bytes of x moved by bulk copies (a multiple of 16)
  int64_t nchunks;
};

__device__ __forceinline__ StreamShape stream_shape(int64_t n) {
  StreamShape sh;
  sh.main_bytes = (n & ~int64_t(7)) * 2;
  sh.nchunks = (sh.main_bytes + kStreamChunkBytes - 1) / kStreamChunkBytes;
  return sh;
}

__device__ __forceinline__ void stream_produce(const uint16_t* __restrict__ x, uint8_t* bufs, uint64_t* full,
                                               uint64_t* empty, const StreamShape& sh, volatile int* abort_flag,
                                               int* err) {
  int64_t issued = 0;
  for (int64_t c = blockIdx.x; c < sh.nchunks; c += gridDim.x, ++issued) {
    const int stage = static_cast<int>(issued % kStreamStages);
    if (issued >= kStreamStages &&
        !mbar_wait(&empty[stage], static_cast<uint32_t>((issued / kStreamStages - 1) & 1), abort_flag, err,
                   kErrTimeoutQuant))
      break;
    const int64_t off = c * kStreamChunkBytes;
    const int64_t left = sh.main_bytes - off;
    const uint32_t bytes = static_cast<uint32_t>(left < kStreamChunkBytes ? left : kStreamChunkBytes);
    mbar_arrive_expect_tx(&full[stage], bytes);
    bulk_load_1d(bufs + stage * kStreamChunkBytes, reinterpret_cast<const uint8_t*>(x) + off, bytes, &full[stage]);
  }
  if (*abort_flag) {
    // Consumers gave up: let the copies still in flight land before the CTA exits.
    volatile int never = 0;
    const int64_t first = issued > kStreamStages ? issued - kStreamStages : 0;
    for (int64_t i = first; i < issued; ++i)
      mbar_wait(&full[i % kStreamStages], static_cast<uint32_t>((i / kStreamStages) & 1), &never, err,
                kErrTimeoutDrain);
  }
}

// Consumer side; returns this thread's packed |x| maxima (amax kinds).
template <int KIND, class Div>
__device__ __forceinline__ uint32_t stream_consume(const uint8_t* bufs, uint64_t* full, uint64_t* empty,
                                                   uint8_t* __restrict__ q, const StreamShape& sh, const Div& div,
                                                   volatile int* abort_flag, int* err) {
  uint32_t m2 = 0u;
  const int t = threadIdx.x;
  int64_t i = 0;
  for (int64_t c = blockIdx.x; c < sh.nchunks; c += gridDim.x, ++i) {
    const int stage = static_cast<int>(i % kStreamStages);
    // Every lane waits (each needs the copy's bytes visible); the vote keeps the
    // warp together if the wait gives up.
    const bool ok = mbar_wait(&full[stage], static_cast<uint32_t>((i / kStreamStages) & 1), abort_flag, err,
                              kErrTimeoutQuant);
    if (!__all_sync(0xffffffffu, ok)) break;
    const int64_t off = c * kStreamChunkBytes;
    const int64_t left = sh.main_bytes - off;
    const int nv = static_cast<int>((left < kStreamChunkBytes ? left : kStreamChunkBytes) >> 4);
    const uint8_t* buf = bufs + stage * kStreamChunkBytes;
    uint4 a[kStreamVecPerThread];
#pragma unroll
    for (int j = 0; j < kStreamVecPerThread; ++j) {
      const int v = t + j * kStreamConsumers;
      a[j] = v < nv ? ld_shared_v4(buf + v * 16) : make_uint4(0u, 0u, 0u, 0u);
    }
    // The chunk is in registers: hand the stage back to the producer.
    __syncwarp();
    if ((t & 31) == 0) mbar_arrive(&empty[stage]);
    if (KIND != kStreamAmax) {
      uint2* qv = reinterpret_cast<uint2*>(q + (off >> 1));
#pragma unroll
      for (int j = 0; j < kStreamVecPerThread; ++j) {
        const int v = t + j * kStreamConsumers;
        if (v < nv) qv[v] = cast_vec(a[j], div);
      }
    }
    if (KIND != kStreamCastCurrent) {
#pragma unroll
      for (int j = 0; j < kStreamVecPerThread; ++j) m2 = bf16x2_max(m2, absmax_vec2(a[j]));
    }
  }
  return m2;
}

// Consumer side plus the tail; returns this thread's |x| max (amax kinds).  CTA 0's
// consumers also handle the n % 8 tail elements with plain loads.
template <int KIND, class Div>
__device__ __forceinline__ float stream_consume_all(const uint16_t* __restrict__ x, uint8_t* __restrict__ q,
                                                    int64_t n, const uint8_t* bufs, uint64_t* full, uint64_t* empty,
                                                    const StreamShape& sh, const Div& div, volatile int* abort_flag,
                                                    int* err) {
  float m = unpack_max2(stream_consume<KIND>(bufs, full, empty, q, sh, div, abort_flag, err));
  if (blockIdx.x == 0) {
    for (int64_t i = (sh.main_bytes >> 1) + threadIdx.x; i < n; i += kStreamConsumers) {
      const uint32_t w = x[i];
      if (KIND != kStreamCastCurrent) m = fmaxf(m, fabsf(__uint_as_float(w << 16)));
      if (KIND != kStreamAmax) q[i] = static_cast<uint8_t>(div.word(w) & 0xFFu);
    }
  }
  return m;
}

// Named barrier of the consumer warps (the producer warp streams meanwhile).
constexpr int kStreamConsumerBar = 1;

// x 16-byte aligned, q 8-byte aligned.  Dynamic shared memory: kStreamSmemBytes.
// The producer starts its copies as soon as the barriers exist; the consumers fold the
// scale (current: the amax partials; delayed: the previous scale or the history max)
// while the first chunks are in flight.
template <int KIND>
__global__ void __launch_bounds__(kStreamThreads) quant_stream_kernel(
    const uint16_t* __restrict__ x, uint8_t* __restrict__ q, int64_t n, const float* __restrict__ partials_in,
    int n_partials, DelayedSource prev_scale, float* __restrict__ scale_out, float* __restrict__ partials_out,
    int* err, ScaleFold fold) {
  extern __shared__ __align__(128) uint8_t stream_smem[];
  pdl_wait();
  uint8_t* bufs = stream_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stream_smem + kStreamStages * kStreamChunkBytes);
  uint64_t* empty = full + kStreamStages;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStreamStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStreamConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const StreamShape sh = stream_shape(n);
  float m = 0.0f;
  if (threadIdx.x >= kStreamConsumers) {
    if (threadIdx.x == kStreamConsumers) stream_produce(x, bufs, full, empty, sh, &abort_flag, err);
  } else {
    float s = 1.0f;
    if (KIND == kStreamCastCurrent) {
      s = fold_partials_to_scale<kStreamConsumers, kStreamConsumerBar>(partials_in, n_partials);
      if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
    } else if (KIND == kStreamCastDelayed) {
      s = delayed_scale<kStreamConsumers, kStreamConsumerBar>(prev_scale);
    }
    if (KIND == kStreamAmax || !markstein_applies(s))  // s is uniform over the grid: no divergence
      m = stream_consume_all<KIND>(x, q, n, bufs, full, empty, sh, DivF64(s), &abort_flag, err);
    else
      m = stream_consume_all<KIND>(x, q, n, bufs, full, empty, sh, make_markstein(s), &abort_flag, err);
  }
  if (KIND != kStreamCastCurrent) {
    const float bm = block_max<kStreamThreads>(m);
    if (threadIdx.x == 0) partials_out[blockIdx.x] = bm;
    if (KIND == kStreamCastDelayed && fold.counter != nullptr) fold_scale_if_last<kStreamThreads>(partials_out, fold);
  }
}

// ---------------------------------------------------------------- several tensors per launch
// Current scaling of up to kMaxMultiTensors tensors in one amax launch and one
// cast launch (a layer's input and weight are quantized together): the chunks of
// all tensors form one index space (chunk_begin holds the prefix sums), every CTA
// keeps one |x| maximum per tensor, and every tensor gets its own scale.  Each
// tensor's bytes are those fp8_quantize_current would produce.
constexpr int kMaxMultiTensors = 4;

struct MultiQuant {
  const uint16_t* x[kMaxMultiTensors];
  uint8_t* q[kMaxMultiTensors];
  float* scale_out[kMaxMultiTensors];
  int64_t n[kMaxMultiTensors];
  int64_t main_bytes[kMaxMultiTensors];
  int64_t chunk_begin[kMaxMultiTensors + 1];
  int count;
};

__device__ __forceinline__ int multi_tensor_of(const MultiQuant& m, int64_t k) {
  int t = 0;
#pragma unroll
  for (int i = 1; i < kMaxMultiTensors; ++i)
    if (i < m.count && k >= m.chunk_begin[i]) t = i;
  return t;
}

// Producer side for the multi-tensor passes (same pacing as stream_produce).
__device__ __forceinline__ void multi_produce(const MultiQuant& m, uint8_t* bufs, uint64_t* full, uint64_t* empty,
                                              volatile int* abort_flag, int* err) {
  int64_t issued = 0;
  for (int64_t k = blockIdx.x; k < m.chunk_begin[m.count]; k += gridDim.x, ++issued) {
    const int stage = static_cast<int>(issued % kStreamStages);
    if (issued >= kStreamStages &&
        !mbar_wait(&empty[stage], static_cast<uint32_t>((issued / kStreamStages - 1) & 1), abort_flag, err,
                   kErrTimeoutQuant))
      break;
    const int t = multi_tensor_of(m, k);
    const int64_t off = (k - m.chunk_begin[t]) * kStreamChunkBytes;
    const int64_t left = m.main_bytes[t] - off;
    const uint32_t bytes = static_cast<uint32_t>(left < kStreamChunkBytes ? left : kStreamChunkBytes);
    mbar_arrive_expect_tx(&full[stage], bytes);
    bulk_load_1d(bufs + stage * kStreamChunkBytes, reinterpret_cast<const uint8_t*>(m.x[t]) + off, bytes,
                 &full[stage]);
  }
  if (*abort_flag) {
    volatile int never = 0;
    const int64_t first = issued > kStreamStages ? issued - kStreamStages : 0;
    for (int64_t i = first; i < issued; ++i)
      mbar_wait(&full[i % kStreamStages], static_cast<uint32_t>((i / kStreamStages) & 1), &never, err,
                kErrTimeoutDrain);
  }
}

__device__ __forceinline__ void multi_init(uint64_t* full, uint64_t* empty, int* abort_flag) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStreamStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStreamConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
}

// partials[t * gridDim.x + cta] = max |x_t| over the chunks of tensor t this CTA streamed.
__global__ void __launch_bounds__(kStreamThreads) quant_multi_amax_kernel(MultiQuant m, float* __restrict__ partials,
                                                                          int* err) {
  extern __shared__ __align__(128) uint8_t stream_smem[];
  pdl_wait();
  uint8_t* bufs = stream_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stream_smem + kStreamStages * kStreamChunkBytes);
  uint64_t* empty = full + kStreamStages;
  __shared__ int abort_flag;
  multi_init(full, empty, &abort_flag);
  uint32_t m2[kMaxMultiTensors] = {0u, 0u, 0u, 0u};
  if (threadIdx.x == kStreamConsumers) {
    multi_produce(m, bufs, full, empty, &abort_flag, err);
  } else if (threadIdx.x < kStreamConsumers) {
    const int t0 = threadIdx.x;
    int64_t i = 0;
    for (int64_t k = blockIdx.x; k < m.chunk_begin[m.count]; k += gridDim.x, ++i) {
      const int stage = static_cast<int>(i % kStreamStages);
      const bool ok = mbar_wait(&full[stage], static_cast<uint32_t>((i / kStreamStages) & 1), &abort_flag, err,
                                kErrTimeoutQuant);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int t = multi_tensor_of(m, k);
      const int64_t off = (k - m.chunk_begin[t]) * kStreamChunkBytes;
      const int64_t left = m.main_bytes[t] - off;
      const int nv = static_cast<int>((left < kStreamChunkBytes ? left : kStreamChunkBytes) >> 4);
      const uint8_t* buf = bufs + stage * kStreamChunkBytes;
      uint32_t mv = 0u;
#pragma unroll
      for (int j = 0; j < kStreamVecPerThread; ++j) {
        const int v = t0 + j * kStreamConsumers;
        if (v < nv) mv = bf16x2_max(mv, absmax_vec2(ld_shared_v4(buf + v * 16)));
      }
      __syncwarp();
      if ((t0 & 31) == 0) mbar_arrive(&empty[stage]);
#pragma unroll
      for (int u = 0; u < kMaxMultiTensors; ++u)
        if (u == t) m2[u] = bf16x2_max(m2[u], mv);
    }
  }
  for (int u = 0; u < m.count; ++u) {
    float mu = unpack_max2(m2[u]);
    if (blockIdx.x == 0)
      for (int64_t e = (m.main_bytes[u] >> 1) + threadIdx.x; e < m.n[u]; e += kStreamThreads)
        mu = fmaxf(mu, fabsf(__uint_as_float(uint32_t(m.x[u][e]) << 16)));
    mu = block_max<kStreamThreads>(mu);
    if (threadIdx.x == 0) partials[u * gridDim.x + blockIdx.x] = mu;
  }
}

// Cast pass: scale_t = fold(partials[t * n_partials .. +n_partials]); CTA 0 publishes them.
__global__ void __launch_bounds__(kStreamThreads) quant_multi_cast_kernel(MultiQuant m,
                                                                          const float* __restrict__ partials,
                                                                          int n_partials, int* err) {
  extern __shared__ __align__(128) uint8_t stream_smem[];
  pdl_wait();
  uint8_t* bufs = stream_smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(stream_smem + kStreamStages * kStreamChunkBytes);
  uint64_t* empty = full + kStreamStages;
  __shared__ int abort_flag;
  float sc[kMaxMultiTensors] = {1.0f, 1.0f, 1.0f, 1.0f};
  multi_init(full, empty, &abort_flag);
  if (threadIdx.x == kStreamConsumers) {
    multi_produce(m, bufs, full, empty, &abort_flag, err);  // starts while the consumers fold the scales
  } else if (threadIdx.x < kStreamConsumers) {
    for (int u = 0; u < m.count; ++u) {
      const float su = fold_partials_to_scale<kStreamConsumers, kStreamConsumerBar>(partials + u * n_partials,
                                                                                     n_partials);
#pragma unroll
      for (int w = 0; w < kMaxMultiTensors; ++w)
        if (w == u) sc[w] = su;
      if (blockIdx.x == 0 && threadIdx.x == 0) *m.scale_out[u] = su;
    }
    const int t0 = threadIdx.x;
    int64_t i = 0;
    for (int64_t k = blockIdx.x; k < m.chunk_begin[m.count]; k += gridDim.x, ++i) {
      const int stage = static_cast<int>(i % kStreamStages);
      const bool ok = mbar_wait(&full[stage], static_cast<uint32_t>((i / kStreamStages) & 1), &abort_flag, err,
                                kErrTimeoutQuant);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int t = multi_tensor_of(m, k);
      const int64_t off = (k - m.chunk_begin[t]) * kStreamChunkBytes;
      const int64_t left = m.main_bytes[t] - off;
      const int nv = static_cast<int>((left < kStreamChunkBytes ? left : kStreamChunkBytes) >> 4);
      const uint8_t* buf = bufs + stage * kStreamChunkBytes;
      uint4 a[kStreamVecPerThread];
#pragma unroll
      for (int j = 0; j < kStreamVecPerThread; ++j) {
        const int v = t0 + j * kStreamConsumers;
        a[j] = v < nv ? ld_shared_v4(buf + v * 16) : make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
      if ((t0 & 31) == 0) mbar_arrive(&empty[stage]);
      float s = sc[0];
#pragma unroll
      for (int w = 1; w < kMaxMultiTensors; ++w)
        if (w == t) s = sc[w];
      uint2* qv = reinterpret_cast<uint2*>(m.q[t] + (off >> 1));
      if (markstein_applies(s)) {  // uniform over the chunk: no divergence
        const CastMarkstein d = make_markstein(s);
#pragma unroll
        for (int j = 0; j < kStreamVecPerThread; ++j) {
          const int v = t0 + j * kStreamConsumers;
          if (v < nv) qv[v] = cast_vec(a[j], d);
        }
      } else {
        const DivF64 d(s);
#pragma unroll
        for (int j = 0; j < kStreamVecPerThread; ++j) {
          const int v = t0 + j * kStreamConsumers;
          if (v < nv) qv[v] = cast_vec(a[j], d);
        }
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < kStreamConsumers) {  // the tails, with the consumers' folded scales
    for (int u = 0; u < m.count; ++u) {
      float s = sc[0];
#pragma unroll
      for (int w = 1; w < kMaxMultiTensors; ++w)
        if (w == u) s = sc[w];
      for (int64_t e = (m.main_bytes[u] >> 1) + threadIdx.x; e < m.n[u]; e += kStreamConsumers) {
        const uint32_t wv = m.x[u][e];
        m.q[u][e] = static_cast<uint8_t>((markstein_applies(s) ? make_markstein(s).word(wv) : DivF64(s).word(wv)) &
                                         0xFFu);
      }
    }
  }
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
  pdl_wait();
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
  pdl_wait();
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

// The data-grad re-layout of many conv weights in one launch: tensor t is
// [Cout][9][Cin] e4m3 -> [Cin][9][Cout] (per tap a Cout x Cin transpose), the
// layout fp8_conv3x3_dgrad reads; Cout and Cin multiples of 64, 16-byte aligned.
// CTA k takes one 64x64 tile of one tap of one tensor (prefix sums in tile_begin).
constexpr int kMaxTransTensors = 64;

struct TransBatch {
  const uint8_t* src[kMaxTransTensors];
  uint8_t* dst[kMaxTransTensors];
  int cout[kMaxTransTensors];
  int cin[kMaxTransTensors];
  int tile_begin[kMaxTransTensors + 1];
  int count;
};
static_assert(sizeof(TransBatch) < 4000, "kernel parameter size");

__global__ void __launch_bounds__(256) transpose_conv_weights_kernel(TransBatch b) {
  __shared__ __align__(16) uint8_t tile[kTransTile][kTransTile + 4];
  pdl_wait();
  const int k = blockIdx.x;
  int lo = 0, hi = b.count - 1;  // last t with tile_begin[t] <= k
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.tile_begin[mid] <= k) lo = mid; else hi = mid - 1;
  }
  const int t = lo, cout = b.cout[t], cin = b.cin[t];
  const int local = k - b.tile_begin[t];
  const int tr = cout / kTransTile, tc = cin / kTransTile;
  const int tap = local / (tr * tc), rem = local % (tr * tc);
  const int64_t r0 = static_cast<int64_t>(rem / tc) * kTransTile, c0 = static_cast<int64_t>(rem % tc) * kTransTile;
  const int64_t src_ld = 9ll * cin, dst_ld = 9ll * cout;
  const uint8_t* s = b.src[t] + static_cast<int64_t>(tap) * cin;
  uint8_t* d = b.dst[t] + static_cast<int64_t>(tap) * cout;
  const int row = threadIdx.x >> 2, seg = (threadIdx.x & 3) * 16;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(s + (r0 + row) * src_ld + c0 + seg));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 16; ++i) tile[row][seg + i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
  __syncthreads();
  uint32_t o[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i >> 2] |= static_cast<uint32_t>(tile[seg + i][row]) << (8 * (i & 3));
  *reinterpret_cast<uint4*>(d + (c0 + row) * dst_ld + r0 + seg) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------- batched weight quantize
// The delayed quantize of many fp32 weight tensors at once (every FP8 conv of a
// model, once per step): each weight is rounded to bf16 -- the reference's
// weight.to(bfloat16), fp8_kernels.py:836 -- then cast exactly as the delayed
// quantize casts a bf16 tensor, with its module's scale history max as the scale;
// its own scale goes into that history at the module's position, which is not
// advanced (the module's activation quantize writes at the same position and
// advances it, so the histories end up as the reference's per-call bookkeeping
// leaves them).  Three launches for all tensors: history maxima, cast (one
// |w| partial per chunk), finalize.
constexpr int kMaxBatchWeights = 64;
constexpr int kWeightChunk = 4096;  // elements per chunk (16 KB of fp32)

struct WeightBatch {
  const float* w[kMaxBatchWeights];
  uint8_t* q[kMaxBatchWeights];
  float* window[kMaxBatchWeights];
  const int64_t* pos[kMaxBatchWeights];
  float* used[kMaxBatchWeights];  // the scale each tensor is cast with (its history max)
  int64_t n[kMaxBatchWeights];
  int chunk_begin[kMaxBatchWeights + 1];
  int count;
  int window_len;
  int empty_zero;  // as WindowUpdate::empty_zero
};
static_assert(sizeof(WeightBatch) < 4096, "kernel parameter size");

__device__ __forceinline__ int weight_of_chunk(const WeightBatch& b, int k) {
  int lo = 0, hi = b.count - 1;  // last t with chunk_begin[t] <= k
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.chunk_begin[mid] <= k) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One CTA per tensor: used[t] = max(window[t][0 .. len)).
__global__ void __launch_bounds__(kQuantThreads) weight_window_max_kernel(WeightBatch b) {
  pdl_wait();
  const int t = blockIdx.x;
  const DelayedSource d{nullptr, b.window[t], b.window_len, nullptr};
  const float m = delayed_scale<kQuantThreads>(d);
  if (threadIdx.x == 0) *b.used[t] = m;
}

// One CTA per chunk of kWeightChunk elements; partials[k] = max |bf16(w)| of chunk k.
__global__ void __launch_bounds__(kQuantThreads) weight_cast_kernel(WeightBatch b, float* __restrict__ partials) {
  pdl_wait();
  const int k = blockIdx.x;
  const int t = weight_of_chunk(b, k);
  const int64_t begin = static_cast<int64_t>(k - b.chunk_begin[t]) * kWeightChunk;
  const int64_t end = min(begin + kWeightChunk, b.n[t]);
  const float s = *b.used[t];
  const float* __restrict__ w = b.w[t];
  uint8_t* __restrict__ q = b.q[t];
  float m = 0.0f;
  // 8 elements per step where w is 16-byte and q 8-byte aligned (uniform per tensor), then pairs:
  // round to bf16 (RN), |.| max, cast
  const bool vec = ((reinterpret_cast<uintptr_t>(w) & 15u) | (reinterpret_cast<uintptr_t>(q) & 7u)) == 0;
  const int64_t end8 = vec ? begin + ((end - begin) & ~int64_t(7)) : begin;
  auto body = [&](const auto& div) {
    uint32_t m2 = 0u;
    for (int64_t i = begin + 8 * threadIdx.x; i < end8; i += 8 * kQuantThreads) {
      const float4 a = *reinterpret_cast<const float4*>(w + i);
      const float4 c = *reinterpret_cast<const float4*>(w + i + 4);
      const uint4 h = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(c.x, c.y),
                                 pack_bf16x2(c.z, c.w));
      m2 = bf16x2_max(m2, absmax_vec2(h));
      *reinterpret_cast<uint2*>(q + i) = cast_vec(h, div);
    }
    m = unpack_max2(m2);
    for (int64_t i = end8 + 2 * threadIdx.x; i < end; i += 2 * kQuantThreads) {
      const float f0 = w[i];
      const float f1 = i + 1 < end ? w[i + 1] : 0.0f;
      const uint32_t word = pack_bf16x2(f0, f1);
      m = fmaxf(m, unpack_max2(word & kAbsMask2));
      const uint32_t bytes = div.word(word);
      if (i + 1 < end)  // i is even and q 2-byte aligned: one 16-bit store
        *reinterpret_cast<uint16_t*>(q + i) = static_cast<uint16_t>(bytes & 0xFFFFu);
      else
        q[i] = static_cast<uint8_t>(bytes & 0xFFu);
    }
  };
  if (markstein_applies(s))  // uniform over the CTA
    body(make_markstein(s));
  else
    body(DivF64(s));
  m = block_max(m);
  if (threadIdx.x == 0) partials[k] = m;
}

// One CTA per tensor: its scale from its chunks' partials, stored at window[pos].
__global__ void __launch_bounds__(kQuantThreads) weight_finalize_kernel(WeightBatch b,
                                                                         const float* __restrict__ partials) {
  pdl_wait();
  const int t = blockIdx.x;
  const float* part = partials + b.chunk_begin[t];
  const int count = b.chunk_begin[t + 1] - b.chunk_begin[t];
  float m = 0.0f;
  for (int i = threadIdx.x; i < count; i += kQuantThreads) m = fmaxf(m, part[i]);
  m = block_max<kQuantThreads>(m);
  if (threadIdx.x == 0) b.window[t][*b.pos[t]] = history_entry(m, b.empty_zero);
}


// ---------------------------------------------------------------- shared-memory-resident current scaling
// Current scaling of up to kMaxMultiTensors tensors in ONE launch when every
// CTA's share of them fits in its shared memory (config 2's 33.5 MB activation
// is 227 KB per SM on 148 SMs): one CTA per SM (cooperative launch, so all are
// resident), each CTA bulk-loads its contiguous slice of every tensor into
// shared memory in 16 KB pieces (all in flight at once), takes the slice's |x|
// max per tensor as the pieces land, meets the other CTAs at a grid barrier that
// hands every CTA the tensors' maxima, and casts its slice from shared memory.
// x is read from HBM once and q written once, instead of a read, a second read
// and a write by two launches.  Bytes and scales are those of the two-pass kernels.
constexpr int kResThreads = 512;
constexpr int kResPiece = 16384;       // bytes per bulk copy / mbarrier
constexpr int kResMaxPieces = 16;      // 256 KB > any CTA's shared memory
// Dynamic bytes a CTA may use: the 227 KB per-CTA limit less 1 KB for the kernel's static
// arrays (barriers, reduction scratch; about 300 bytes).  Config 2's conv input and weight
// together need 228,720 bytes per CTA on 148 SMs (226,720 + 2,000).
constexpr int kResSmemCap = 232448 - 1024;

// Slices: tensor t has vecs = vq * G + vr vectors of 8 elements (the host splits
// it); CTA c of G owns [floor(vecs c / G), floor(vecs (c + 1) / G)), computed as
// vq c + (vr c) / G with a 32-bit division (vr c < G^2): the 64-bit divisions
// this replaces took 0.45 us of the kernel's start.
struct ResSlices {
  int64_t vq[kMaxMultiTensors];
  int vr[kMaxMultiTensors];
};
__device__ __forceinline__ int64_t res_slice_begin(int64_t vq, int vr, int c, int G) {
  return vq * c + static_cast<int64_t>(static_cast<unsigned>(vr * c) / static_cast<unsigned>(G));
}

// Words of the grid barrier, all zero when the launch starts and zeroed again by
// the last CTA to take a departure ticket (every CTA takes it after its reads).
// The CTAs' |x| maxima meet in one atomic-max word per tensor (non-negative
// floats order like their bit patterns), and a CTA that saw a NaN sets the
// tensor's NaN word.  A CTA publishes its maxima, then arrives with a release
// add; thread 0 of every CTA polls `arrive` with acquire loads and then reads
// the words.  The departure ticket's value is only needed at the kernel's end.
struct ResSync {
  unsigned int* arrive;
  unsigned int* depart;
  unsigned int* amax[kMaxMultiTensors];
  unsigned int* nan[kMaxMultiTensors];
};

// NaN-propagating packed max (max.NaN): the |x| max that shows whether a share holds a NaN.
__device__ __forceinline__ uint32_t bf16x2_max_nan(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t absmax_vec2_nan(const uint4& a) {
  return bf16x2_max_nan(bf16x2_max_nan(a.x & kAbsMask2, a.y & kAbsMask2),
                        bf16x2_max_nan(a.z & kAbsMask2, a.w & kAbsMask2));
}
__device__ __forceinline__ bool bf16x2_has_nan(uint32_t w) {
  return (w & 0x7FFFu) > 0x7F80u || ((w >> 16) & 0x7FFFu) > 0x7F80u;
}

// CastMarkstein without the clamp, for current scaling of a tensor that holds no
// NaN: s = RN(amax / 448) and |x| <= amax bound |x / s| by 448 (1 + 2^-23), inside
// the range where Markstein's step is exact, and cvt.satfinite saturates the rest.
// The sign of each byte is x's sign bit or'd in (one byte permute and one logic
// op per four elements), which also makes -0 the byte 0x80 as the reference's
// division does.  tests/quantize_division_check.c (part 4) compares the bytes
// with the reference for every bf16 x with |x| <= amax over every bf16 amax in
// the scale window.  Measured: the cast phase of config 2's input 5.5 -> 3.0 us.
struct CastMarksteinNoClamp {
  float2 r2, ns2;
  __device__ __forceinline__ explicit CastMarksteinNoClamp(const CastMarkstein& m) : r2(m.r2), ns2(m.ns2) {}
  // Four bf16 (w0 low, w0 high, w1 low, w1 high) -> four e4m3 bytes in that order.
  __device__ __forceinline__ uint32_t quad(uint32_t w0, uint32_t w1) const {
    const float2 xa = make_float2(__uint_as_float(w0 << 16), __uint_as_float(w0 & 0xFFFF0000u));
    const float2 xb = make_float2(__uint_as_float(w1 << 16), __uint_as_float(w1 & 0xFFFF0000u));
    float2 qa = f32x2_mul(xa, r2), qb = f32x2_mul(xb, r2);
    const float2 ea = f32x2_fma(qa, ns2, xa), eb = f32x2_fma(qb, ns2, xb);
    qa = f32x2_fma(ea, r2, qa);
    qb = f32x2_fma(eb, r2, qb);
    const uint32_t lo = cvt_e4m3x2(qa.x, qa.y), hi = cvt_e4m3x2(qb.x, qb.y);
    return __byte_perm(lo, hi, 0x5410) | (__byte_perm(w0, w1, 0x7531) & 0x80808080u);
  }
};
__device__ __forceinline__ uint2 cast_vec(const uint4& a, const CastMarksteinNoClamp& d) {
  return make_uint2(d.quad(a.x, a.y), d.quad(a.z, a.w));
}

__global__ void __launch_bounds__(kResThreads, 1) quant_resident_kernel(MultiQuant m, ResSlices sl, ResSync sy,
                                                                         int* err) {
  extern __shared__ __align__(128) uint8_t res_smem[];
  __shared__ __align__(8) uint64_t bars[kResMaxPieces];
  __shared__ int abort_flag, passed;
  __shared__ unsigned int cta_max[kMaxMultiTensors], cta_nan[kMaxMultiTensors];
  __shared__ unsigned int all_max[kMaxMultiTensors], all_nan[kMaxMultiTensors];
  pdl_wait();
  const int G = gridDim.x, c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t vbeg[kMaxMultiTensors], vcnt[kMaxMultiTensors], soff[kMaxMultiTensors];
  int64_t total = 0;
#pragma unroll
  for (int t = 0; t < kMaxMultiTensors; ++t) {  // vq = vr = 0 beyond m.count
    vbeg[t] = res_slice_begin(sl.vq[t], sl.vr[t], c, G);
    vcnt[t] = res_slice_begin(sl.vq[t], sl.vr[t], c + 1, G) - vbeg[t];
    soff[t] = total;
    total += vcnt[t] * 16;
  }
  const int npieces = static_cast<int>((total + kResPiece - 1) / kResPiece);
  if (threadIdx.x < kMaxMultiTensors) {
    cta_max[threadIdx.x] = 0u;
    cta_nan[threadIdx.x] = 0u;
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < npieces; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // piece i covers smem bytes [i * kResPiece, ...), possibly spanning tensors: one copy per (piece, tensor)
    for (int i = 0; i < npieces; ++i) {
      const int64_t p0 = static_cast<int64_t>(i) * kResPiece, p1 = min(total, p0 + kResPiece);
      mbar_arrive_expect_tx(&bars[i], static_cast<uint32_t>(p1 - p0));
#pragma unroll
      for (int t = 0; t < kMaxMultiTensors; ++t) {
        const int64_t a = max(p0, soff[t]), b = min(p1, soff[t] + vcnt[t] * 16);
        if (t < m.count && a < b)
          bulk_load_1d(res_smem + a, reinterpret_cast<const uint8_t*>(m.x[t] + vbeg[t] * 8) + (a - soff[t]),
                       static_cast<uint32_t>(b - a), &bars[i]);
      }
    }
  }
  // |x| max per tensor (NaN-propagating) as the copies land: warp w takes pieces w,
  // w + 16, ..., so each warp waits on its own pieces' barriers only; within a piece,
  // the part of each tensor it holds (offsets are multiples of 16 bytes).
  uint32_t m2[kMaxMultiTensors] = {0u, 0u, 0u, 0u};
  bool ok = true;
  for (int i = warp; i < npieces; i += kResThreads / 32) {
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[i], 0, &abort_flag, err, kErrTimeoutQuant));
    if (!ok) break;
    const int64_t p0 = static_cast<int64_t>(i) * kResPiece, p1 = min(total, p0 + kResPiece);
#pragma unroll
    for (int u = 0; u < kMaxMultiTensors; ++u) {
      const int64_t lo = max(p0, soff[u]), hi = min(p1, soff[u] + vcnt[u] * 16);  // empty for u >= count
      uint32_t mu = 0u;
#pragma unroll 4
      for (int64_t o = lo + lane * 16; o < hi; o += 32 * 16)
        mu = bf16x2_max_nan(mu, absmax_vec2_nan(ld_shared_v4(res_smem + o)));
      m2[u] = bf16x2_max_nan(m2[u], mu);
    }
  }
  if (!__syncthreads_and(ok)) {
    // let the copies still in flight land before the CTA exits (the other CTAs give up at the barrier)
    volatile int never = 0;
    if (threadIdx.x == 0)
      for (int i = 0; i < npieces; ++i) mbar_wait(&bars[i], 0, &never, err, kErrTimeoutDrain);
    __syncthreads();
    return;
  }
  // The CTA's max per tensor.  A thread whose share held a NaN takes its share's max
  // again without NaN (bf16 max skips it, as the reference's amax does) and flags it.
#pragma unroll
  for (int t = 0; t < kMaxMultiTensors; ++t) {
    if (t < m.count) {
      uint32_t mt = m2[t];
      const bool nan = bf16x2_has_nan(mt);
      if (nan) {
        mt = 0u;
        for (int i = warp; i < npieces; i += kResThreads / 32) {
          const int64_t p0 = static_cast<int64_t>(i) * kResPiece, p1 = min(total, p0 + kResPiece);
          const int64_t lo = max(p0, soff[t]), hi = min(p1, soff[t] + vcnt[t] * 16);
          for (int64_t o = lo + lane * 16; o < hi; o += 32 * 16)
            mt = bf16x2_max(mt, absmax_vec2(ld_shared_v4(res_smem + o)));
        }
      }
      const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(unpack_max2(mt)));
      const unsigned wn = __reduce_or_sync(0xffffffffu, nan ? 1u : 0u);
      if (lane == 0) {
        atomicMax(&cta_max[t], wm);
        if (wn) cta_nan[t] = 1u;
      }
    }
  }
  __syncthreads();
  unsigned int ticket = 0u;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int t = 0; t < kMaxMultiTensors; ++t) {
      if (t < m.count) {
        atomicMax(sy.amax[t], cta_max[t]);
        if (cta_nan[t]) atomicOr(sy.nan[t], 1u);
      }
    }
    red_release_gpu_add_u32(sy.arrive, 1u);  // orders the maxima above before the arrival
    int okb = 1;
    if (ld_acquire_gpu_u32(sy.arrive) < static_cast<unsigned>(G)) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu_u32(sy.arrive) < static_cast<unsigned>(G)) {
        if (globaltimer_ns() - t0 > FP8_WAIT_TIMEOUT_NS) {
          record_error(err, kErrTimeoutGrid);
          okb = 0;
          break;
        }
      }
    }
    if (okb) {
#pragma unroll
      for (int t = 0; t < kMaxMultiTensors; ++t) {
        if (t < m.count) {
          all_max[t] = ld_relaxed_gpu_u32(sy.amax[t]);
          all_nan[t] = ld_relaxed_gpu_u32(sy.nan[t]);
        }
      }
      ticket = atom_add_acq_rel_gpu_u32(sy.depart, 1u);
    }
    passed = okb;
  }
  __syncthreads();
  if (!passed) return;
#pragma unroll
  for (int t = 0; t < kMaxMultiTensors; ++t) {
    if (t >= m.count) continue;
    const float s = scale_from_amax(__uint_as_float(all_max[t]));
    if (c == 0 && threadIdx.x == 0) *m.scale_out[t] = s;
    uint2* qv = reinterpret_cast<uint2*>(m.q[t] + vbeg[t] * 8);
    const uint8_t* src = res_smem + soff[t];
    auto cast_all = [&](const auto& div) {
      const int64_t nv = vcnt[t];
      int64_t v = threadIdx.x;
      for (; v + 3 * kResThreads < nv; v += 4 * kResThreads) {  // four independent vectors in flight
        uint4 a[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) a[j] = ld_shared_v4(src + (v + j * kResThreads) * 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) qv[v + j * kResThreads] = cast_vec(a[j], div);
      }
      for (; v < nv; v += kResThreads) qv[v] = cast_vec(ld_shared_v4(src + v * 16), div);
    };
    if (!markstein_applies(s))  // s and all_nan are uniform over the grid
      cast_all(DivF64(s));
    else if (all_nan[t])
      cast_all(make_markstein(s));
    else
      cast_all(CastMarksteinNoClamp(make_markstein(s)));
  }
  // The last CTA to take a ticket zeroes the words (every CTA read them before its ticket).
  if (threadIdx.x == 0 && ticket == static_cast<unsigned>(G) - 1u) {
    *sy.arrive = 0u;
#pragma unroll
    for (int t = 0; t < kMaxMultiTensors; ++t) {
      if (t < m.count) {
        *sy.amax[t] = 0u;
        *sy.nan[t] = 0u;
      }
    }
    *sy.depart = 0u;
  }
}

}  // namespace fp8b

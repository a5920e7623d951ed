// cast_batch.cuh — fp32 <-> bf16 casts of many tensors in one launch.
//
// Under bf16 autocast every fp32 weight a bf16 layer reads is cast to bf16 by
// its own launch (the reference's attention projections, 1x1 skip convs and
// time-embedding linears, unet.py:101, 139, 171-172, 331-336), and the bf16
// weight gradient is cast back to fp32 by another launch per weight.  These
// passes move a few MB each and are launch-bound; here one launch casts a whole
// list.  Element values are those of the torch casts: fp32 -> bf16 rounds to
// nearest even, bf16 -> fp32 is exact.  Tensors are dense memory ranges of n
// elements; the chunks of all tensors form one index space (chunk_begin holds
// the prefix sums), a CTA per chunk.
#pragma once

#include "sm100_common.cuh"

namespace fp8b {

constexpr int kCastTensors = 64;
constexpr int kCastChunk = 8192;  // elements per CTA
constexpr int kCastThreads = 256;

struct CastBatch {
  const void* src[kCastTensors];
  void* dst[kCastTensors];
  int64_t n[kCastTensors];
  int chunk_begin[kCastTensors + 1];
  int count;
};
static_assert(sizeof(CastBatch) < 4000, "kernel parameter size");

__device__ __forceinline__ int cast_tensor_of(const CastBatch& b, int k) {
  int lo = 0, hi = b.count - 1;  // last t with chunk_begin[t] <= k
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.chunk_begin[mid] <= k) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// TO_BF16: src fp32, dst bf16.  Otherwise src bf16, dst fp32.
template <bool TO_BF16>
__global__ void __launch_bounds__(kCastThreads) cast_batch_kernel(CastBatch b) {
  pdl_wait();
  const int k = blockIdx.x;
  const int t = cast_tensor_of(b, k);
  const int64_t begin = static_cast<int64_t>(k - b.chunk_begin[t]) * kCastChunk;
  const int64_t end = min(begin + kCastChunk, b.n[t]);
  int64_t tail = begin;
  if constexpr (TO_BF16) {
    const float* __restrict__ s = static_cast<const float*>(b.src[t]);
    uint16_t* __restrict__ d = static_cast<uint16_t*>(b.dst[t]);
    if (((reinterpret_cast<uintptr_t>(s) & 15u) | (reinterpret_cast<uintptr_t>(d) & 7u)) == 0) {
      const int64_t end4 = begin + ((end - begin) & ~int64_t(3));
      for (int64_t i = begin + 4 * threadIdx.x; i < end4; i += 4 * kCastThreads) {
        const float4 v = *reinterpret_cast<const float4*>(s + i);
        *reinterpret_cast<uint2*>(d + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      }
      tail = end4;
    }
    for (int64_t i = tail + threadIdx.x; i < end; i += kCastThreads)
      d[i] = static_cast<uint16_t>(pack_bf16x2(s[i], 0.0f) & 0xFFFFu);
  } else {
    const uint16_t* __restrict__ s = static_cast<const uint16_t*>(b.src[t]);
    float* __restrict__ d = static_cast<float*>(b.dst[t]);
    if (((reinterpret_cast<uintptr_t>(s) & 7u) | (reinterpret_cast<uintptr_t>(d) & 15u)) == 0) {
      const int64_t end4 = begin + ((end - begin) & ~int64_t(3));
      for (int64_t i = begin + 4 * threadIdx.x; i < end4; i += 4 * kCastThreads) {
        const uint2 v = *reinterpret_cast<const uint2*>(s + i);
        *reinterpret_cast<float4*>(d + i) = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                                        __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
      }
      tail = end4;
    }
    for (int64_t i = tail + threadIdx.x; i < end; i += kCastThreads)
      d[i] = __uint_as_float(static_cast<uint32_t>(s[i]) << 16);
  }
}

}  // namespace fp8b

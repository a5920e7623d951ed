// attention.cuh — FP8 self-attention of the UNet's attention blocks on tcgen05.
//
// The reference computes, per attention block (diffusion/unet.py:189-199),
//   q, k, v = chunk(qkv, 3); o = scaled_dot_product_attention(q, k, v)
// with nh = 4 heads of 64 channels, in bf16 (autocast).  Here one CTA owns one
// (image, head) pair: L <= 256 tokens, head dim 64, so the whole L x L score
// matrix fits in tensor memory and no online softmax is needed.
//
// Forward (attn_fwd_fp8_kernel):
//   * q, k, v of the pair are read from the qkv projection output [B][L][3C]
//     (head h at columns h*64, C + h*64, 2C + h*64) and quantized per pair with
//     the reference's per-tensor scale s = amax/448 (1 if amax == 0,
//     fp8_kernels.py:90-102 applied to each head slice) and the cast
//     e4m3(x * (1/s)) saturating (one multiply by the fp32 reciprocal);
//   * S = Qq Kq^T on tcgen05 kind::f8f6f4 (M = 128 queries per tile, N = keys,
//     K = 64), fp32 in TMEM;
//   * softmax in fp32 from TMEM, one thread per query row: m = max_j S,
//     p_j = exp((S_j - m) * sq * sk / 8), l = sum_j p_j (fp32, unquantized);
//   * P is quantized as e4m3(p * 448) (p <= 1) and O = Pq Vq on kind::f8f6f4,
//     scaled by sv / (448 l) in the epilogue, stored bf16 to o [B][L][C];
//   * lse = m * sq * sk / 8 + ln l per row and the three scales are kept for the
//     backward.
//   Operands are K-major 128B-swizzled tiles: q and k rows hold 64 bytes of K in
//   128-byte rows (two K steps of 32), V is written transposed ([d][keys]) as it
//   is quantized so that it is a K-major B operand too.
//
// Backward (attn_bwd_kernel), the gradient of that forward with straight-through
// quantizers (the e4m3 values of q, k, v and p stand for q, k, v and p):
//   P = exp(S * c - lse) with S = Qq Kq^T recomputed, dP = sv * dO Vq^T,
//   delta = rowsum(dO o O), dS = P (dP - delta),
//   dV = P^T dO, dK = c sq dS^T Qq, dQ = c sk dS Kq      (c = 1/8 = 1/sqrt(64))
// on tcgen05 kind::f16 with bf16 operands (the e4m3 values of q, k, v are exact
// in bf16; P and dS are rounded to bf16).  Key tiles of 128 are the outer loop,
// query tiles the inner one; S and dP of one (key, query) tile pair, dV and dK of
// the key tile and dQ of both query tiles live in TMEM at once (128 + 128 + 64 +
// 64 + 2 x 64 = 512 columns).  P and dS are stored once, [query][key], and read
// K-major (dQ) or MN-major (dV, dK); q, k, v and dO once, [token][d], read
// K-major (S, dP) or MN-major (dV, dK, dQ): no transposed copies.
//
// Every mbarrier wait is bounded (mbar_wait); on a timeout the kernel records
// the error code, skips the remaining work and frees its tensor memory.
#pragma once

#include "quantize.cuh"
#include "sm100_common.cuh"

namespace fp8b {

constexpr int kAttnThreads = 256;
constexpr int kAttnHeadDim = 64;
constexpr int kAttnMaxSeq = 256;
constexpr uint32_t kAttnTmemCols = 512;

struct AttnParams {
  const uint16_t* qkv;  // bf16 [B][L][ld_qkv]
  uint16_t* o;          // bf16 [B][L][ld_o] (forward output)
  const uint16_t* o_in; // bf16 [B][L][ld_o] (forward output, backward input)
  const uint16_t* dout; // bf16 [B][L][ld_o]
  uint16_t* dqkv;       // bf16 [B][L][ld_qkv]
  float* lse;           // [B][heads][L]
  float* scales;        // [B][heads][4]: sq, sk, sv, 0
  int seq, heads, ld_qkv, ld_o;
  int* err;
};

// kind::f16 instruction descriptor: bf16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
         (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Per-tensor scale of the reference quantize: amax/448 in IEEE fp32, 1 for amax 0.
__device__ __forceinline__ float attn_scale(float amax) { return amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f; }

// The attention's cast of q, k, v: e4m3(RN(x * r)) with r = RN(1 / s) in fp32 (saturating at
// +-448), one multiply per element -- the attention has no reference kernel whose division
// bits it must match, and this cast is what the oracle restates.
__device__ __forceinline__ uint2 quant8_bf16(const uint4& v, float r) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) b[i] = cvt_e4m3x2(bf16_lo_f(w[i]) * r, bf16_hi_f(w[i]) * r);
  return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
}

__device__ __forceinline__ float attn_recip(float s) { return __fdiv_rn(1.0f, s); }

// 2^x (the SFU's approximation; relative error ~2^-22).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two e4m3 bytes (low byte first) -> the same two values as bf16x2 (exact: e4m3 values are
// f16 and bf16 values).
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t two) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(two & 0xFFFFu)));
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
  return pack_bf16x2(f.x, f.y);
}

// The 8 bf16 of a chunk -> the bf16 of their e4m3 values quant8_bf16(x, r) (exact in bf16).
__device__ __forceinline__ uint4 quant_dequant8_bf16(const uint4& v, float r) {
  const uint2 q = quant8_bf16(v, r);
  return make_uint4(e4m3x2_to_bf16x2(q.x), e4m3x2_to_bf16x2(q.x >> 16), e4m3x2_to_bf16x2(q.y),
                    e4m3x2_to_bf16x2(q.y >> 16));
}

__device__ __forceinline__ float bf16x8_absmax(const uint4& v) {
  float m = 0.0f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) m = fmaxf(m, fmaxf(fabsf(bf16_lo_f(w[i])), fabsf(bf16_hi_f(w[i]))));
  return m;
}

// Maximum over the CTA of three per-thread values (all threads call it).
__device__ __forceinline__ void block_max3(float (&v)[3], float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < 3; ++t)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[t] = fmaxf(v[t], __shfl_xor_sync(0xffffffffu, v[t], o));
  if (lane == 0)
#pragma unroll
    for (int t = 0; t < 3; ++t) red[t * 8 + warp] = v[t];
  __syncthreads();
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    float m = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnThreads / 32; ++w) m = fmaxf(m, red[t * 8 + w]);
    v[t] = m;
  }
}

// Byte offset of 16-byte chunk `chunk` of `row` in a K-major 128B-swizzled tile
// stack (128-row tiles of 128-byte rows, 16 KB apart).
__device__ __forceinline__ uint32_t sw128_row_chunk(int row, int chunk) {
  return static_cast<uint32_t>((row >> 7) * 16384) + swizzle128_offset(row & 127, chunk);
}

// ============================================================================ forward
// One CTA per (image, head, 128-query tile): 96 KB of shared memory, 256 TMEM
// columns and at most 128 registers per thread, so two CTAs share an SM and one
// CTA's loads overlap the other's softmax.  Each CTA reads its pair's whole q
// (for the per-pair scale), k and v.
struct AttnFwdLayout {
  static constexpr int kQ = 0;          // 16 KB: this tile's q rows, 64 of 128 bytes used
  static constexpr int kK = 16384;      // 2 x 16 KB: k rows (keys)
  static constexpr int kVt = 49152;     // 2 x 8 KB: v^T, [d][keys], keys in 128-byte K blocks
  static constexpr int kP = 65536;      // 2 x 16 KB: p, [query][keys]
  static constexpr int kRed = 98304;    // row max / sum exchange [2][128] floats, amax scratch
  static constexpr int kBar = kRed + 1024 + 128;
  static constexpr int kBytes = kBar + 64;
  static constexpr int kSmemBytes = kBytes + 1024;  // + alignment slack
};
static_assert(2 * AttnFwdLayout::kSmemBytes <= 232448, "two attention-forward CTAs per SM");
constexpr uint32_t kAttnFwdTmemCols = 256;

// |x| max of one tensor's head slice (rows < L, 16-byte chunks c = tid + 256 r).
__device__ __forceinline__ float head_absmax(const uint16_t* col0, int L, int ld) {
  uint32_t m2 = 0u;
#pragma unroll 4
  for (int c = threadIdx.x; c < L * 8; c += kAttnThreads)
    m2 = bf16x2_max(m2, absmax_vec2(__ldg(reinterpret_cast<const uint4*>(col0 + static_cast<int64_t>(c >> 3) * ld +
                                                                          (c & 7) * 8))));
  return unpack_max2(m2);
}

__global__ void __launch_bounds__(kAttnThreads, 2) attn_fwd_fp8_kernel(const AttnParams p) {
  using Ly = AttnFwdLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + Ly::kRed);  // [2][128] row partials, then amax scratch at +1024
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + Ly::kBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_o + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.seq;
  const int nkp = (L + 31) & ~31;  // keys, padded to the e4m3 K step
  const int nqt = (L + 127) >> 7;  // query tiles
  const int pair = blockIdx.x / nqt, tile = blockIdx.x - pair * nqt;
  const int b = pair / p.heads, h = pair - b * p.heads;
  const int C = p.heads * kAttnHeadDim;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kAttnFwdTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  // ---- per-pair scales from the whole head slices of q, k, v
  const uint16_t* src = p.qkv + static_cast<int64_t>(b) * L * p.ld_qkv + h * kAttnHeadDim;
  float amax[3] = {head_absmax(src, L, p.ld_qkv), head_absmax(src + C, L, p.ld_qkv),
                   head_absmax(src + 2 * C, L, p.ld_qkv)};
  block_max3(amax, red + 256);
  const float sq = attn_scale(amax[0]), sk = attn_scale(amax[1]), sv = attn_scale(amax[2]);
  const float rq = attn_recip(sq), rk = attn_recip(sk), rv = attn_recip(sv);

  // ---- quantize into the operand tiles (second read of the slices: L1 / L2 hits)
  for (int c = tid; c < 128 * 8; c += kAttnThreads) {  // this tile's q rows
    const int r = c >> 3, c16 = c & 7, row = tile * 128 + r;
    const uint2 qb = row < L ? quant8_bf16(__ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(row) *
                                                                                 p.ld_qkv + c16 * 8)), rq)
                             : make_uint2(0, 0);
    *reinterpret_cast<uint2*>(smem + Ly::kQ + swizzle128_offset(r, c16 >> 1) + (c16 & 1) * 8) = qb;
  }
  for (int c = tid; c < nkp * 8; c += kAttnThreads) {  // k rows
    const int row = c >> 3, c16 = c & 7;
    const uint2 kb = row < L ? quant8_bf16(__ldg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(row) *
                                                                                 p.ld_qkv + C + c16 * 8)), rk)
                             : make_uint2(0, 0);
    *reinterpret_cast<uint2*>(smem + Ly::kK + sw128_row_chunk(row, c16 >> 1) + (c16 & 1) * 8) = kb;
  }
  {
    // v^T: this thread's 8 consecutive keys vkey0 .. + 7 at channels 8 vc16 .. 8 vc16 + 7; byte e of
    // key vkey0 + r goes to row d = 8 vc16 + e, so each row gets 8 consecutive bytes (keys past L: 0)
    const int vkey0 = (tid >> 3) * 8, vc16 = tid & 7;
    if (vkey0 < nkp) {
      uint2 vb[8];
#pragma unroll
      for (int r = 0; r < 8; ++r)
        vb[r] = vkey0 + r < L ? quant8_bf16(__ldg(reinterpret_cast<const uint4*>(
                                                src + static_cast<int64_t>(vkey0 + r) * p.ld_qkv + 2 * C + vc16 * 8)),
                                            rv)
                              : make_uint2(0, 0);
      const int kb_blk = vkey0 >> 7, kr = vkey0 & 127;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          lo |= ((((e < 4 ? vb[r].x : vb[r].y) >> ((e & 3) * 8)) & 0xFFu) << (8 * r));
          hi |= ((((e < 4 ? vb[r + 4].x : vb[r + 4].y) >> ((e & 3) * 8)) & 0xFFu) << (8 * r));
        }
        const int d = vc16 * 8 + e;
        const uint32_t o = kb_blk * 8192 + d * 128 + ((((kr >> 4) ^ (d & 7)) & 7) << 4) + (kr & 15);
        *reinterpret_cast<uint2*>(smem + Ly::kVt + o) = make_uint2(lo, hi);
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();

  // ---- S = Qq Kq^T (TMEM columns [0, nkp))
  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = make_idesc_e4m3(128, nkp, 0, 0);
    const uint32_t sa = smem_u32(smem + Ly::kQ), sb = smem_u32(smem + Ly::kK);
#pragma unroll
    for (int k = 0; k < 2; ++k)
      umma_f8(tmem, make_smem_desc(sa + k * 32, 16, 1024), make_smem_desc(sb + k * 32, 16, 1024), idesc,
              k > 0 ? 1u : 0u);
    umma_commit(bar_s);
  }

  // ---- softmax: query row r (lanes of quadrant warp % 4), 32-column chunks of parity half = warp / 4
  const int quad = warp & 3, half = warp >> 2, r = quad * 32 + lane, qi = tile * 128 + r;
  const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
  const float c2 = sq * sk * 0.125f * 1.4426950408889634f;  // raw S -> log2 units
  const int nchunks = nkp >> 5;
  bool ok = __all_sync(0xffffffffu, mbar_wait(bar_s, 0, abort_flag, p.err, kErrTimeoutEpilogue));
  float m = -INFINITY, l = 0.0f;
  if (ok) {
    tc_fence_after();
    for (int ch = half; ch < nchunks; ch += 2) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + ch * 32, v);
      tmem_ld_wait();
      const int valid = min(32, L - ch * 32);  // keys of this chunk below L
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < valid) m = fmaxf(m, __uint_as_float(v[j]));
    }
  }
  red[half * 128 + r] = m;
  __syncthreads();
  m = fmaxf(red[r], red[128 + r]);
  // P scaled by 448 into e4m3: 448 p = 2^((S - m) c2 + log2 448); S - m first (exact near the
  // max), so that large logits keep the offset
  if (ok) {
    for (int ch = half; ch < nchunks; ch += 2) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + ch * 32, v);
      tmem_ld_wait();
      const int valid = qi < L ? min(32, L - ch * 32) : 0;
      uint32_t packed[8];
      if (valid == 32) {  // whole chunk inside the sequence: no masks
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float pj[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pj[e] = exp2_approx(fmaf(__uint_as_float(v[j + e]) - m, c2, 8.807354922057604f));
            l += pj[e];
          }
          packed[j >> 2] = uint32_t(cvt_e4m3x2(pj[0], pj[1])) | (uint32_t(cvt_e4m3x2(pj[2], pj[3])) << 16);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float pj[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pj[e] = j + e < valid ? exp2_approx(fmaf(__uint_as_float(v[j + e]) - m, c2, 8.807354922057604f)) : 0.0f;
            l += pj[e];
          }
          packed[j >> 2] = uint32_t(cvt_e4m3x2(pj[0], pj[1])) | (uint32_t(cvt_e4m3x2(pj[2], pj[3])) << 16);
        }
      }
      const int kblk = ch >> 2, kc = (ch & 3) * 2;  // 16-byte chunks kc, kc + 1 of the 128-byte row
      uint8_t* base = smem + Ly::kP + kblk * 16384;
      *reinterpret_cast<uint4*>(base + swizzle128_offset(r, kc)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      *reinterpret_cast<uint4*>(base + swizzle128_offset(r, kc + 1)) =
          make_uint4(packed[4], packed[5], packed[6], packed[7]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();  // every read of S is done and P is in shared memory
  red[half * 128 + r] = l;
  if (*abort_flag) ok = false;
  if (ok && tid == 0) {
    tc_fence_after();
    const uint32_t idesc = make_idesc_e4m3(128, kAttnHeadDim, 0, 0);
    const uint32_t sp = smem_u32(smem + Ly::kP), svt = smem_u32(smem + Ly::kVt);
    for (int ks = 0; ks < nchunks; ++ks) {
      const int kblk = ks >> 2, k = ks & 3;
      umma_f8(tmem, make_smem_desc(sp + kblk * 16384 + k * 32, 16, 1024),
              make_smem_desc(svt + kblk * 8192 + k * 32, 16, 1024), idesc, ks > 0 ? 1u : 0u);
    }
    umma_commit(bar_o);
  }
  __syncthreads();
  l = red[r] + red[128 + r];  // sum of 448 p over the row
  if (ok) ok = mbar_wait(bar_o, 0, abort_flag, p.err, kErrTimeoutEpilogue);
  if (__all_sync(0xffffffffu, ok)) {
    tc_fence_after();
    uint32_t o[32];
    tmem_ld_32x32b_x32(trow + half * 32, o);  // output channels [32 half, 32 half + 32)
    tmem_ld_wait();
    if (qi < L) {
      const float f = __fdiv_rn(sv, l);
      uint16_t* dst = p.o + (static_cast<int64_t>(b) * L + qi) * p.ld_o + h * kAttnHeadDim + half * 32;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8)
        reinterpret_cast<uint4*>(dst)[c8] =
            make_uint4(pack_bf16x2(__uint_as_float(o[8 * c8]) * f, __uint_as_float(o[8 * c8 + 1]) * f),
                       pack_bf16x2(__uint_as_float(o[8 * c8 + 2]) * f, __uint_as_float(o[8 * c8 + 3]) * f),
                       pack_bf16x2(__uint_as_float(o[8 * c8 + 4]) * f, __uint_as_float(o[8 * c8 + 5]) * f),
                       pack_bf16x2(__uint_as_float(o[8 * c8 + 6]) * f, __uint_as_float(o[8 * c8 + 7]) * f));
      // lse of the logits S sq sk / 8:  m c + ln(l / 448)
      if (half == 0) p.lse[static_cast<int64_t>(pair) * L + qi] = m * (sq * sk * 0.125f) + logf(l * (1.0f / 448.0f));
    }
  }
  if (tid == 0 && tile == 0) {
    float* sc = p.scales + static_cast<int64_t>(pair) * 4;
    sc[0] = sq;
    sc[1] = sk;
    sc[2] = sv;
    sc[3] = 0.0f;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnFwdTmemCols);
  }
}

// ============================================================================ backward
struct AttnBwdLayout {
  static constexpr int kQ = 0;        // 2 x 16 KB each: bf16 [token][64], 128-byte rows
  static constexpr int kK = 32768;
  static constexpr int kV = 65536;
  static constexpr int kDO = 98304;
  static constexpr int kP = 131072;   // 2 x 16 KB: bf16 [query][key], 64-key blocks
  static constexpr int kDS = 163840;  // same for dS
  static constexpr int kLse = 196608; // fp32 [256]
  static constexpr int kDelta = kLse + 1024;
  static constexpr int kBar = kDelta + 1024;
  static constexpr int kBytes = kBar + 128;
  static constexpr int kSmemBytes = kBytes + 1024;
};
static_assert(AttnBwdLayout::kSmemBytes <= 232448, "attention backward smem");

// TMEM columns of the backward's accumulators.
constexpr uint32_t kBwdS = 0, kBwdDP = 128, kBwdDV = 256, kBwdDK = 320, kBwdDQ = 384;

// 64 fp32 columns of one TMEM row quarter-lane -> 64 bf16 * f stored to dst (128 bytes).
__device__ __forceinline__ void store_row64(uint32_t taddr, float f, uint16_t* dst, bool store) {
  uint32_t a[32], c[32];
  tmem_ld_32x32b_x32(taddr, a);
  tmem_ld_32x32b_x32(taddr + 32, c);
  tmem_ld_wait();
  if (!store) return;
#pragma unroll
  for (int c8 = 0; c8 < 8; ++c8) {
    const uint32_t* s = c8 < 4 ? a + 8 * c8 : c + 8 * (c8 - 4);
    reinterpret_cast<uint4*>(dst)[c8] =
        make_uint4(pack_bf16x2(__uint_as_float(s[0]) * f, __uint_as_float(s[1]) * f),
                   pack_bf16x2(__uint_as_float(s[2]) * f, __uint_as_float(s[3]) * f),
                   pack_bf16x2(__uint_as_float(s[4]) * f, __uint_as_float(s[5]) * f),
                   pack_bf16x2(__uint_as_float(s[6]) * f, __uint_as_float(s[7]) * f));
  }
}

__global__ void __launch_bounds__(kAttnThreads, 1) attn_bwd_kernel(const AttnParams p) {
  using Ly = AttnBwdLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* lse_s = reinterpret_cast<float*>(smem + Ly::kLse);
  float* delta_s = reinterpret_cast<float*>(smem + Ly::kDelta);
  uint64_t* bar_sp = reinterpret_cast<uint64_t*>(smem + Ly::kBar);
  uint64_t* bar_acc = bar_sp + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_acc + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.seq;
  const int npad = (L + 31) & ~31;
  const int ntile = (L + 127) >> 7;  // key tiles = query tiles
  const int b = blockIdx.x / p.heads, h = blockIdx.x - (blockIdx.x / p.heads) * p.heads;
  const int C = p.heads * kAttnHeadDim;

  if (tid == 0) {
    mbar_init(bar_sp, 1);
    mbar_init(bar_acc, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  const int64_t pair = static_cast<int64_t>(b) * p.heads + h;
  const float* sc = p.scales + pair * 4;
  const float sq = sc[0], sk = sc[1], sv = sc[2];
  const float rq = attn_recip(sq), rk = attn_recip(sk), rv = attn_recip(sv);
  const uint16_t* src = p.qkv + static_cast<int64_t>(b) * L * p.ld_qkv + h * kAttnHeadDim;
  const uint16_t* dsrc = p.dout + static_cast<int64_t>(b) * L * p.ld_o + h * kAttnHeadDim;
  const uint16_t* osrc = p.o_in + static_cast<int64_t>(b) * L * p.ld_o + h * kAttnHeadDim;

  // ---- operands: e4m3 values of q, k, v (as bf16) and dO, [token][64]; rows past L zero
  for (int c = tid; c < 2 * 128 * 8; c += kAttnThreads) {
    const int row = c >> 3, c16 = c & 7;
    const uint32_t off = sw128_row_chunk(row, c16);
    uint4 q = make_uint4(0, 0, 0, 0), k = q, v = q, d = q;
    if (row < L) {
      const uint16_t* s = src + static_cast<int64_t>(row) * p.ld_qkv + c16 * 8;
      q = quant_dequant8_bf16(__ldg(reinterpret_cast<const uint4*>(s)), rq);
      k = quant_dequant8_bf16(__ldg(reinterpret_cast<const uint4*>(s + C)), rk);
      v = quant_dequant8_bf16(__ldg(reinterpret_cast<const uint4*>(s + 2 * C)), rv);
      d = __ldg(reinterpret_cast<const uint4*>(dsrc + static_cast<int64_t>(row) * p.ld_o + c16 * 8));
    }
    *reinterpret_cast<uint4*>(smem + Ly::kQ + off) = q;
    *reinterpret_cast<uint4*>(smem + Ly::kK + off) = k;
    *reinterpret_cast<uint4*>(smem + Ly::kV + off) = v;
    *reinterpret_cast<uint4*>(smem + Ly::kDO + off) = d;
  }
  // ---- per query row: lse and delta = sum_d dO * O
  for (int row = tid; row < kAttnMaxSeq; row += kAttnThreads) {
    float lse = 0.0f, delta = 0.0f;
    if (row < L) {
      lse = p.lse[pair * L + row];
      const uint4* d4 = reinterpret_cast<const uint4*>(dsrc + static_cast<int64_t>(row) * p.ld_o);
      const uint4* o4 = reinterpret_cast<const uint4*>(osrc + static_cast<int64_t>(row) * p.ld_o);
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const uint4 dv = __ldg(d4 + c8), ov = __ldg(o4 + c8);
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, ow[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          delta += bf16_lo_f(dw[e]) * bf16_lo_f(ow[e]) + bf16_hi_f(dw[e]) * bf16_hi_f(ow[e]);
      }
    }
    lse_s[row] = lse;
    delta_s[row] = delta;
  }
  fence_proxy_async_smem();
  __syncthreads();

  const float cs2 = sq * sk * 0.125f * 1.4426950408889634f;  // raw S -> logits in log2 units
  const int quad = warp & 3, half = warp >> 2, r = quad * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t sQ = smem_u32(smem + Ly::kQ), sK = smem_u32(smem + Ly::kK), sV = smem_u32(smem + Ly::kV),
                 sDO = smem_u32(smem + Ly::kDO), sP = smem_u32(smem + Ly::kP), sDS = smem_u32(smem + Ly::kDS);
  bool ok = true;
  int it = 0;
  for (int j = 0; j < ntile && ok; ++j) {
    const int nk = min(128, npad - 128 * j);  // keys of this tile (multiple of 32)
    for (int i = 0; i < ntile && ok; ++i, ++it) {
      const int nq = min(128, npad - 128 * i);
      if (tid == 0) {
        tc_fence_after();
        const uint32_t idesc = make_idesc_bf16(128, nk, 0, 0);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          umma_bf16(tmem + kBwdS, make_smem_desc(sQ + i * 16384 + k * 32, 16, 1024),
                    make_smem_desc(sK + j * 16384 + k * 32, 16, 1024), idesc, k > 0 ? 1u : 0u);
          umma_bf16(tmem + kBwdDP, make_smem_desc(sDO + i * 16384 + k * 32, 16, 1024),
                    make_smem_desc(sV + j * 16384 + k * 32, 16, 1024), idesc, k > 0 ? 1u : 0u);
        }
        umma_commit(bar_sp);
      }
      ok = mbar_wait(bar_sp, it & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      if (ok && it > 0) ok = mbar_wait(bar_acc, (it - 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      if (ok) {
        tc_fence_after();
        const int qi = i * 128 + r;
        const float lse2 = lse_s[qi < kAttnMaxSeq ? qi : 0] * 1.4426950408889634f;  // log2 units
        const float delta = delta_s[qi < kAttnMaxSeq ? qi : 0];
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          const int col0 = half * 64 + cc * 32;  // key column within the tile
          uint32_t s[32], dp[32];
          if (col0 < nk) {
            tmem_ld_32x32b_x32(tmem + lane_off + kBwdS + col0, s);
            tmem_ld_32x32b_x32(tmem + lane_off + kBwdDP + col0, dp);
            tmem_ld_wait();
          }
          uint32_t pw[16], dw[16];
#pragma unroll
          for (int jj = 0; jj < 32; jj += 2) {
            float pv[2], dv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int key = j * 128 + col0 + jj + e;
              const bool valid = col0 < nk && qi < L && key < L;
              const float pe = valid ? exp2_approx(fmaf(__uint_as_float(s[jj + e]), cs2, -lse2)) : 0.0f;
              pv[e] = pe;
              dv[e] = valid ? pe * (__uint_as_float(dp[jj + e]) * sv - delta) : 0.0f;
            }
            pw[jj >> 1] = pack_bf16x2(pv[0], pv[1]);
            dw[jj >> 1] = pack_bf16x2(dv[0], dv[1]);
          }
          // keys col0 .. col0+31: 64-key block col0 / 64, chunks (col0 % 64) / 8 .. + 3
          const int blk = col0 >> 6, ch = (col0 & 63) >> 3;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t off = blk * 16384 + swizzle128_offset(r, ch + u);
            *reinterpret_cast<uint4*>(smem + Ly::kP + off) =
                make_uint4(pw[4 * u], pw[4 * u + 1], pw[4 * u + 2], pw[4 * u + 3]);
            *reinterpret_cast<uint4*>(smem + Ly::kDS + off) =
                make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (*abort_flag) ok = false;
      if (ok && tid == 0) {
        tc_fence_after();
        const uint32_t idesc_kv = make_idesc_bf16(128, kAttnHeadDim, 1, 1);
        for (int ks = 0; ks < nq / 16; ++ks) {
          const uint32_t acc = (i > 0 || ks > 0) ? 1u : 0u;
          umma_bf16(tmem + kBwdDV, make_smem_desc(sP + ks * 2048, 16384, 1024),
                    make_smem_desc(sDO + i * 16384 + ks * 2048, 16384, 1024), idesc_kv, acc);
          umma_bf16(tmem + kBwdDK, make_smem_desc(sDS + ks * 2048, 16384, 1024),
                    make_smem_desc(sQ + i * 16384 + ks * 2048, 16384, 1024), idesc_kv, acc);
        }
        const uint32_t idesc_q = make_idesc_bf16(128, kAttnHeadDim, 0, 1);
        for (int kk = 0; kk < nk / 16; ++kk)
          umma_bf16(tmem + kBwdDQ + 64 * i, make_smem_desc(sDS + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    make_smem_desc(sK + j * 16384 + kk * 2048, 16384, 1024), idesc_q, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar_acc);
      }
      if (ok && i == ntile - 1) {
        // dV and dK of key tile j are complete once this iteration's MMAs are
        ok = __all_sync(0xffffffffu, mbar_wait(bar_acc, it & 1, abort_flag, p.err, kErrTimeoutEpilogue));
        if (ok) {
          tc_fence_after();
          const int key = j * 128 + r;
          uint16_t* dst = p.dqkv + (static_cast<int64_t>(b) * L + (key < L ? key : 0)) * p.ld_qkv + h * kAttnHeadDim;
          if (half == 0)
            store_row64(tmem + lane_off + kBwdDV, 1.0f, dst + 2 * C, key < L);
          else
            store_row64(tmem + lane_off + kBwdDK, 0.125f * sq, dst + C, key < L);
        }
        tc_fence_before();
        __syncthreads();
        if (*abort_flag) ok = false;
      }
    }
  }
  if (ok && half < ntile) {
    // the last iteration's accumulator commit was waited for above (i == ntile - 1)
    tc_fence_after();
    const int qi = half * 128 + r;
    uint16_t* dst = p.dqkv + (static_cast<int64_t>(b) * L + (qi < L ? qi : 0)) * p.ld_qkv + h * kAttnHeadDim;
    store_row64(tmem + lane_off + kBwdDQ + 64 * half, 0.125f * sk, dst, qi < L);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }
}

}  // namespace fp8b

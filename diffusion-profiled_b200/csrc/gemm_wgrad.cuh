// gemm_wgrad.cuh — tcgen05 FP8 weight-gradient GEMM with MN-major operands and
// split-K over the pixel (token) dimension:
//
//   acc[co, j] += sum_{m in split s} dY[m, co] * B[m, j]      (every split s, in L2)
//   dW[co, j]   = bf16( acc[co, j] * sx * sdy )
//
// 3x3 conv (reference conv2d_dw_fp8_kernel + conv2d_dw_reduce_fp8_kernel,
// fp8_kernels.py:385-468): j = tap * Cin + ci and B[m, j] = Xq at pixel m shifted
// by the tap (zero outside the image, from TMA out-of-bounds fill), so dW comes
// out as [Cout][3][3][Cin], the channels_last layout of [Cout, Cin, 3, 3].
// FP8 linear: B = Xq [M][K] and dW = [N][K], the nn.Linear weight layout.
//
// Both operands are read in their natural row-major layout: dY rows are
// [pixels][Cout] (co contiguous) and X rows are [pixels][C] (channel contiguous),
// i.e. MN-major for this contraction, so the transpose of dY that the reference
// performs before its dW kernel (fp8_kernels.py:754-771) is not needed.
//
// Halo mode (3x3 conv with W in {16, 32}, G = 3): a column group is one column
// tap kw and one 128-channel chunk, and its three boxes are the row taps
// kh = 0, 1, 2.  X is MN-major here (pixels are K), so one 4-D TMA box of R+2
// image rows (R = 128 / W rows per 128-pixel K block, one halo row above and
// below) holds all three: row tap kh starts kh*W rows into the box, a whole
// number of 1024-byte swizzle atoms.  kh = 0 and 1 are one N = 256 MMA whose
// two 128-column blocks are W*128 bytes apart (the descriptor's leading byte
// offset), kh = 2 an N = 128 MMA.  Per K block the CTA loads 16 KB of dY and
// (R+2)*W*128 bytes of X instead of 16 KB + 3 x 16 KB.
//
// Each CTA owns one output tile (128 rows of co x G*128 columns of j) and one
// K split; it is not persistent.  Roles as in the K-major kernel: warp 0 TMA,
// warp 1 TMEM + MMA, warps 2..5 move the fp32 tile out.  Split results are
// summed by TMA reduce-add (cp.reduce.async.bulk.tensor .add) into one fp32
// accumulator that the host zeroes first, instead of materialising one partial
// matrix per split and reading them all back (the reference's reduce kernel);
// the order of those fp32 additions is not fixed.
#pragma once

#include "gemm_kmajor.cuh"

namespace fp8b {

constexpr int kBoxBytes = 128 * 128;  // one 128 (K rows) x 128 (bytes of MN) TMA box

struct WGradParams {
  int num_tiles;       // co tiles x column groups
  int num_groups;      // column groups (G boxes of 128 columns each)
  int splits;
  int k_blocks;        // ceil(pixels / 128)
  int b_conv;          // 1: B is a 3x3 conv window over NHWC X, 0: plain [M][K]
  int HW, W, cchunks;  // conv geometry
  int halo_box_bytes;  // halo mode: bytes of one X box ((128 / W + 2) * W * 128)
  int n_cols;          // columns of the partial / dW rows (9*Cin or K)
  int m_rows;          // rows of dW (Cout or N)
  float* acc;          // [m_rows][n_cols] fp32, zeroed before the launch
  int* err;
  // Fused conversion (cooperative launch, every CTA resident): after the last split's
  // reduce-add, out = acc * (*scale_a) * (*scale_b) as bf16, or those bf16 values widened to
  // fp32 (out_f32), each CTA converting its share after a grid barrier.  grid_arrive == null:
  // the conversion is a separate launch (wgrad_reduce_kernel).
  unsigned int* grid_arrive;
  unsigned int* grid_depart;
  const float* scale_a;
  const float* scale_b;
  void* out;
  int out_f32;
};

// out[i] = convert(acc[i] * scale) for this CTA's share of the m_rows x n_cols accumulator
// (four elements per step; the count is a multiple of 4).
__device__ __forceinline__ void wgrad_convert_share(const WGradParams& p) {
  const int64_t n4 = static_cast<int64_t>(p.m_rows) * p.n_cols / 4;
  const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
  const int64_t b = per * blockIdx.x, e = min(n4, b + per);
  const float scale = __ldg(p.scale_a) * __ldg(p.scale_b);
  const float4* a4 = reinterpret_cast<const float4*>(p.acc);
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) {
    const float4 v = __ldcg(a4 + i);
    const uint32_t lo = pack_bf16x2(v.x * scale, v.y * scale), hi = pack_bf16x2(v.z * scale, v.w * scale);
    if (p.out_f32)
      reinterpret_cast<float4*>(p.out)[i] = make_float4(__uint_as_float(lo << 16), __uint_as_float(lo & 0xFFFF0000u),
                                                        __uint_as_float(hi << 16), __uint_as_float(hi & 0xFFFF0000u));
    else
      reinterpret_cast<uint2*>(p.out)[i] = make_uint2(lo, hi);
  }
}

constexpr int kMaxHaloBoxBytes = (128 / 32 + 2) * 32 * 128;  // W = 32 (W = 16 needs 20 KB)

template <int G, bool HALO = false>
struct WGradConfig {
  static_assert(!HALO || G == 3, "halo mode groups the three row taps");
  static constexpr int kStageBytes = HALO ? kBoxBytes + kMaxHaloBoxBytes : (1 + G) * kBoxBytes;
  static constexpr int kStages = HALO ? 4 : ((G == 1) ? 6 : (G == 2 ? 4 : 3));
  static constexpr int kAccCols = G * 128;
  static constexpr int kTmemCols = (kAccCols <= 128) ? 128 : (kAccCols <= 256 ? 256 : 512);
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiSmemBytes + 1024 + 1024;
  static_assert(kSmemBytes <= 232448, "smem");
};

template <int G, bool HALO = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    wgrad_fp8_kernel(const __grid_constant__ CUtensorMap tmap_dy, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_acc, const WGradParams p) {
  using Cfg = WGradConfig<G, HALO>;
  constexpr int STAGES = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + STAGES * Cfg::kStageBytes;
  uint8_t* bar_area = epi_smem + kEpiSmemBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* drain_bar = tfull_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int tile = blockIdx.x % p.num_tiles;
  const int split = blockIdx.x / p.num_tiles;
  const int co_tile = tile / p.num_groups;
  const int group = tile - co_tile * p.num_groups;
  const int kb_begin = static_cast<int>((static_cast<int64_t>(split) * p.k_blocks) / p.splits);
  const int kb_end = static_cast<int>((static_cast<int64_t>(split + 1) * p.k_blocks) / p.splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_dy);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_acc);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_sync();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full_bar[stage], HALO ? kBoxBytes + p.halo_box_bytes : Cfg::kStageBytes);
        const int m0 = kb * 128;
        tma_load_2d(sa, &tmap_dy, &full_bar[stage], co_tile * 128, m0);
        if (HALO) {
          const int img = m0 / p.HW;
          const int h0 = (m0 - img * p.HW) / p.W;
          const int kw = group % 3, chunk = group / 3;
          tma_load_4d(sa + kBoxBytes, &tmap_b, &full_bar[stage], chunk * 128, kw - 1, h0 - 1, img);
        } else if (p.b_conv) {
          const int img = m0 / p.HW;
          const int h0 = (m0 - img * p.HW) / p.W;
#pragma unroll
          for (int b = 0; b < G; ++b) {
            const int gb = group * G + b;
            const int tap = gb / p.cchunks;
            const int chunk = gb - tap * p.cchunks;
            const int kh = tap / 3, kw = tap - 3 * (tap / 3);
            tma_load_4d(sa + (1 + b) * kBoxBytes, &tmap_b, &full_bar[stage], chunk * 128, kw - 1, h0 + kh - 1,
                        img);
          }
        } else {
#pragma unroll
          for (int b = 0; b < G; ++b)
            tma_load_2d(sa + (1 + b) * kBoxBytes, &tmap_b, &full_bar[stage], (group * G + b) * 128, m0);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        const int64_t first = issued > STAGES ? issued - STAGES : 0;
        volatile int never = 0;
        for (int64_t i = first; i < issued; ++i)
          mbar_wait(&full_bar[i % STAGES], uint32_t((i / STAGES) & 1), &never, p.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_pair = make_idesc_e4m3(128, 256, 1, 1);
      constexpr uint32_t idesc_single = make_idesc_e4m3(128, 128, 1, 1);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
        const uint32_t accumulate_base = (kb != kb_begin) ? 1u : 0u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // 4 x 32 K rows per 128-row block
          // MN-major SW128: 8-row core groups 1024 B apart (SBO); 128-column blocks
          // of the operand 16 KB apart (LBO).
          const uint64_t adesc = make_smem_desc(sa + k * 4096, kBoxBytes, 1024);
          const uint32_t acc = (accumulate_base | (k != 0 ? 1u : 0u));
          if (HALO) {
            // row taps 0 and 1: two 128-column blocks W*128 bytes apart; row tap 2 alone
            const uint32_t sb = sa + kBoxBytes + k * 4096;
            const uint32_t row = static_cast<uint32_t>(p.W) * 128u;
            umma_f8(tmem_base, adesc, make_smem_desc(sb, row, 1024), idesc_pair, acc);
            umma_f8(tmem_base + 256, adesc, make_smem_desc(sb + 2 * row, kBoxBytes, 1024), idesc_single, acc);
          } else {
#pragma unroll
            for (int b = 0; b + 1 < G + 1; b += 2) {
              const uint64_t bdesc = make_smem_desc(sa + (1 + b) * kBoxBytes + k * 4096, kBoxBytes, 1024);
              if (b + 1 < G)
                umma_f8(tmem_base + b * 128, adesc, bdesc, idesc_pair, acc);
              else
                umma_f8(tmem_base + b * 128, adesc, bdesc, idesc_single, acc);
            }
          }
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(tfull_bar);
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, p.err, kErrTimeoutDrain);
    }
  } else {
    // Epilogue: this split's fp32 rows, 32 columns (128 B) at a time, staged
    // 128B-swizzled in shared memory and added into the accumulator by TMA.
    const int quarter = warp & 3;
    uint8_t* stage_buf = epi_smem + (warp - 2) * 2 * kEpiBufBytes;
    const int row0 = co_tile * 128 + quarter * 32;
    const bool has_work = kb_end > kb_begin;
    if (has_work && mbar_wait(tfull_bar, 0, abort_flag, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      int buf = 0;
#pragma unroll 1
      for (int c = 0; c < G * 128; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (uint32_t(quarter * 32) << 16) + c, r);
        tmem_ld_wait();
        uint8_t* sbuf = stage_buf + buf * kEpiBufBytes;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(sbuf + swizzle128_offset(lane, j), r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // Halo mode: TMEM block b is row tap kh = b of column tap kw, chunk.
          const int col = HALO ? ((c >> 7) * 3 + group % 3) * p.cchunks * 128 + (group / 3) * 128 + (c & 127)
                               : group * G * 128 + c;
          tma_reduce_add_2d(&tmap_acc, sbuf, col, row0);
          bulk_commit_group();
        }
        buf ^= 1;
      }
      if (lane == 0) bulk_wait_group<0>();
    }
    // the reduce-adds are complete; order them before the generic-proxy reads after the barrier
    if (lane == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (p.grid_arrive != nullptr && grid_barrier(p.grid_arrive, p.grid_depart, p.err, kErrTimeoutGrid))
    wgrad_convert_share(p);
}

// dW[i] = bf16( (sum_s partials[s][i]) * sx * sdy ), i over rows*cols (multiple of 4):
// the reference's reduce (fp8_kernels.py:463-468) — sum the splits, then scale.
// With the in-L2 split reduction there is one "split" (the accumulator).
// OutT = float stores the same bf16 values widened to fp32: the gradient an fp32
// weight receives when autograd casts the bf16 gradient to the weight's dtype.
template <typename OutT>
__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float* __restrict__ partials, int splits,
                                                           int64_t count, const float* __restrict__ sa,
                                                           const float* __restrict__ sb, OutT* __restrict__ out) {
  pdl_wait();
  const float scale = __ldg(sa) * __ldg(sb);
  const int64_t n4 = count >> 2;
  const float4* p4 = reinterpret_cast<const float4*>(partials);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = __ldg(p4 + i);
    for (int s = 1; s < splits; ++s) {
      const float4 v = __ldg(p4 + static_cast<int64_t>(s) * n4 + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x * scale, acc.y * scale);
    o.y = pack_bf16x2(acc.z * scale, acc.w * scale);
    if constexpr (sizeof(OutT) == 2) {
      reinterpret_cast<uint2*>(out)[i] = o;
    } else {  // fp32 holding the bf16 values (exact widening)
      reinterpret_cast<float4*>(out)[i] =
          make_float4(__uint_as_float(o.x << 16), __uint_as_float(o.x & 0xFFFF0000u), __uint_as_float(o.y << 16),
                      __uint_as_float(o.y & 0xFFFF0000u));
    }
  }
}

}  // namespace fp8b

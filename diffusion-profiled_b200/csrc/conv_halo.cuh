// conv_halo.cuh — tcgen05 3x3 conv (forward and data-grad) that loads each
// input row once per column tap instead of once per tap.
//
// Same contraction as kgemm_fp8_kernel's conv mode (reference
// conv2d_fwd_fp8_kernel fp8_kernels.py:168-247, conv2d_dx_fp8_kernel :250-318):
//   OUT[m, n] = sum_{tap, c} A_tap[m, c] * B[n, tap, c]
// but the A operand is fetched differently.  A 128-pixel M tile is R = 128/W
// whole image rows (tiles never cross images: H*W >= 128).  For one
// 128-channel chunk and one column tap kw, a single 4-D TMA box of R+2 image
// rows (the tile's rows plus one halo row above and below, shifted by kw-1
// columns, zero-filled outside the image) holds the A operand of all three row
// taps kh = 0, 1, 2: tap kh is the same box viewed kh*W rows further on, and
// kh*W*128 bytes is a multiple of the 1024-byte swizzle atom for W >= 8, so the
// UMMA descriptors need no base offset.  A traffic per tile drops from 9 boxes
// of R rows to 3 boxes of R+2 rows.
//
// B (weights, K-major [N][9*C]) is either
//   * resident: the CTA's whole [BN x 9*C] slice is loaded once and stays in
//     shared memory for every tile the CTA computes (used when it fits: C = 128,
//     BN = 128, 144 KB), or
//   * streamed per tap through a ring, as in kgemm_fp8_kernel.
//
// Roles, TMEM double buffering, epilogue (TMA store of bf16 tiles) and bounded
// waits are those of kgemm_fp8_kernel.
#pragma once

#include "gemm_kmajor.cuh"

namespace fp8b {

struct HaloParams {
  int num_n_tiles;
  int num_m_tiles;     // tiles of 128 output pixels
  int cchunks;         // 128-channel chunks of the reduced dimension (C = Cin fwd, Cout dgrad)
  int HW, W, R;        // pixels per image, image width, image rows per tile (128 / W)
  int fwd;             // 1: forward (in row = out row + kh - 1), 0: data-grad (flipped taps)
  int N;               // output channels (columns)
  const float* scale_a;
  const float* scale_b;
  const __nv_bfloat16* bias;
  int epilogue;
  int* err;
};

template <int BN, bool RESIDENT_B, int W>
struct HaloConfig {
  static constexpr int R = 128 / W;
  static constexpr int kABoxBytes = (R + 2) * W * 128;     // rows of 128 channel bytes
  static constexpr int kBTileBytes = BN * kKBlockBytes;
  static constexpr int kAStages = RESIDENT_B ? 2 : 3;
  static constexpr int kBStages = RESIDENT_B ? 9 : 4;      // resident: 9 taps x 1 chunk (C = 128)
  static constexpr int kAccCols = BN;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kEpiBytes = kEpiWarps * kEpiBufBytes;  // one staging buffer per epilogue warp
  static constexpr int kSmemBytes =
      kBStages * kBTileBytes + kAStages * kABoxBytes + kEpiBytes + 1024 /*barriers*/ + 1024 /*align*/;
  static_assert(kSmemBytes <= 232448, "smem");
  static_assert((W * 128) % 1024 == 0, "row-tap shift must be a whole number of swizzle atoms");
  static_assert(kABoxBytes % 1024 == 0, "A boxes must stay 1024-byte aligned");
};

template <int BN, bool RESIDENT_B, int W>
__global__ void __launch_bounds__(kGemmThreads, 1)
    conv_halo_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_out, const HaloParams p) {
  using Cfg = HaloConfig<BN, RESIDENT_B, W>;

  constexpr int AS = Cfg::kAStages;
  constexpr int BS = Cfg::kBStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_smem = smem;
  uint8_t* a_smem = b_smem + BS * Cfg::kBTileBytes;
  uint8_t* epi_smem = a_smem + AS * Cfg::kABoxBytes;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(epi_smem + Cfg::kEpiBytes);
  uint64_t* a_empty = a_full + AS;
  uint64_t* b_full = a_empty + AS;
  uint64_t* b_empty = b_full + BS;
  uint64_t* tfull_bar = b_empty + BS;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Resident B: a CTA works on one column tile only, so its weights stay put.
  const int nt_fixed = RESIDENT_B ? static_cast<int>(blockIdx.x % p.num_n_tiles) : 0;
  const int cta_rank = RESIDENT_B ? static_cast<int>(blockIdx.x / p.num_n_tiles) : static_cast<int>(blockIdx.x);
  const int cta_count = RESIDENT_B ? static_cast<int>(gridDim.x / p.num_n_tiles) : static_cast<int>(gridDim.x);
  const int num_tiles = RESIDENT_B ? p.num_m_tiles : p.num_m_tiles * p.num_n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_out);
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

  // Column shift of the A box for column tap kw, and row shift (in image rows)
  // inside the box for row tap kh.  Forward reads input (h + kh - 1, w + kw - 1);
  // data-grad reads dY (h + 1 - kh, w + 1 - kw).
  auto col_shift = [&](int kw) { return p.fwd ? kw - 1 : 1 - kw; };
  auto row_in_box = [&](int kh) { return p.fwd ? kh : 2 - kh; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      int64_t a_issued = 0, b_issued = 0;
      bool ok = true;
      if (RESIDENT_B) {
        // all 9 taps x 1 chunk of this CTA's column tile, one barrier
        mbar_arrive_expect_tx(&b_full[0], BS * Cfg::kBTileBytes);
        for (int t = 0; t < 9; ++t)
          tma_load_2d(b_smem + t * Cfg::kBTileBytes, &tmap_b, &b_full[0], t * kKBlockBytes, nt_fixed * BN);
        b_issued = 1;
      }
      for (int i = cta_rank; i < num_tiles && ok; i += cta_count) {
        const int mt = RESIDENT_B ? i : i / p.num_n_tiles;
        const int nt = RESIDENT_B ? nt_fixed : i - mt * p.num_n_tiles;
        const int m0 = mt * kSubTileRows;
        const int img = m0 / p.HW;
        const int h0 = (m0 - img * p.HW) / W;
        for (int c = 0; c < p.cchunks && ok; ++c) {
          for (int kw = 0; kw < 3 && ok; ++kw) {
            if (!mbar_wait(&a_empty[as], aph ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&a_full[as], Cfg::kABoxBytes);
            tma_load_4d(a_smem + as * Cfg::kABoxBytes, &tmap_a, &a_full[as], c * kKBlockBytes, col_shift(kw),
                        h0 - 1, img);
            ++a_issued;
            if (++as == AS) {
              as = 0;
              aph ^= 1u;
            }
            if (!RESIDENT_B) {
              for (int kh = 0; kh < 3; ++kh) {
                if (!mbar_wait(&b_empty[bs], bph ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
                  ok = false;
                  break;
                }
                const int tap = kh * 3 + kw;
                mbar_arrive_expect_tx(&b_full[bs], Cfg::kBTileBytes);
                tma_load_2d(b_smem + bs * Cfg::kBTileBytes, &tmap_b, &b_full[bs],
                            (tap * p.cchunks + c) * kKBlockBytes, nt * BN);
                ++b_issued;
                if (++bs == BS) {
                  bs = 0;
                  bph ^= 1u;
                }
              }
            }
          }
        }
      }
      if (!ok) {
        volatile int never = 0;
        for (int64_t k = (a_issued > AS ? a_issued - AS : 0); k < a_issued; ++k)
          mbar_wait(&a_full[k % AS], uint32_t((k / AS) & 1), &never, p.err, kErrTimeoutDrain);
        if (RESIDENT_B) {
          mbar_wait(&b_full[0], 0, &never, p.err, kErrTimeoutDrain);
        } else {
          for (int64_t k = (b_issued > BS ? b_issued - BS : 0); k < b_issued; ++k)
            mbar_wait(&b_full[k % BS], uint32_t((k / BS) & 1), &never, p.err, kErrTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_e4m3(kSubTileRows, BN, 0, 0);
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      int local = 0;
      bool ok = true;
      if (RESIDENT_B) ok = mbar_wait(&b_full[0], 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) tc_fence_after();
      for (int i = cta_rank; i < num_tiles && ok; i += cta_count, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        bool first = true;
        for (int c = 0; c < p.cchunks && ok; ++c) {
          for (int kw = 0; kw < 3 && ok; ++kw) {
            if (!mbar_wait(&a_full[as], aph, abort_flag, p.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_smem + as * Cfg::kABoxBytes);
            for (int kh = 0; kh < 3; ++kh) {
              uint32_t b_base;
              if (RESIDENT_B) {
                b_base = smem_u32(b_smem + (kh * 3 + kw) * Cfg::kBTileBytes);
              } else {
                if (!mbar_wait(&b_full[bs], bph, abort_flag, p.err, kErrTimeoutMma)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                b_base = smem_u32(b_smem + bs * Cfg::kBTileBytes);
              }
              const uint32_t a_tap = a_base + row_in_box(kh) * W * 128;
#pragma unroll
              for (int k = 0; k < kKBlockBytes / 32; ++k) {
                const uint64_t adesc = make_smem_desc(a_tap + k * 32, 16, 1024);
                const uint64_t bdesc = make_smem_desc(b_base + k * 32, 16, 1024);
                umma_f8(d_tmem, adesc, bdesc, idesc, first ? 0u : 1u);
                first = false;
              }
              if (!RESIDENT_B) {
                umma_commit(&b_empty[bs]);
                if (++bs == BS) {
                  bs = 0;
                  bph ^= 1u;
                }
              }
            }
            umma_commit(&a_empty[as]);
            if (++as == AS) {
              as = 0;
              aph ^= 1u;
            }
          }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    uint8_t* sbuf = epi_smem + (warp - 2) * kEpiBufBytes;
    const float scale = __ldg(p.scale_a) * __ldg(p.scale_b);
    int local = 0;
    for (int i = cta_rank; i < num_tiles; i += cta_count, ++local) {
      const int mt = RESIDENT_B ? i : i / p.num_n_tiles;
      const int nt = RESIDENT_B ? nt_fixed : i - mt * p.num_n_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int m0 = mt * kSubTileRows + quarter * 32;
#pragma unroll 1
      for (int c = 0; c < BN; c += 64) {
        uint32_t r[64];
        const uint4 bias_chunk = load_bias_chunk(p.epilogue, p.bias, nt * BN + c, p.N, lane);
        const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + acc * Cfg::kAccCols + c;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (c + 64 >= BN) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
        }
        const int n0 = nt * BN + c;
        if (n0 >= p.N) continue;
        if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the staging buffer
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 o = epilogue8(&r[8 * j], scale, p.epilogue,
                                     p.epilogue != kEpiNone ? bias_vec(bias_chunk, j) : make_uint4(0u, 0u, 0u, 0u));
          st_shared_v4(sbuf + swizzle128_offset(lane, j), o.x, o.y, o.z, o.w);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_out, sbuf, n0, m0);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------- CTA-pair variant
// The resident-weights case (C = 128, 128 output channels per column tile) on
// a cluster of two CTAs with M = 256 tcgen05 MMAs (cta_group::2), selected by
// conv algorithm 3 only: on config 2 it measured ~7% slower than the single-CTA
// kernel, because the limit there is not shared-memory bandwidth.  A single-CTA
// M = 128, N = 128, K = 32 MMA reads 4 KB of A and 4 KB of B from shared memory,
// about what one SM's shared memory delivers in the MMA's duration; in the
// pair each SM reads its 4 KB of A and only its half of B (64 columns), so the
// same tensor-core work needs 3/4 of the shared-memory bandwidth.
//   * The pair computes 256 output pixels = 2R image rows of one image (H*W is a
//     multiple of 256); CTA rank r owns rows [128 r, 128 r + 128) of the tile:
//     its A box (R+2 rows, as above) and its accumulator lanes.
//   * Each CTA keeps 64 of the 128 weight columns resident (9 taps x 8 KB).
//   * Loads of both CTAs complete on the leader's (rank 0) full barriers, whose
//     expected byte count covers both; the leader's MMA issuer releases stages
//     and signals accumulators to both CTAs with one multicast commit; both
//     epilogues report drained accumulators to the leader's barrier.
template <int W>
struct HaloPairConfig {
  static constexpr int R = 128 / W;
  static constexpr int kABoxBytes = (R + 2) * W * 128;
  static constexpr int kBHalfBytes = 64 * kKBlockBytes;  // 64 weight columns x one tap of 128 channels
  static constexpr int kAStages = W == 32 ? 5 : 6;
  static constexpr int kTmemCols = 2 * 128;               // two 128-column accumulators
  static constexpr int kEpiBytes = kEpiWarps * kEpiBufBytes;
  static constexpr int kSmemBytes = 9 * kBHalfBytes + kAStages * kABoxBytes + kEpiBytes + 1024 + 1024;
  static_assert(kSmemBytes <= 232448, "smem");
  static_assert((W * 128) % 1024 == 0 && kABoxBytes % 1024 == 0, "swizzle-atom alignment");
};

template <int W>
__global__ void __launch_bounds__(kGemmThreads, 1)
    conv_halo_pair_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                              const __grid_constant__ CUtensorMap tmap_out, const HaloParams p) {
  using Cfg = HaloPairConfig<W>;
  constexpr int AS = Cfg::kAStages;
  constexpr uint16_t kBoth = 0x3;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_smem = smem;
  uint8_t* a_smem = b_smem + 9 * Cfg::kBHalfBytes;
  uint8_t* epi_smem = a_smem + AS * Cfg::kABoxBytes;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(epi_smem + Cfg::kEpiBytes);
  uint64_t* a_empty = a_full + AS;
  uint64_t* b_full = a_empty + AS;
  uint64_t* tfull_bar = b_full + 1;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  // Pairs own one column tile each; pair tiles are 256 pixels.
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  const int nt_fixed = pair % p.num_n_tiles;
  const int pair_rank = pair / p.num_n_tiles;
  const int pair_count = num_pairs / p.num_n_tiles;
  const int num_tiles = p.num_m_tiles / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(b_full, 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);  // one arrival per epilogue warp of each CTA
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_sync();

  auto col_shift = [&](int kw) { return p.fwd ? kw - 1 : 1 - kw; };
  auto row_in_box = [&](int kh) { return p.fwd ? kh : 2 - kh; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int as = 0;
      uint32_t aph = 0;
      int64_t a_issued = 0;
      bool ok = true;
      const uint32_t lead_b_full = mapa_shared(smem_u32(b_full), 0);
      if (leader) mbar_arrive_expect_tx(b_full, 2 * 9 * Cfg::kBHalfBytes);
      for (int t = 0; t < 9; ++t)
        tma_load_2d_pair(b_smem + t * Cfg::kBHalfBytes, &tmap_b, lead_b_full, t * kKBlockBytes,
                         nt_fixed * 128 + static_cast<int>(rank) * 64);
      for (int i = pair_rank; i < num_tiles && ok; i += pair_count) {
        const int m0 = i * 256 + static_cast<int>(rank) * kSubTileRows;
        const int img = m0 / p.HW;
        const int h0 = (m0 - img * p.HW) / W;
        for (int kw = 0; kw < 3; ++kw) {
          if (!mbar_wait(&a_empty[as], aph ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&a_full[as], 2 * Cfg::kABoxBytes);
          tma_load_4d_pair(a_smem + as * Cfg::kABoxBytes, &tmap_a, mapa_shared(smem_u32(&a_full[as]), 0), 0,
                           col_shift(kw), h0 - 1, img);
          ++a_issued;
          if (++as == AS) {
            as = 0;
            aph ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // The leader's full barriers count both CTAs' bytes: waiting on them
        // covers the copies the peer still has in flight.
        volatile int never = 0;
        for (int64_t k = (a_issued > AS ? a_issued - AS : 0); k < a_issued; ++k)
          mbar_wait(&a_full[k % AS], uint32_t((k / AS) & 1), &never, p.err, kErrTimeoutDrain);
        mbar_wait(b_full, 0, &never, p.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_e4m3(2 * kSubTileRows, 128, 0, 0);
      int as = 0;
      uint32_t aph = 0;
      int local = 0;
      bool ok = mbar_wait(b_full, 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) tc_fence_after();
      for (int i = pair_rank; i < num_tiles && ok; i += pair_count, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 128;
        bool first = true;
        for (int kw = 0; kw < 3 && ok; ++kw) {
          if (!mbar_wait(&a_full[as], aph, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(a_smem + as * Cfg::kABoxBytes);
          for (int kh = 0; kh < 3; ++kh) {
            const uint32_t b_base = smem_u32(b_smem + (kh * 3 + kw) * Cfg::kBHalfBytes);
            const uint32_t a_tap = a_base + row_in_box(kh) * W * 128;
#pragma unroll
            for (int k = 0; k < kKBlockBytes / 32; ++k) {
              const uint64_t adesc = make_smem_desc(a_tap + k * 32, 16, 1024);
              const uint64_t bdesc = make_smem_desc(b_base + k * 32, 16, 1024);
              umma_f8_pair(d_tmem, adesc, bdesc, idesc, first ? 0u : 1u);
              first = false;
            }
          }
          umma_commit_pair(&a_empty[as], kBoth);
          if (++as == AS) {
            as = 0;
            aph ^= 1u;
          }
        }
        if (ok) umma_commit_pair(&tfull_bar[acc], kBoth);
      }
      umma_commit_pair(drain_bar, 0x1);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    uint8_t* sbuf = epi_smem + (warp - 2) * kEpiBufBytes;
    const float scale = __ldg(p.scale_a) * __ldg(p.scale_b);
    const uint32_t lead_tempty[2] = {mapa_shared(smem_u32(&tempty_bar[0]), 0),
                                     mapa_shared(smem_u32(&tempty_bar[1]), 0)};
    int local = 0;
    for (int i = pair_rank; i < num_tiles; i += pair_count, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const int m0 = i * 256 + static_cast<int>(rank) * kSubTileRows + quarter * 32;
#pragma unroll 1
      for (int c = 0; c < 128; c += 64) {
        uint32_t r[64];
        const uint4 bias_chunk = load_bias_chunk(p.epilogue, p.bias, nt_fixed * 128 + c, p.N, lane);
        const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + acc * 128 + c;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (c == 64) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_tempty[acc]);
        }
        const int n0 = nt_fixed * 128 + c;
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 o = epilogue8(&r[8 * j], scale, p.epilogue,
                                     p.epilogue != kEpiNone ? bias_vec(bias_chunk, j) : make_uint4(0u, 0u, 0u, 0u));
          st_shared_v4(sbuf + swizzle128_offset(lane, j), o.x, o.y, o.z, o.w);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_out, sbuf, n0, m0);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync();  // the leader's MMAs into this CTA's TMEM are complete and both epilogues are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace fp8b

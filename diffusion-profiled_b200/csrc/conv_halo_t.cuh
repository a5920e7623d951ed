// conv_halo_t.cuh — tcgen05 3x3 conv (forward and data-grad) for a 128-channel
// reduction with the output pixels on the MMA's N side.
//
// Same contraction as conv_halo_fp8_kernel (reference conv2d_fwd_fp8_kernel
// fp8_kernels.py:168-247, conv2d_dx_fp8_kernel :250-318), computed transposed:
//   OUT^T[n, m] = sum_{tap, c} B[n, tap, c] * A_tap[m, c]
// with n the output channel (M = 128 rows of one column tile) and m the output
// pixel (N = 256 pixels per MMA).  Why: a tcgen05.commit costs the MMA issue
// stream a bubble of a few hundred cycles, which 128x128x32 instructions (64
// cycles each) cannot hide and 128x256x32 instructions (128 cycles) can; with
// 128 output channels the pixel side is the only one that reaches 256.
//   * The CTA keeps its 128 x (9 x 128) weight slice resident (the UMMA A
//     operand, 144 KB, loaded in three column-tap groups so the first tile
//     starts after one third of it).
//   * A tile is 256 pixels = 2R image rows of one image (R = 128 / W).  For
//     each column tap kw one 4-D TMA box of 2R+2 rows (zero-filled outside the
//     image) is the B operand of all three row taps: tap kh starts kh*W rows
//     into the box, a whole number of 1024-byte swizzle atoms.
//   * The accumulator (128 lanes x 256 fp32 columns) is double buffered: all
//     512 TMEM columns.
//   * The epilogue holds one output channel per thread and 32 pixels per
//     tcgen05.ld; lane pairs swap halves so that every store is a 4-byte pair
//     of channels, written straight to the NHWC bf16 output.
//   * A_MN: the data-grad can take the forward's weights [Cout][3][3][Cin] as they
//     are: per tap a 128 (Cout = K) x 128 (Cin = M) box is an MN-major UMMA A
//     operand (M contiguous), so no transposed copy of the weights is needed.
//   * Tiles are split across the persistent grid in whole rounds; the tiles
//     left over after the last whole round are cut into 128-pixel halves
//     (N = 128 MMAs), so no CTA ends a full tile behind the others.
#pragma once

#include "gemm_kmajor.cuh"

namespace fp8b {

struct HaloTParams {
  int num_n_tiles;   // output-channel tiles of 128
  int full_tiles;    // 256-pixel tiles in the batch
  int whole_tiles;   // tiles processed whole: full_tiles rounded down to a multiple of the CTAs per column tile
  int HW, W;         // pixels per image, image width
  int fwd;           // 1: forward, 0: data-grad (flipped taps)
  int N;             // output channels (row pitch of out)
  const float* scale_a;
  const float* scale_b;
  const __nv_bfloat16* bias;
  __nv_bfloat16* out;  // NHWC bf16 [B*H*W][N]
  int epilogue;
  int* err;
};

template <int W>
struct HaloTConfig {
  static constexpr int R = 128 / W;
  static constexpr int kBoxRows = 2 * R + 2;
  static constexpr int kBoxBytes = kBoxRows * W * 128;
  static constexpr int kWTapBytes = 128 * kKBlockBytes;  // 128 output channels x one tap of 128 channels
  static constexpr int kStages = 2;
  static constexpr int kTmemCols = 512;
  static constexpr int kSmemBytes = 9 * kWTapBytes + kStages * kBoxBytes + 256 /*barriers*/ + 1024 /*align*/;
  static_assert(kSmemBytes <= 232448, "smem");
  static_assert((W * 128) % 1024 == 0 && kBoxBytes % 1024 == 0, "swizzle-atom alignment");
};

template <int W, bool A_MN = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    conv_halo_t_fp8_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_w,
                           const HaloTParams p) {
  using Cfg = HaloTConfig<W>;
  constexpr int AS = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_smem = smem;
  uint8_t* box_smem = w_smem + 9 * Cfg::kWTapBytes;
  uint64_t* box_full = reinterpret_cast<uint64_t*>(box_smem + AS * Cfg::kBoxBytes);
  uint64_t* box_empty = box_full + AS;
  uint64_t* w_full = box_empty + AS;  // one per column tap kw
  uint64_t* tfull_bar = w_full + 3;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // CTAs own one column tile each; tiles of that column tile go round-robin.
  const int nt = static_cast<int>(blockIdx.x % p.num_n_tiles);
  const int cta_rank = static_cast<int>(blockIdx.x / p.num_n_tiles);
  const int cta_count = static_cast<int>(gridDim.x / p.num_n_tiles);
  const int n_whole = p.whole_tiles / cta_count;  // whole tiles per CTA
  const int halves = 2 * (p.full_tiles - p.whole_tiles);
  const int n_half = cta_rank < halves ? (halves - cta_rank + cta_count - 1) / cta_count : 0;
  const int n_items = n_whole + n_half;
  // Work item u -> first output pixel and pixel count (256 or 128).
  auto item = [&](int u, int& m0, int& npix) {
    if (u < n_whole) {
      m0 = (cta_rank + u * cta_count) * 256;
      npix = 256;
    } else {
      m0 = p.whole_tiles * 256 + (cta_rank + (u - n_whole) * cta_count) * 128;
      npix = 128;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) {
      mbar_init(&box_full[s], 1);
      mbar_init(&box_empty[s], 1);
    }
    for (int k = 0; k < 3; ++k) mbar_init(&w_full[k], 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_act);
    tma_prefetch_desc(&tmap_w);
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

  // Forward reads input (h + kh - 1, w + kw - 1); data-grad reads dY (h + 1 - kh, w + 1 - kw).
  auto col_shift = [&](int kw) { return p.fwd ? kw - 1 : 1 - kw; };
  auto row_in_box = [&](int kh) { return p.fwd ? kh : 2 - kh; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // Weights, column tap by column tap (the order the MMA loop uses them), each group
      // issued just before the first tile's box of the same column tap, so that the first
      // MMAs wait for one weight group and one box rather than all 144 KB of weights.
      // (Every CTA has at least one item: the grid is at most the tiles of a column tile.)
      int w_issued = 0;
      auto load_weights = [&](int kw) {
        ++w_issued;
        mbar_arrive_expect_tx(&w_full[kw], 3 * Cfg::kWTapBytes);
        for (int kh = 0; kh < 3; ++kh) {
          const int tap = kh * 3 + kw;
          if (A_MN)  // 3-D map over [Cout][tap][Cin]: box (128 Cin, 1 tap, 128 Cout)
            tma_load_3d(w_smem + tap * Cfg::kWTapBytes, &tmap_w, &w_full[kw], nt * 128, tap, 0);
          else
            tma_load_2d(w_smem + tap * Cfg::kWTapBytes, &tmap_w, &w_full[kw], tap * kKBlockBytes, nt * 128);
        }
      };
      int s = 0;
      uint32_t ph = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int u = 0; u < n_items && ok; ++u) {
        int m0, npix;
        item(u, m0, npix);
        const int img = m0 / p.HW;
        const int h0 = (m0 - img * p.HW) / W;
        for (int kw = 0; kw < 3; ++kw) {
          if (u == 0) load_weights(kw);
          if (!mbar_wait(&box_empty[s], ph ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&box_full[s], Cfg::kBoxBytes);
          tma_load_4d(box_smem + s * Cfg::kBoxBytes, &tmap_act, &box_full[s], 0, col_shift(kw), h0 - 1, img);
          ++issued;
          if (++s == AS) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        volatile int never = 0;
        for (int64_t k = (issued > AS ? issued - AS : 0); k < issued; ++k)
          mbar_wait(&box_full[k % AS], uint32_t((k / AS) & 1), &never, p.err, kErrTimeoutDrain);
        for (int k = 0; k < w_issued; ++k) mbar_wait(&w_full[k], 0, &never, p.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc256 = make_idesc_e4m3(128, 256, A_MN ? 1 : 0, 0);
      constexpr uint32_t idesc128 = make_idesc_e4m3(128, 128, A_MN ? 1 : 0, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = 0; u < n_items && ok; ++u) {
        int m0, npix;
        item(u, m0, npix);
        const int acc = u & 1;
        const uint32_t acc_phase = (u >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        const uint32_t idesc = npix == 256 ? idesc256 : idesc128;
        bool first = true;
        for (int kw = 0; kw < 3 && ok; ++kw) {
          if (!mbar_wait(&w_full[kw], 0, abort_flag, p.err, kErrTimeoutMma) ||
              !mbar_wait(&box_full[s], ph, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t box = smem_u32(box_smem + s * Cfg::kBoxBytes);
          for (int kh = 0; kh < 3; ++kh) {
            const uint32_t w_tap = smem_u32(w_smem + (kh * 3 + kw) * Cfg::kWTapBytes);
            const uint32_t b_tap = box + row_in_box(kh) * W * 128;
#pragma unroll
            for (int k = 0; k < kKBlockBytes / 32; ++k) {
              // K-major A: a K step is 32 bytes along a row; MN-major A: 32 rows of 128 bytes.
              const uint64_t adesc = A_MN ? make_smem_desc(w_tap + k * 4096, Cfg::kWTapBytes, 1024)
                                          : make_smem_desc(w_tap + k * 32, 16, 1024);
              const uint64_t bdesc = make_smem_desc(b_tap + k * 32, 16, 1024);
              umma_f8(d_tmem, adesc, bdesc, idesc, first ? 0u : 1u);
              first = false;
            }
          }
          umma_commit(&box_empty[s]);
          if (++s == AS) {
            s = 0;
            ph ^= 1u;
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
    // Warp w may read TMEM lanes [32 (w % 4), +32): output channels of this thread.
    const int quarter = warp & 3;
    const int ch = nt * 128 + quarter * 32 + lane;
    const float scale = __ldg(p.scale_a) * __ldg(p.scale_b);
    const float bias = p.epilogue != kEpiNone ? __bfloat162float(p.bias[ch]) : 0.0f;
    const bool odd = lane & 1;
    // Even lanes store channels (ch, ch+1) of even pixels, odd lanes (ch-1, ch) of odd pixels.
    __nv_bfloat16* out_col = p.out + (odd ? ch - 1 : ch);
    for (int u = 0; u < n_items; ++u) {
      int m0, npix;
      item(u, m0, npix);
      const int acc = u & 1;
      const uint32_t acc_phase = (u >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < npix; c += 64) {
        uint32_t r[64];
        const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + acc * 256 + c;
        tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (c + 64 >= npix) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
        }
        __nv_bfloat16* row = out_col + (static_cast<int64_t>(m0) + c + (odd ? 1 : 0)) * p.N;
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
          float v0 = __uint_as_float(r[j]) * scale;
          float v1 = __uint_as_float(r[j + 1]) * scale;
          if (p.epilogue != kEpiNone) {
            v0 += bias;
            v1 += bias;
            if (p.epilogue == kEpiBiasSilu) {
              v0 = silu_f32(v0);
              v1 = silu_f32(v1);
            }
          }
          const uint32_t w2 = pack_bf16x2(v0, v1);  // this channel at pixels j, j+1
          const uint32_t send = odd ? (w2 & 0xFFFFu) : (w2 >> 16);
          const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
          const uint32_t pair = odd ? (recv | (w2 & 0xFFFF0000u)) : ((w2 & 0xFFFFu) | (recv << 16));
          *reinterpret_cast<uint32_t*>(row + static_cast<int64_t>(j) * p.N) = pair;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace fp8b

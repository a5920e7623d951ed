// gemm_kmajor.cuh — persistent, warp-specialised tcgen05 FP8 GEMM with both
// operands K-major:   OUT[m, n] = epi( (sum_k A[m, k] * B[n, k]) * sa * sb )
//
// One kernel serves three hot-path ops:
//   * 3x3 conv forward  (reference conv2d_fwd_fp8_kernel, fp8_kernels.py:168-247):
//       A = im2col(Xq) fetched tap by tap with 4-D TMA boxes over NHWC Xq; the
//       zero padding comes from TMA out-of-bounds fill; B = Wq as [Cout][9*Cin].
//   * 3x3 conv data-grad (reference conv2d_dx_fp8_kernel, fp8_kernels.py:250-318):
//       A = dYq windows at the flipped taps (offset 1-kh, 1-kw); B = Wq re-laid
//       out as [Cin][9*Cout].
//   * FP8 linear (no reference kernel): A = Xq [M][K], B = Wq [N][K] (nn.Linear layout).
//
// Roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one lane) — fills a STAGES-deep smem ring
//   warp 1      TMEM allocator + MMA issuer (one lane) — tcgen05.mma kind::f8f6f4,
//               M=128 per sub-tile, N=BN, K=32 per instruction (4 per 128-byte K block)
//   warps 2..5  epilogue — each owns one 32-lane quarter of TMEM: tcgen05.ld the
//               fp32 accumulator 64 columns at a time, scale (+ bias, + SiLU),
//               round to bf16, write a 32x64 tile into a 128B-swizzled staging
//               buffer and TMA-store it (coalesced; rows past M and columns past
//               N are clipped by TMA).  Two accumulator buffers in TMEM let the
//               epilogue of tile i overlap the MMAs of tile i+1; the accumulator
//               is released as soon as its last TMEM load has landed.
#pragma once

#include "sm100_common.cuh"

namespace fp8b {

constexpr int kGemmThreads = 192;
constexpr int kKBlockBytes = 128;          // one 128-byte swizzle row of K per stage
constexpr int kSubTileRows = 128;          // UMMA M
constexpr int kATileBytes = kSubTileRows * kKBlockBytes;  // 16 KB
constexpr int kEpiWarps = 4;
constexpr int kEpiBufBytes = 32 * 128;     // 32 rows x 128 bytes (64 bf16 or 32 fp32 columns)
constexpr int kEpiSmemBytes = kEpiWarps * 2 * kEpiBufBytes;  // double buffered per warp

enum Epilogue : int { kEpiNone = 0, kEpiBias = 1, kEpiBiasSilu = 2 };

struct KGemmParams {
  int num_n_tiles;
  int num_tiles;
  int k_blocks;      // K / 128 (rounded up; TMA zero-fills the ragged end)
  int M, N;          // logical output extent
  // A operand source: 1 = 3x3 conv window over NHWC activations, 0 = plain [M][K]
  int a_conv;
  int HW, W;         // conv geometry (pixels per image, image width)
  int cchunks;       // conv: 128-channel chunks per tap
  int tap_sign;      // conv: +1 forward (input row = out row + kh - 1), -1 data-grad
  const float* scale_a;
  const float* scale_b;
  const __nv_bfloat16* bias;  // [N], used by kEpiBias / kEpiBiasSilu
  int epilogue;
  int* err;
};

// EPI epilogue warps (4 or 8): with 8, two warps share each TMEM lane quarter and
// take alternate 64-column chunks, which doubles the rate at which accumulators
// are drained -- the limit of GEMMs with a short K (2-4 K blocks per tile), where
// a tile's epilogue takes longer than its MMAs.
template <int BM_SUB, int BN, int STAGES, int EPI = kEpiWarps>
struct KGemmConfig {
  static_assert(BM_SUB == 1 || BM_SUB == 2, "BM_SUB");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
  static_assert(EPI == 4 || EPI == 8, "EPI");
  static constexpr int kThreads = 64 + 32 * EPI;
  static constexpr int kBTileBytes = BN * kKBlockBytes;
  static constexpr int kStageBytes = BM_SUB * kATileBytes + kBTileBytes;
  static constexpr int kAccCols = BM_SUB * BN;            // TMEM columns per accumulator buffer
  static constexpr int kTmemCols = (2 * kAccCols <= 32) ? 32 : 2 * kAccCols;  // power of two here
  static constexpr int kEpiStageBytes = EPI * 2 * kEpiBufBytes;  // two staging buffers per epilogue warp
  static constexpr int kBiasBytes = EPI * 64 * 4;                // a chunk's bias as fp32, one copy per warp
  static constexpr int kBarBytes = 1024;
  static constexpr int kSmemBytes = STAGES * kStageBytes + kEpiStageBytes + kBiasBytes + kBarBytes + 1024;  // +1024 alignment
  static_assert(2 * kAccCols <= 512, "two accumulator buffers must fit in TMEM");
  static_assert(kSmemBytes <= 232448, "smem");
};

// The bias of the 64 output columns n0 .. n0 + 63 spread over lanes 0..7 (one
// 8-column vector each).  Loaded at the top of a chunk, before the accumulator
// is read, so the load latency overlaps the TMEM load instead of sitting in
// the store loop; bias_vec() hands vector j to every lane.
__device__ __forceinline__ uint4 load_bias_chunk(int epi, const __nv_bfloat16* bias, int n0, int n_total, int lane) {
  uint4 b = make_uint4(0u, 0u, 0u, 0u);
  if (epi != kEpiNone && lane < 8 && n0 + lane * 8 < n_total)
    b = __ldg(reinterpret_cast<const uint4*>(bias + n0 + lane * 8));
  return b;
}
__device__ __forceinline__ uint4 bias_vec(const uint4& chunk, int j) {
  return make_uint4(__shfl_sync(0xffffffffu, chunk.x, j), __shfl_sync(0xffffffffu, chunk.y, j),
                    __shfl_sync(0xffffffffu, chunk.z, j), __shfl_sync(0xffffffffu, chunk.w, j));
}

// 8 consecutive output columns of one row from fp32 accumulator bits: acc * scale, then
// + bias (8 fp32 from shared memory) and SiLU, as packed f32x2 operations (the same two
// roundings as the scalar form), bf16x8.
__device__ __forceinline__ uint4 epilogue8_f32bias(const uint32_t* acc, float2 scale2, int epi, const float* bias8) {
  float2 v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    v[i] = __fmul2_rn(make_float2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1])), scale2);
  if (epi != kEpiNone) {
    const float4 b0 = *reinterpret_cast<const float4*>(bias8);
    const float4 b1 = *reinterpret_cast<const float4*>(bias8 + 4);
    v[0] = __fadd2_rn(v[0], make_float2(b0.x, b0.y));
    v[1] = __fadd2_rn(v[1], make_float2(b0.z, b0.w));
    v[2] = __fadd2_rn(v[2], make_float2(b1.x, b1.y));
    v[3] = __fadd2_rn(v[3], make_float2(b1.z, b1.w));
    if (epi == kEpiBiasSilu) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = make_float2(silu_f32(v[i].x), silu_f32(v[i].y));
    }
  }
  return make_uint4(pack_bf16x2(v[0].x, v[0].y), pack_bf16x2(v[1].x, v[1].y), pack_bf16x2(v[2].x, v[2].y),
                    pack_bf16x2(v[3].x, v[3].y));
}

// 8 consecutive output columns of one row: scale, optional bias / SiLU, bf16x8.
__device__ __forceinline__ uint4 epilogue8(const uint32_t* acc, float scale, int epi, const uint4& b) {
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(acc[i]) * scale;
  if (epi != kEpiNone) {
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] += bf16_lo_f(bw[j]);
      v[2 * j + 1] += bf16_hi_f(bw[j]);
    }
    if (epi == kEpiBiasSilu) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = silu_f32(v[i]);
    }
  }
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

template <int BM_SUB, int BN, int STAGES, int EPI = kEpiWarps>
__global__ void __launch_bounds__(KGemmConfig<BM_SUB, BN, STAGES, EPI>::kThreads, 1)
    kgemm_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_out, const KGemmParams p) {
  using Cfg = KGemmConfig<BM_SUB, BN, STAGES, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + STAGES * Cfg::kStageBytes;
  float* bias_smem = reinterpret_cast<float*>(epi_smem + Cfg::kEpiStageBytes);
  uint8_t* bar_area = epi_smem + Cfg::kEpiStageBytes + Cfg::kBiasBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], EPI * 32);
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int mt = tile / p.num_n_tiles;
        const int nt = tile - mt * p.num_n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + BM_SUB * kATileBytes;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          if (p.a_conv) {
            const int tap = kb / p.cchunks;
            const int chunk = kb - tap * p.cchunks;
            const int kh = tap / 3, kw = tap - 3 * (tap / 3);
            const int dh = p.tap_sign * (kh - 1), dw = p.tap_sign * (kw - 1);
#pragma unroll
            for (int sub = 0; sub < BM_SUB; ++sub) {
              const int m0 = (mt * BM_SUB + sub) * kSubTileRows;
              const int img = m0 / p.HW;
              const int h0 = (m0 - img * p.HW) / p.W;
              tma_load_4d(sa + sub * kATileBytes, &tmap_a, &full_bar[stage], chunk * kKBlockBytes, dw, h0 + dh,
                          img);
            }
          } else {
#pragma unroll
            for (int sub = 0; sub < BM_SUB; ++sub) {
              tma_load_2d(sa + sub * kATileBytes, &tmap_a, &full_bar[stage], kb * kKBlockBytes,
                          (mt * BM_SUB + sub) * kSubTileRows);
            }
          }
          tma_load_2d(sb, &tmap_b, &full_bar[stage], kb * kKBlockBytes, nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the loads already in flight land before the CTA can exit.
        const int64_t first = issued > STAGES ? issued - STAGES : 0;
        volatile int never = 0;
        for (int64_t i = first; i < issued; ++i)
          mbar_wait(&full_bar[i % STAGES], uint32_t((i / STAGES) & 1), &never, p.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_e4m3(kSubTileRows, BN, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + BM_SUB * kATileBytes;
#pragma unroll
          for (int sub = 0; sub < BM_SUB; ++sub) {
#pragma unroll
            for (int k = 0; k < kKBlockBytes / 32; ++k) {
              const uint64_t adesc = make_smem_desc(sa + sub * kATileBytes + k * 32, 16, 1024);
              const uint64_t bdesc = make_smem_desc(sb + k * 32, 16, 1024);
              umma_f8(d_tmem + sub * BN, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      // Drain: wait until every MMA issued by this thread has retired.
      umma_commit(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w may read TMEM lanes [32 (w % 4), +32); with 8 epilogue warps the two warps
    // of a lane quarter (w - 2 < 4 and w - 2 >= 4) take alternate 64-column chunks.
    const int quarter = warp & 3;
    constexpr int kPerQuarter = EPI / 4;
    const int part = (warp - 2) / 4;
    uint8_t* stage_buf = epi_smem + (warp - 2) * 2 * kEpiBufBytes;
    float* bias_w = bias_smem + (warp - 2) * 64;  // this warp's fp32 copy of the chunk's bias
    const float scale = __ldg(p.scale_a) * __ldg(p.scale_b);
    const float2 scale2 = make_float2(scale, scale);
    constexpr int kChunks = BM_SUB * (BN / 64);  // 64-column chunks per tile: ch = sub * (BN / 64) + c / 64
    // every epilogue warp reads (and releases) at least one chunk of every tile, so that each
    // accumulator use gets exactly EPI * 32 arrivals on its tempty barrier
    static_assert(kChunks >= kPerQuarter, "fewer 64-column chunks than epilogue warps per lane quarter");
    // Lane l's two bias values (columns 2l, 2l + 1) of chunk ch of tile t.  Each chunk's pair is
    // loaded one chunk ahead (the first chunk of a tile at the end of the previous one), so the
    // load latency hides behind a chunk's work instead of stalling the warp.
    auto bias_pair = [&](int t, int ch) -> uint32_t {
      if (p.epilogue == kEpiNone || t >= p.num_tiles) return 0u;
      const int n = (t % p.num_n_tiles) * BN + (ch % (BN / 64)) * 64 + 2 * lane;
      return n < p.N ? __ldg(reinterpret_cast<const uint32_t*>(p.bias + n)) : 0u;
    };
    uint32_t bw_next = bias_pair(blockIdx.x, part);
    int local = 0;
    int buf = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      const int mt = tile / p.num_n_tiles;
      const int nt = tile - mt * p.num_n_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + acc * Cfg::kAccCols;
#pragma unroll 1
      for (int ch = part; ch < kChunks; ch += kPerQuarter) {
        const int sub = ch / (BN / 64), c = (ch % (BN / 64)) * 64;
        const int m0 = (mt * BM_SUB + sub) * kSubTileRows + quarter * 32;
        const int n0 = nt * BN + c;
        const uint32_t bw = bw_next;
        bw_next = ch + kPerQuarter < kChunks ? bias_pair(tile, ch + kPerQuarter) : bias_pair(tile + gridDim.x, part);
        uint32_t r[64];
        tmem_ld_32x32b_x32(tbase + ch * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld_32x32b_x32(tbase + ch * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (ch + kPerQuarter >= kChunks) {
          // this warp's last read of the accumulator: hand it back to the MMA warp
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);
        }
        if (p.epilogue != kEpiNone) {
          __syncwarp();  // every lane is done with the previous chunk's bias
          *reinterpret_cast<float2*>(bias_w + 2 * lane) = make_float2(bf16_lo_f(bw), bf16_hi_f(bw));
          __syncwarp();
        }
        if (n0 < p.N) {
          uint8_t* sbuf = stage_buf + buf * kEpiBufBytes;
          if (lane == 0) bulk_wait_group_read<1>();  // this buffer's previous store has read smem
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 o = epilogue8_f32bias(&r[8 * j], scale2, p.epilogue, bias_w + 8 * j);
            st_shared_v4(sbuf + swizzle128_offset(lane, j), o.x, o.y, o.z, o.w);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, sbuf, n0, m0);
            bulk_commit_group();
          }
          buf ^= 1;
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

}  // namespace fp8b

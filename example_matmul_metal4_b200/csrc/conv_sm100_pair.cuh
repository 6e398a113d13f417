// CTA-pair (cta_group::2) implicit-GEMM convolution for stride-1 convs whose
// activations and weights both load by TMA: one cluster of two CTAs computes
// 256 consecutive output pixels x BN output channels with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA stages its own 128 pixels
// (one TMA im2col box per filter tap and 64-channel slab) and half of the
// weight columns, so the shared-memory bytes read per MMA flop drop by a
// third against the one-CTA kernel; with BN = 128 (Cout = 128) the one-CTA
// kernel's N = 128 instructions are bound by shared-memory reads.
//
// Tap rows (TAPROW): for dilation-1 filters 2 or 3 taps wide, the tile walks
// virtual pixels of rows OW + KW - 1 wide, and one im2col box of
// 128 + KW - 1 pixels per (kd, kh, channel slab) feeds all KW taps: tap kw
// is the same box read from row kw on, so its MMA descriptors start kw
// 128-byte rows further. TMA writes the 128-byte swizzle by absolute
// shared-memory address and tcgen05 reads it the same way, so a start that
// is a whole number of rows into a 1024-byte-aligned box reads those rows
// unchanged. Activation bytes per MMA flop drop by a factor of KW; the KW - 1
// virtual columns per row are computed and not stored (3 % at W = 64).
//
// Roles as in the CTA-pair GEMM (gemm_sm100_pair.cuh): warp 0 of both CTAs
// issues TMA into its own ring with completion counted on the leader's full
// barrier, the leader's warp 1 issues the MMAs and commits to both CTAs,
// warps 2-5 of both CTAs run the shared epilogue on their 128 rows.
#pragma once

#include "conv_sm100.cuh"
#include "gemm_sm100_pair.cuh"

namespace mm4 {

// TAPROW: a stage holds one activation box of up to 130 pixels (136 rows
// reserved, a whole number of 1024-byte swizzle atoms) and the weights of up
// to CONV_ROW_MAX_KW taps.
constexpr int CONV_ROW_MAX_KW = 3;

template <int BN, bool TAPROW = false>
struct ConvPairCfg {
  static constexpr int A_ROWS = TAPROW ? GEMM_BM + 8 : GEMM_BM;
  static constexpr int A_BYTES = A_ROWS * GEMM_BK * 2;     // this CTA's pixels x 64 channels
  static constexpr int B_TAP_BYTES = (BN / 2) * GEMM_BK * 2;  // this CTA's half of one tap's weight columns
  static constexpr int B_BYTES = (TAPROW ? CONV_ROW_MAX_KW : 1) * B_TAP_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = TAPROW ? ((BN == 128) ? 5 : 3) : ((BN == 128) ? 8 : 6);
  static constexpr int TMEM_COLS = 2 * BN;                 // two accumulators
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 256 + 1024;
  static_assert(A_BYTES % 1024 == 0 && STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte swizzle alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

enum : int {
  SITE_CONVPAIR_PRODUCER_EMPTY = 70,
  SITE_CONVPAIR_PRODUCER_DRAIN = 71,
  SITE_CONVPAIR_MMA_TMEM_EMPTY = 72,
  SITE_CONVPAIR_MMA_FULL = 73,
  SITE_CONVPAIR_MMA_DRAIN = 74,
};

template <int BN, bool B_MN, bool TAPROW>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    conv_sm100_pair_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                           const GemmArgs args, const ConvGeom g) {
  using Cfg = ConvPairCfg<BN, TAPROW>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_f16_f32(2 * GEMM_BM, BN, false, B_MN);
  constexpr int HALF_N = BN / 2;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* drain = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_vote = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_last = s_vote + 4;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const Watchdog wd{args.status, args.timeout_ns};
  const int u0 = static_cast<int>(blockIdx.x >> 1);
  const int ustep = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one()) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      uint32_t fills = 0;
      bool ok = true;
      for (int u = u0; u < args.num_units && ok; u += ustep) {
        const GemmUnit w = gemm_decode_unit(args, u);
        // This CTA's 128 output pixels start at m0 (n, oz, oy, ox order; ox
        // runs over the virtual row width with TAPROW).
        const int m0 = w.mt * 2 * GEMM_BM + static_cast<int>(rank) * GEMM_BM;
        const int row_w = TAPROW ? args.rm_vw : g.OW;
        const int ox = m0 % row_w;
        const int r1 = m0 / row_w;
        const int oy = r1 % g.OH;
        const int r2 = r1 / g.OH;
        const int oz = r2 % g.OD;
        const int n = r2 / g.OD;
        const int n0 = w.nt * BN + static_cast<int>(rank) * HALF_N;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(fills % STAGES);
          const uint32_t ph = (fills / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, wd, SITE_CONVPAIR_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = ring + s * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          const uint32_t lbar = mapa_shared(smem_u32(&full[s]), 0);
          if constexpr (TAPROW) {
            // k-block kb = (kd, kh, slab): one box of 128 + KW - 1 pixels and
            // the weights of taps (kd, kh, 0 .. KW-1).
            if (rank == 0)
              mbar_arrive_expect_tx(&full[s], 2u * ((GEMM_BM + g.KW - 1) * GEMM_BK * 2 + g.KW * Cfg::B_TAP_BYTES));
            const int khd = kb / g.ncb;
            const int cb = kb - khd * g.ncb;
            const int kd = khd / g.KH;
            const int kh = khd - kd * g.KH;
            tma_load_5d_im2col_pair(&tmX, lbar, sA, cb * 64, ox - g.PL, oy - g.PT, oz - g.PF, n, 0,
                                    static_cast<uint16_t>(kh * g.DY), static_cast<uint16_t>(kd * g.DZ));
            for (int kw = 0; kw < g.KW; ++kw) {
              const int tap = khd * g.KW + kw;
              uint8_t* sBt = sB + kw * Cfg::B_TAP_BYTES;
              if (!B_MN) {
                tma_load_3d_pair(&tmW, lbar, sBt, cb * 64, tap, n0);
              } else {
#pragma unroll
                for (int j = 0; j < HALF_N / 64; ++j)
                  tma_load_3d_pair(&tmW, lbar, sBt + j * 8192, n0 + 64 * j, cb * 64, tap);
              }
            }
            ++fills;
            continue;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
          const int tap = kb / g.ncb;
          const int cb = kb - tap * g.ncb;
          const int kd = tap / (g.KH * g.KW);
          const int khw = tap - kd * (g.KH * g.KW);
          const int kh = khw / g.KW;
          const int kw = khw - kh * g.KW;
          tma_load_5d_im2col_pair(&tmX, lbar, sA, cb * 64, ox - g.PL, oy - g.PT, oz - g.PF, n,
                                  static_cast<uint16_t>(kw * g.DX), static_cast<uint16_t>(kh * g.DY),
                                  static_cast<uint16_t>(kd * g.DZ));
          if (!B_MN) {
            // [Cout][taps][Cin]: box 64(Cin) x 1(tap) x HALF_N(Cout)
            tma_load_3d_pair(&tmW, lbar, sB, cb * 64, tap, n0);
          } else {
            // [taps][Cin][Cout]: box 64(Cout) x 64(Cin) x 1(tap), HALF_N/64 boxes
#pragma unroll
            for (int j = 0; j < HALF_N / 64; ++j) tma_load_3d_pair(&tmW, lbar, sB + j * 8192, n0 + 64 * j, cb * 64, tap);
          }
          ++fills;
        }
      }
      if (rank == 0) {
        const uint32_t first = fills > STAGES ? fills - STAGES : 0u;
        for (uint32_t i = first; i < fills; ++i) {
          if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, wd, SITE_CONVPAIR_PRODUCER_DRAIN)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && elect_one()) {
      uint32_t consumed = 0;
      uint32_t tiles_done = 0;
      bool ok = true;
      for (int u = u0; u < args.num_units && ok; u += ustep) {
        const GemmUnit w = gemm_decode_unit(args, u);
        const uint32_t acc = tiles_done & 1u;
        const uint32_t aph = (tiles_done >> 1) & 1u;
        if (!mbar_wait_cluster(&tmem_empty[acc], aph ^ 1u, wd, SITE_CONVPAIR_MMA_TMEM_EMPTY)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(consumed % STAGES);
          const uint32_t ph = (consumed / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, wd, SITE_CONVPAIR_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(ring + s * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
          const int taps_here = TAPROW ? g.KW : 1;
          for (int kw = 0; kw < taps_here; ++kw) {
            // TAPROW: tap kw reads the box from pixel row kw on.
            const uint32_t a_tap = a_base + static_cast<uint32_t>(kw) * 128u;
            const uint32_t b_tap = b_base + static_cast<uint32_t>(kw) * Cfg::B_TAP_BYTES;
#pragma unroll
            for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
              const uint64_t adesc = sw128_desc(a_tap + kk * 32, 16, 1024);
              const uint64_t bdesc =
                  B_MN ? sw128_desc(b_tap + kk * 2048, 8192, 1024) : sw128_desc(b_tap + kk * 32, 16, 1024);
              umma_f16_ss_pair(d_tmem, adesc, bdesc, IDESC, (kb > w.kb0 || kw > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(&empty[s], 0x3);
          ++consumed;
        }
        if (!ok) break;
        umma_commit_pair(&tmem_full[acc], 0x3);
        ++tiles_done;
      }
      umma_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, wd, SITE_CONVPAIR_MMA_DRAIN);
    }
  } else {
    epilogue_role<BN, MODE_DIRECT_F16, true>(args, tmem_full, tmem_empty, tmem_base, s_vote, s_last, nullptr, wd,
                                             warp, lane, rank);
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mm4

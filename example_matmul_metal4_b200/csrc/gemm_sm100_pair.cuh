// 2-CTA (cta_group::2) variant of the GEMM: one cluster of two CTAs on two
// SMs computes a 256-row tile with tcgen05.mma.cta_group::2 (M = 256).
//
// Each CTA stages only its own 128 rows of A and its own half of the B
// columns, so the shared-memory fill per MMA flop is 2/3 of the one-CTA
// 128 x 256 tile: the L2 -> SM traffic, not the tensor core, bounds the
// one-CTA kernel at large sizes, and for split-K each SM streams 1/3 fewer
// bytes from HBM.
//
//   both CTAs, warp 0   TMA producer into its own ring. The completion of
//                       both CTAs' copies is counted on the LEADER's (rank 0)
//                       full barrier (.cta_group::2 loads); only the leader
//                       posts the expected byte count.
//   leader, warp 1      one thread issues the pair's MMAs (A from both CTAs'
//                       rows, B from both CTAs' column halves) and commits
//                       each stage / accumulator to the barriers at the same
//                       offset in BOTH CTAs (commit multicast, mask 0b11).
//   both, warps 2-5     epilogue of the CTA's own 128 rows (its TMEM half),
//                       then a remote arrive on the leader's tmem_empty.
// A cluster barrier after set-up and before TMEM release keeps each CTA's
// shared memory and TMEM alive while its partner may still use them.
// No load uses cluster multicast: every CTA fetches its own bytes.
#pragma once

#include "gemm_sm100.cuh"

namespace mm4 {

// BN: N of the pair tile (256, or 512 for split-K). Per CTA: B stage holds
// BN/2 columns, the accumulator is 128 x BN fp32 in TMEM.
template <int BN>
struct PairCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;      // 16 KB: this CTA's 128 rows
  static constexpr int B_BYTES = (BN / 2) * GEMM_BK * 2;     // this CTA's half of the columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 512) ? 4 : 6;
  static constexpr int ACC_BUFS = (BN == 512) ? 1 : 2;
  static constexpr int TMEM_COLS = ACC_BUFS * BN;
  static constexpr int N_HALVES = BN / 256;                  // MMA instructions (N = 256) per k-step
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_STAGE_BYTES + 256 + 1024;
};

enum : int {
  SITE_PAIR_PRODUCER_EMPTY = 60,
  SITE_PAIR_PRODUCER_DRAIN = 61,
  SITE_PAIR_MMA_TMEM_EMPTY = 62,
  SITE_PAIR_MMA_FULL = 63,
  SITE_PAIR_MMA_DRAIN = 64,
};

template <int BN, bool A_MN, bool B_MN, int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_sm100_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs args) {
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_f16_f32(2 * GEMM_BM, 256, A_MN, B_MN);
  constexpr uint32_t B_HH = 16384;  // bytes of this CTA's 128 columns of one N=256 instruction

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* ring = smem;
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + EPI_STAGE_BYTES);
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
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t fills = 0;
      bool ok = true;
      for (int u = u0; u < args.num_units && ok; u += ustep) {
        const GemmUnit w = gemm_decode_unit(args, u);
        const int row0 = w.mt * 2 * GEMM_BM + static_cast<int>(rank) * GEMM_BM;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(fills % STAGES);
          const uint32_t ph = (fills / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, wd, SITE_PAIR_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = ring + s * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          const uint32_t lbar = mapa_shared(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
          const int k0 = kb * GEMM_BK;
          if (!A_MN) {
            tma_load_2d_pair(&tmA, lbar, sA, k0, row0);
          } else {
            tma_load_2d_pair(&tmA, lbar, sA, row0, k0);
            tma_load_2d_pair(&tmA, lbar, sA + 8192, row0 + 64, k0);
          }
#pragma unroll
          for (int hh = 0; hh < Cfg::N_HALVES; ++hh) {
            const int n0 = w.nt * BN + hh * 256 + static_cast<int>(rank) * 128;
            if (!B_MN) {
              tma_load_2d_pair(&tmB, lbar, sB + hh * B_HH, k0, n0);
            } else {
              tma_load_2d_pair(&tmB, lbar, sB + hh * B_HH, n0, k0);
              tma_load_2d_pair(&tmB, lbar, sB + hh * B_HH + 8192, n0 + 64, k0);
            }
          }
          ++fills;
        }
      }
      // The leader sees both CTAs' copies complete on its own full barriers;
      // the peer's copies are covered by the leader's MMA drain + the final
      // cluster barrier.
      if (rank == 0) {
        const uint32_t first = fills > STAGES ? fills - STAGES : 0u;
        for (uint32_t i = first; i < fills; ++i) {
          if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, wd, SITE_PAIR_PRODUCER_DRAIN)) break;
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
        const uint32_t acc = tiles_done % Cfg::ACC_BUFS;
        const uint32_t aph = (tiles_done / Cfg::ACC_BUFS) & 1u;
        if (!mbar_wait_cluster(&tmem_empty[acc], aph ^ 1u, wd, SITE_PAIR_MMA_TMEM_EMPTY)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(consumed % STAGES);
          const uint32_t ph = (consumed / STAGES) & 1u;
          if (!mbar_wait(&full[s], ph, wd, SITE_PAIR_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(ring + s * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            const uint64_t adesc =
                A_MN ? sw128_desc(a_base + kk * 2048, 8192, 1024) : sw128_desc(a_base + kk * 32, 16, 1024);
#pragma unroll
            for (int hh = 0; hh < Cfg::N_HALVES; ++hh) {
              const uint32_t bb = b_base + hh * B_HH;
              const uint64_t bdesc =
                  B_MN ? sw128_desc(bb + kk * 2048, 8192, 1024) : sw128_desc(bb + kk * 32, 16, 1024);
              umma_f16_ss_pair(d_tmem + hh * 256, adesc, bdesc, IDESC, (kb > w.kb0 || kk > 0) ? 1u : 0u);
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
      mbar_wait(drain, 0, wd, SITE_PAIR_MMA_DRAIN);
    }
  } else {
    epilogue_role<BN, MODE, true>(args, tmem_full, tmem_empty, tmem_base, s_vote, s_last, epi_stage, wd, warp, lane,
                                  rank);
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mm4

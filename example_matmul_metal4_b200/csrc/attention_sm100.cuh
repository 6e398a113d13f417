// Flash-attention forward (non-causal) for sm_100a.
//
// Replaces the reference's generated `attention` kernel
// (Sources/attention/attention.swift:23-382): O = softmax(scale * Q K^T) V
// with an fp32 online softmax in base 2 (the log2(e)*scale factor folded into
// one multiply, as attention.swift:24 folds it into dotScale), fp16 P, fp32 O,
// and a final O * (1/l) epilogue (:354-379). The reference takes the head
// dimension as a parameter (attention.swift:398); this kernel is instantiated
// for head_dim 128 and 64.
//
// One CTA per (batch, head, 256 query rows) = two 128-row Q tiles that share
// every K_j / V_j tile staged in shared memory. 12 warps:
//   warp 0      TMA producer: Q0, Q1 once, then K_j / V_j (128 keys each) into
//               rings (128-byte-swizzled boxes of 64 columns x 128 rows).
//   warp 1      TMEM alloc (512 columns: S0 | S1 | O0 | O1); one elected lane
//               issues tcgen05.mma. S_i = Q_i K_j^T (M=128, both operands in
//               smem) is issued in two N = 64 halves; O_i += P_i V_j (M=128,
//               N=D, K=128) reads P_i from TMEM and V as an MN-major smem
//               operand. Per key tile: S_lo_0(j+1), PV_0(j), S_lo_1(j+1),
//               S_hi_0(j+1), PV_1(j), S_hi_1(j+1): while one tile's softmax
//               runs, the tensor core works on the other tile and on the
//               first half of this tile's next S.
//   warps 4-7   softmax of Q tile 0, warps 8-11 of Q tile 1: thread r owns
//               query row r (TMEM lane r). Per key tile it reads its S row
//               (tcgen05.ld), releases the S columns, forms P = 2^(s - m)
//               against the running max m while taking the new row max,
//               writes P as fp16 pairs into the upper half of its S row
//               (tcgen05.st), and only when the max grew by more than 8 in
//               the log2 domain (a factor of 256) rescales its O row in TMEM
//               and its running sum l and redoes P (lazy rescaling). At the
//               end it reads O, multiplies by 1/l and stores fp16.
// Keys past the sequence end are masked to -inf; query rows past the end are
// computed on zero-filled Q and not stored.
#pragma once

#include "mm4_ptx.cuh"

namespace mm4 {

struct AttnArgs {
  int batch, heads_q, heads_kv, R, C;  // R = query rows, C = key/value rows
  int layout;                           // 0: [B][H][S][D], 1: [B][S][H][D]
  float scale_log2;                     // scale * log2(e)
  __half* O;
  float* lse;                           // optional [B][Hq][R]: natural-log sum of exp(scale * S) per row
  int* status;
  unsigned long long timeout_ns;
};

constexpr int ATT_D = 128;
constexpr int ATT_BM = 128;                     // query rows per Q tile
constexpr int ATT_QTILES = 2;                   // Q tiles per CTA
constexpr int ATT_CTA_ROWS = ATT_BM * ATT_QTILES;
constexpr int ATT_BN = 128;                     // keys per tile
constexpr int ATT_THREADS = 384;
constexpr int ATT_TILE_BYTES = 128 * 128 * 2;   // 32 KB: one head-dim-128 Q, K_j or V_j tile
// Register split: warps 0-3 (producer, MMA, two idle) give registers to the
// two softmax warpgroups. 128 * ATT_REGS_LOW + 256 * ATT_REGS_HIGH must not
// exceed 384 * (registers per thread at launch); the launcher checks it.
constexpr int ATT_REGS_LOW = 96;
constexpr int ATT_REGS_HIGH = 200;
constexpr int ATT_REGS_NEEDED = (128 * ATT_REGS_LOW + 256 * ATT_REGS_HIGH + ATT_THREADS - 1) / ATT_THREADS;

enum : int {
  SITE_ATT_PRODUCER = 40,
  SITE_ATT_PRODUCER_DRAIN = 41,
  SITE_ATT_MMA_Q = 42,
  SITE_ATT_MMA_K = 43,
  SITE_ATT_MMA_P = 45,
  SITE_ATT_MMA_V = 46,
  SITE_ATT_MMA_DRAIN = 47,
  SITE_ATT_SOFTMAX_S = 48,
  SITE_ATT_SOFTMAX_O = 49,
  SITE_ATT_MMA_S = 50,
  SITE_ATT_MMA_PV = 51,
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, to take part of the exponentials off the MUFU unit.
// x = n + f with n = round(x) taken from the low mantissa bits of
// x + 1.5*2^23, |f| <= 1/2; 2^f from a cubic fitted for this kernel by
// iteratively reweighted least squares on [-1/2, 1/2] (max relative error
// 7.5e-5, below fp16's half-ulp 4.9e-4: P is stored as fp16); 2^n is added
// into the exponent field. x is clamped at -125 so the result stays a normal
// float (masked scores become ~2e-38). Two lanes at a time on the packed
// fp32x2 pipe.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const float2 t = fadd2(x, make_float2(kRound, kRound));
  const float2 n = fadd2(t, make_float2(-kRound, -kRound));
  const float2 f = fadd2(x, make_float2(-n.x, -n.y));
  float2 p = ffma2(make_float2(0.05517161f, 0.05517161f), f, make_float2(0.24261114f, 0.24261114f));
  p = ffma2(p, f, make_float2(0.69326103f, 0.69326103f));
  p = ffma2(p, f, make_float2(0.99992806f, 0.99992806f));
  // p + (n << 23) with n = bits(t) - bits(kRound), in unsigned arithmetic.
  const uint32_t bias = 0u - (__float_as_uint(kRound) << 23);
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23) + bias),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23) + bias));
}

// Of every 8 consecutive scores of a row, this many (an even number) take the
// FMA-pipe exponential and the rest the hardware ex2.
#ifndef ATT_EMU_PER8
#define ATT_EMU_PER8 2
#endif

// Per-head-dim constants of the forward kernel. A tile is 128 rows x D
// fp16, loaded as D/64 boxes of 64 columns (128-byte swizzle); TMEM holds
// S0 | S1 (128 columns each) then O0 | O1 (D columns each).
template <int D>
struct AttFwdCfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int BOXES = D / 64;
  static constexpr int K_STAGES = (D == 128) ? 3 : 4;
  static constexpr int V_STAGES = (D == 128) ? 2 : 4;
  static constexpr int SMEM_BYTES = (ATT_QTILES + K_STAGES + V_STAGES) * TILE_BYTES + 512 + 1024;
};

// Loads one 128-row tile of head dim D (D/64 boxes of 64 columns).
template <int D>
__device__ __forceinline__ void att_load_tile_d(const CUtensorMap* map, uint64_t* bar, uint8_t* dst, int layout,
                                                int row0, int head, int b) {
#pragma unroll
  for (int box = 0; box < D / 64; ++box) {
    if (layout == 0)  // dims {D, S, H, B}
      tma_load_4d(map, bar, dst + box * 16384, box * 64, row0, head, b);
    else  // dims {D, H, S, B}
      tma_load_4d(map, bar, dst + box * 16384, box * 64, head, row0, b);
  }
}

// Row maximum of 128 raw scores: four independent chains of three-input
// maxima (x[0..3] start them, 4..123 join eight at a time, 124..127 last).
__device__ __forceinline__ float att_row_max(const float (&x)[128]) {
  float pm[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
  for (int i = 4; i < 124; i += 8)
#pragma unroll
    for (int e = 0; e < 4; ++e) pm[e] = fmax3(pm[e], x[i + e], x[i + 4 + e]);
  return fmax3(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]), fmaxf(fmaxf(x[124], x[125]), fmaxf(x[126], x[127])));
}

// P = 2^(x * scale_log2 - m) for the 128 scores of this thread's row: one
// packed FFMA per pair, ATT_EMU_PER8 of every 8 exponentials on the FMA pipe
// and the rest on MUFU, packed partial sums. P is written as fp16 pairs into
// the 64 TMEM columns at tP (the upper half of the row's S columns), 16 at a
// time. Returns
// the row's partial sum of P.
__device__ __forceinline__ float att_exp_store(const float (&x)[128], float sl2, float m, uint32_t tP) {
  const float2 sc = make_float2(sl2, sl2);
  const float2 nm = make_float2(-m, -m);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int quarter = 0; quarter < 4; ++quarter) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = quarter * 32 + c * 8 + 2 * e;
        const float2 a = ffma2(make_float2(x[idx], x[idx + 1]), sc, nm);
        float2 pv;
        if (2 * e >= 8 - ATT_EMU_PER8) {
          pv = ex2_poly2(a);
        } else {
          pv.x = ex2_approx(a.x);
          pv.y = ex2_approx(a.y);
        }
        acc[e] = fadd2(acc[e], pv);
        pk[c * 4 + e] = pack_half2(pv.x, pv.y);
      }
    }
    tmem_st_32x32b_x16(tP + quarter * 16, pk);
  }
  const float2 s01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
  return s01.x + s01.y;
}

// Flash-attention forward, head dim D (64 or 128); see the file comment.
//
// TMEM per Q tile i: S_i in columns [128 i, 128 i + 128), O_i in
// [256 + D i, 256 + D (i + 1)). S_i(j) = Q_i K_j^T is issued as two N = 64
// halves: S_lo (keys 0-63 -> columns 0-63) and S_hi (keys 64-127 -> columns
// 64-127). The softmax writes P_i(j) as fp16 pairs into columns 64-127 (over
// S_hi), which O_i += P_i(j) V_j reads. So:
//   - S_lo_i(j+1) only needs the softmax to have loaded S_i(j) into registers
//     (s_read); it runs on the tensor core while the softmax computes P_i(j);
//   - S_hi_i(j+1) overwrites P_i(j): it is issued only after the commit of
//     O_i += P_i(j) V_j has completed (pv_done), which orders the read of P
//     before the overwrite through an mbarrier rather than through the
//     issue order of MMAs on different accumulators.
// Each softmax row takes its exponentials against the running max of the
// previous key tiles while the row max of the new tile is formed alongside
// them; only when the max grew by more than 8 (log2 domain) are O and l
// rescaled and the exponentials redone against the new max (lazy rescaling:
// the stale max cancels exactly in O / l).
template <int D>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  using Cfg = AttFwdCfg<D>;
  constexpr int KS = Cfg::K_STAGES;
  constexpr int VS = Cfg::V_STAGES;
  constexpr int TB = Cfg::TILE_BYTES;
  constexpr uint32_t IDESC_S = idesc_f16_f32(ATT_BM, ATT_BN, false, false);
  constexpr uint32_t IDESC_S_HALF = idesc_f16_f32(ATT_BM, ATT_BN / 2, false, false);
  constexpr uint32_t IDESC_O = idesc_f16_f32(ATT_BM, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;                                          // [2]
  uint8_t* sK = smem + ATT_QTILES * TB;                        // [KS]
  uint8_t* sV = sK + KS * TB;                                  // [VS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * TB);
  uint64_t* q_full = bars;                  // 2
  uint64_t* s_full = bars + 2;              // 2: S_i(j) complete in TMEM
  uint64_t* s_read = bars + 4;              // 2: the softmax holds S_i(j) in registers
  uint64_t* p_full = bars + 6;              // 2: P_i(j) in TMEM (and O_i rescaled)
  uint64_t* pv_done = bars + 8;             // 2: O_i += P_i(j) V_j complete
  uint64_t* o_full = bars + 10;             // 2: last O_i += P V complete
  uint64_t* drain = bars + 12;              // 1
  uint64_t* k_full = bars + 13;             // KS
  uint64_t* k_empty = k_full + KS;          // KS
  uint64_t* v_full = k_empty + KS;          // VS
  uint64_t* v_empty = v_full + VS;          // VS
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_empty + VS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (args.heads_q / args.heads_kv);
  const int nkv = (args.C + ATT_BN - 1) / ATT_BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_read[i], ATT_BM);
      mbar_init(&p_full[i], ATT_BM);
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    regs_dec<ATT_REGS_LOW>();
  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int row0 = blockIdx.x * ATT_CTA_ROWS;
      mbar_arrive_expect_tx(&q_full[0], TB);
      att_load_tile_d<D>(&tmQ, &q_full[0], sQ, args.layout, row0, h, b);
      int kj = 0, vj = 0;  // tiles issued
      for (int j = 0; j < nkv; ++j) {
        const int ks = j % KS;
        if (!mbar_wait(&k_empty[ks], ((j / KS) & 1) ^ 1, wd, SITE_ATT_PRODUCER)) break;
        mbar_arrive_expect_tx(&k_full[ks], TB);
        att_load_tile_d<D>(&tmK, &k_full[ks], sK + ks * TB, args.layout, j * ATT_BN, hk, b);
        kj = j + 1;
        if (j == 0) {
          mbar_arrive_expect_tx(&q_full[1], TB);
          att_load_tile_d<D>(&tmQ, &q_full[1], sQ + TB, args.layout, row0 + ATT_BM, h, b);
        }
        const int vs = j % VS;
        if (!mbar_wait(&v_empty[vs], ((j / VS) & 1) ^ 1, wd, SITE_ATT_PRODUCER)) break;
        mbar_arrive_expect_tx(&v_full[vs], TB);
        att_load_tile_d<D>(&tmV, &v_full[vs], sV + vs * TB, args.layout, j * ATT_BN, hk, b);
        vj = j + 1;
      }
      // Wait for the last copy into every buffer before leaving.
      mbar_wait(&q_full[0], 0, wd, SITE_ATT_PRODUCER_DRAIN);
      if (kj > 0) mbar_wait(&q_full[1], 0, wd, SITE_ATT_PRODUCER_DRAIN);
      for (int i = (kj > KS ? kj - KS : 0); i < kj; ++i)
        mbar_wait(&k_full[i % KS], (i / KS) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
      for (int i = (vj > VS ? vj - VS : 0); i < vj; ++i)
        mbar_wait(&v_full[i % VS], (i / VS) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      // Shared-memory descriptors of the tile bases; a descriptor's low 14
      // bits hold (address >> 4), so the k-step offsets inside a tile are
      // added to it directly (every address stays below 256 KB).
      const uint64_t q_desc0 = sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = sw128_desc(smem_u32(sK), 16, 1024);
      const uint64_t v_desc0 = sw128_desc(smem_u32(sV), 16384, 1024);
      // S_i = Q_i K^T of key stage ks: part 0 = keys 0-63 into columns 0-63,
      // part 1 = keys 64-127 into columns 64-127, part 2 = all 128 keys.
      auto issue_s = [&](int i, int ks, int part) {
        const uint64_t qd = q_desc0 + static_cast<uint32_t>(i * (TB >> 4));
        const uint64_t kd = k_desc0 + static_cast<uint32_t>((ks * TB + (part == 1 ? 8192 : 0)) >> 4);
        const uint32_t d_tmem = tmem_base + i * 128 + (part == 1 ? 64u : 0u);
        const uint32_t idesc = part == 2 ? IDESC_S : IDESC_S_HALF;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          umma_f16_ss(d_tmem, qd + off, kd + off, idesc, kk > 0 ? 1u : 0u);
        }
      };
      // O_i += P_i V: P_i is fp16 pairs in TMEM columns [128 i + 64, 128 i + 128).
      auto issue_pv = [&](int i, int vs, bool acc) {
        const uint64_t vd = v_desc0 + static_cast<uint32_t>((vs * TB) >> 4);
        const uint32_t d_tmem = tmem_base + 256 + i * D;
        const uint32_t p_tmem = tmem_base + i * 128 + 64;
#pragma unroll
        for (int kk = 0; kk < ATT_BN / 16; ++kk)
          umma_f16_ts(d_tmem, p_tmem + kk * 8, vd + static_cast<uint32_t>(kk * (2048 >> 4)), IDESC_O,
                      (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(&q_full[0], 0, wd, SITE_ATT_MMA_Q) && mbar_wait(&k_full[0], 0, wd, SITE_ATT_MMA_K);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0, 2);
        umma_commit(&s_full[0]);
        ok = mbar_wait(&q_full[1], 0, wd, SITE_ATT_MMA_Q);
      }
      if (ok) {
        tc_fence_after();
        issue_s(1, 0, 2);
        umma_commit(&s_full[1]);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int vs = j % VS;
        const bool more = j + 1 < nkv;
        const int ks = (j + 1) % KS;
        const uint32_t par = static_cast<uint32_t>(j & 1);
        // Tile 0: keys 0-63 of the next S while its softmax forms P_0(j).
        if (more) {
          if (!mbar_wait(&s_read[0], par, wd, SITE_ATT_MMA_S) ||
              !mbar_wait(&k_full[ks], ((j + 1) / KS) & 1, wd, SITE_ATT_MMA_K)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, ks, 0);
        }
        // Tile 0: O_0 += P_0(j) V_j.
        if (!mbar_wait(&p_full[0], par, wd, SITE_ATT_MMA_P) ||
            !mbar_wait(&v_full[vs], (j / VS) & 1, wd, SITE_ATT_MMA_V)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(0, vs, j > 0);
        umma_commit(more ? &pv_done[0] : &o_full[0]);
        // Tile 1: keys 0-63 of the next S.
        if (more) {
          if (!mbar_wait(&s_read[1], par, wd, SITE_ATT_MMA_S)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(1, ks, 0);
          // Tile 0: keys 64-127 of the next S, over P_0(j) once O_0 += P_0(j) V_j is done.
          if (!mbar_wait(&pv_done[0], par, wd, SITE_ATT_MMA_PV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, ks, 1);
          umma_commit(&s_full[0]);
        }
        // Tile 1: O_1 += P_1(j) V_j.
        if (!mbar_wait(&p_full[1], par, wd, SITE_ATT_MMA_P)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(1, vs, j > 0);
        umma_commit(&v_empty[vs]);
        umma_commit(more ? &pv_done[1] : &o_full[1]);
        if (more) {
          if (!mbar_wait(&pv_done[1], par, wd, SITE_ATT_MMA_PV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(1, ks, 1);
          umma_commit(&s_full[1]);
          umma_commit(&k_empty[ks]);
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATT_MMA_DRAIN);
    }
  }
  } else {
    // ---------------------------------------------------------- softmax
    regs_inc<ATT_REGS_HIGH>();
    const int ti = (warp - 4) >> 2;  // Q tile of this warpgroup
    const int q = warp & 3;          // TMEM lane quadrant
    const int r = q * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tS = tmem_base + ti * 128 + lane_off;
    const uint32_t tP = tS + 64;
    const uint32_t tO = tmem_base + 256 + ti * D + lane_off;
    const float sl2 = args.scale_log2;
    float m = -INFINITY;  // running max, log2 domain (possibly stale by < 8)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[ti], j & 1, wd, SITE_ATT_SOFTMAX_S));
      if (!ok) break;
      tc_fence_after();
      float x[128];
      {
        uint32_t v0[32], v1[32], v2[32], v3[32];
        tmem_ld_32x32b_x32(tS + 0, v0);
        tmem_ld_32x32b_x32(tS + 32, v1);
        tmem_ld_32x32b_x32(tS + 64, v2);
        tmem_ld_32x32b_x32(tS + 96, v3);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(v0[i]);
          x[32 + i] = __uint_as_float(v1[i]);
          x[64 + i] = __uint_as_float(v2[i]);
          x[96 + i] = __uint_as_float(v3[i]);
        }
      }
      // S_i(j) is in registers: its TMEM columns may take the next S_lo.
      tc_fence_before();
      mbar_arrive(&s_read[ti]);
      const int valid = args.C - j * ATT_BN;
      if (valid < ATT_BN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) x[i] = -INFINITY;
      }
      float part;
      if (j == 0) {
        m = att_row_max(x) * sl2;
        part = att_exp_store(x, sl2, m, tP);
      } else {
        // Exponentials against the running max, the new row max alongside.
        part = att_exp_store(x, sl2, m, tP);
        const float mx = att_row_max(x) * sl2;
        const bool grow = (mx > m + 8.0f);
        if (__any_sync(0xffffffffu, grow)) {
          // Rescale this warp's O rows in TMEM (lanes without growth use 1.0)
          // and redo the exponentials against the new max. The last
          // O_i += P_i(j-1) V has completed: the commit of S_i(j) covers it.
          const float m_new = grow ? mx : m;
          const float factor = grow ? ex2_approx(m - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(tO + c * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * factor);
            tmem_st_32x32b_x16(tO + c * 16, v);
          }
          l *= factor;
          m = m_new;
          tmem_st_wait();
          part = att_exp_store(x, sl2, m, tP);
        }
      }
      l += part;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[ti]);
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[ti], 0, wd, SITE_ATT_SOFTMAX_O));
      if (ok) {
        tc_fence_after();
        const int row = blockIdx.x * ATT_CTA_ROWS + ti * ATT_BM + r;
        const float inv_l = 1.0f / l;
        if (args.lse != nullptr && row < args.R) {
          // m and l share the same (possibly stale) max, so m + log2(l) is
          // the row's log2-sum-exp2 of scale*log2(e)*S; times ln 2 gives the
          // natural-log value (Network.swift createLTerm).
          args.lse[(static_cast<long long>(b) * args.heads_q + h) * args.R + row] =
              (m + log2f(l)) * 0.6931471805599453f;
        }
        __half* dst = nullptr;
        if (row < args.R) {
          const long long off = (args.layout == 0)
                                    ? ((static_cast<long long>(b) * args.heads_q + h) * args.R + row) * D
                                    : ((static_cast<long long>(b) * args.R + row) * args.heads_q + h) * D;
          dst = args.O + off;
        }
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tO + c * 32, v);
          tmem_ld_wait();
          if (dst) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 pk;
              pk.x = pack_half2(__uint_as_float(v[i]) * inv_l, __uint_as_float(v[i + 1]) * inv_l);
              pk.y = pack_half2(__uint_as_float(v[i + 2]) * inv_l, __uint_as_float(v[i + 3]) * inv_l);
              pk.z = pack_half2(__uint_as_float(v[i + 4]) * inv_l, __uint_as_float(v[i + 5]) * inv_l);
              pk.w = pack_half2(__uint_as_float(v[i + 6]) * inv_l, __uint_as_float(v[i + 7]) * inv_l);
              *reinterpret_cast<uint4*>(dst + c * 32 + i) = pk;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace mm4

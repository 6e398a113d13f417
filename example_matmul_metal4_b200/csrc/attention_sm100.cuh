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
// every K_j / V_j tile staged in shared memory. Keys are walked in steps of
// 64 (half a staged tile). 12 warps:
//   warp 0      TMA producer: Q0, Q1 once, then K_j / V_j (128 keys each) into
//               rings (128-byte-swizzled boxes of 64 columns x 128 rows).
//   warp 1      TMEM alloc (512 columns: two 64-column S slots per Q tile,
//               then O0 | O1).
//   warps 1, 2  one elected lane each issues tcgen05.mma: at D = 128 warp 1
//               every S and warp 2 every P.V, at D = 64 one warp per Q tile.
//               S_i(n) = Q_i K(n)^T (M=128, N=64, both operands in smem) goes
//               to slot n % 2 of tile i; O_i += P_i(n) V(n) (M=128, N=D,
//               K=64) reads P_i(n) from TMEM and V as an MN-major smem
//               operand. S_i(n+2) follows PV_i(n): S runs two steps ahead of
//               the softmax.
//   warps 4-7   softmax of Q tile 0, warps 8-11 of Q tile 1: thread r owns
//               query row r (TMEM lane r). Per step it reads its 64 scores
//               (tcgen05.ld), forms P = 2^(s - m) against the running max m
//               while taking the new row max, writes P as fp16 pairs over the
//               first half of the step's slot (tcgen05.st), and only when the
//               max grew by more than 8 in the log2 domain (a factor of 256)
//               rescales its O row in TMEM and its running sum l and redoes P
//               (lazy rescaling). At the end it reads O, multiplies by 1/l and
//               stores fp16.
// Keys past the sequence end are masked to -inf; query rows past the end are
// computed on zero-filled Q and not stored.
#pragma once

#include "mm4_ptx.cuh"

namespace mm4 {

struct AttnArgs {
  int batch, heads_q, heads_kv, R, C;  // R = query rows, C = key/value rows
  int layout;                           // 0: [B][H][S][D], 1: [B][S][H][D]
  int q_blocks;                         // 256-row query blocks per (batch, head)
  int num_units;                        // batch * heads_q * q_blocks
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
constexpr int ATT_BN = 128;                     // keys per staged K / V tile
constexpr int ATT_SN = 64;                      // keys per softmax step (half a staged tile)
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
  SITE_ATT_MMA_O = 52,
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
  // Exponentials per 8 on the FMA pipe. At D = 128 the tensor work per key
  // step leaves the softmax slack, and the MUFU-only loop (fewer
  // instructions) is faster; at D = 64 the softmax bounds the step and
  // moving 2 of 8 off MUFU pays (B4 H16 S4096 on one B200: D = 128 0.449 ms
  // with 0, 0.464 with 2; D = 64 0.360 ms with 2, 0.374 with 0).
  static constexpr int EMU_PER8 = (D == 128) ? 0 : 2;
  // How the two MMA-issuing warps share the work. D = 128: warp 1 issues
  // every S MMA and warp 2 every P.V MMA, so a P.V is never queued behind
  // the issue of the other kind (0.441 ms against 0.452 ms per Q tile). D = 64:
  // one warp per Q tile (0.360 ms against 0.363).
  static constexpr bool ISSUE_BY_KIND = (D == 128);
};

// Prefetches one 128-row tile of head dim D into L2 (see att_load_tile_d).
template <int D>
__device__ __forceinline__ void att_prefetch_tile_d(const CUtensorMap* map, int layout, int row0, int head, int b) {
#pragma unroll
  for (int box = 0; box < D / 64; ++box) {
    if (layout == 0)
      tma_prefetch_l2_4d(map, box * 64, row0, head, b);
    else
      tma_prefetch_l2_4d(map, box * 64, head, row0, b);
  }
}

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

// Row maximum of the 64 raw scores of one key step: four independent chains
// of three-input maxima (x[0..3] start them, 4..59 join eight at a time,
// 60..63 last).
__device__ __forceinline__ float att_row_max64(const float (&x)[64]) {
  float pm[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
  for (int i = 4; i < 60; i += 8)
#pragma unroll
    for (int e = 0; e < 4; ++e) pm[e] = fmax3(pm[e], x[i + e], x[i + 4 + e]);
  return fmax3(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]), fmaxf(fmaxf(x[60], x[61]), fmaxf(x[62], x[63])));
}

// P = 2^(x * scale_log2 - m) for the 64 scores of this thread's row in one
// key step: one packed FFMA per pair, EMU of every 8 exponentials on the FMA
// pipe and the rest on MUFU, packed partial sums. P is written as fp16 pairs
// into the 32 TMEM columns at tP, 16 at a time. Returns the row's partial sum
// of P.
template <int EMU>
__device__ __forceinline__ float att_exp_store64(const float (&x)[64], float sl2, float m, uint32_t tP) {
  const float2 sc = make_float2(sl2, sl2);
  const float2 nm = make_float2(-m, -m);
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = half * 32 + c * 8 + 2 * e;
        const float2 a = ffma2(make_float2(x[idx], x[idx + 1]), sc, nm);
        float2 pv;
        if (2 * e >= 8 - EMU) {
          pv = ex2_poly2(a);
        } else {
          pv.x = ex2_approx(a.x);
          pv.y = ex2_approx(a.y);
        }
        acc[e] = fadd2(acc[e], pv);
        pk[c * 4 + e] = pack_half2(pv.x, pv.y);
      }
    }
    tmem_st_32x32b_x16(tP + half * 16, pk);
  }
  const float2 s01 = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
  return s01.x + s01.y;
}

// Flash-attention forward, head dim D (64 or 128); see the file comment.
//
// Persistent: CTA c takes the units (batch, head, 256 query rows) c, c + G,
// c + 2G, ... (G = gridDim.x), and every role walks them in order, so the
// next unit's Q / K / V loads and first S MMAs overlap the current unit's
// last steps and epilogue. Steps are counted across units (g), which fixes
// the TMEM slot (g % 2) and the mbarrier phases of every per-step barrier.
//
// Keys are walked in steps of 64 (half a staged K_j / V_j tile). TMEM per Q
// tile i: two 64-column slots, [128 i, 128 i + 64) and [128 i + 64,
// 128 i + 128); S_i(g) = Q_i K(g)^T goes to slot g % 2, and the softmax
// writes P_i(g) as fp16 pairs over the first 32 columns of the same slot.
// O_i is in [256 + D i, 256 + D (i + 1)). The MMA issuer keeps S two steps
// ahead: S_i(g + 2) reuses slot g % 2 and is issued once the commit of
// O_i += P_i(g) V(g) has completed (pv_done), so the read of P_i(g) is
// ordered before the overwrite through an mbarrier, not through the issue
// order of MMAs on different accumulators. The softmax of step g + 1 then
// finds S_i(g + 1) ready and never waits for its own P.V. The first P.V of
// a unit overwrites O_i only after the softmax has read the previous unit's
// O_i (o_empty); a unit's Q_i is replaced only after its last S_i (q_empty).
//
// Each softmax row takes its exponentials against the running max of the
// previous steps while the row max of the new step is formed alongside them;
// only when the max grew by more than 8 (log2 domain) are O and l rescaled
// and the exponentials redone against the new max (lazy rescaling: the stale
// max cancels exactly in O / l). The rescale first waits for the previous
// step's P.V (pv_done), the only MMA that can still be writing O_i.
template <int D>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  using Cfg = AttFwdCfg<D>;
  constexpr int KS = Cfg::K_STAGES;
  constexpr int VS = Cfg::V_STAGES;
  constexpr int TB = Cfg::TILE_BYTES;
  constexpr uint32_t IDESC_S = idesc_f16_f32(ATT_BM, ATT_SN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16_f32(ATT_BM, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;                                          // [2]
  uint8_t* sK = smem + ATT_QTILES * TB;                        // [KS]
  uint8_t* sV = sK + KS * TB;                                  // [VS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * TB);
  uint64_t* q_full = bars;                  // [tile]: Q_i of the unit landed
  uint64_t* q_empty = bars + 2;             // [tile]: the unit's last S_i complete
  uint64_t* s_full = bars + 4;              // [tile][slot]: S_i(g) complete in TMEM
  uint64_t* p_full = bars + 8;              // [tile][slot]: P_i(g) in TMEM (and O_i rescaled)
  uint64_t* pv_done = bars + 12;            // [tile][slot]: O_i += P_i(g) V(g) complete
  uint64_t* o_full = bars + 16;             // [tile]: the unit's last O_i += P V complete
  uint64_t* o_empty = bars + 18;            // [tile]: the softmax holds the unit's O_i in registers
  uint64_t* drain = bars + 20;              // 1
  uint64_t* k_full = bars + 21;             // KS
  uint64_t* k_empty = k_full + KS;          // KS
  uint64_t* v_full = k_empty + KS;          // VS
  uint64_t* v_empty = v_full + VS;          // VS
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_empty + VS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};
  const int nkv = (args.C + ATT_BN - 1) / ATT_BN;   // staged K / V tiles per unit
  const int nst = (args.C + ATT_SN - 1) / ATT_SN;   // key steps per unit
  const int units = (args.num_units - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                    static_cast<int>(gridDim.x);     // units of this CTA
  const int total = units * nst;                    // key steps of this CTA
  // (query block, head, batch) of this CTA's unit ul
  auto unit_of = [&](int ul, int& qb, int& h, int& b) {
    const int u = static_cast<int>(blockIdx.x) + ul * static_cast<int>(gridDim.x);
    qb = u % args.q_blocks;
    const int bh = u / args.q_blocks;
    h = bh % args.heads_q;
    b = bh / args.heads_q;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], ATT_BM);
      for (int sl = 0; sl < 2; ++sl) {
        mbar_init(&s_full[2 * i + sl], 1);
        mbar_init(&p_full[2 * i + sl], ATT_BM);
        mbar_init(&pv_done[2 * i + sl], 1);
      }
    }
    mbar_init(drain, 2);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], Cfg::ISSUE_BY_KIND ? 1 : 2);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], Cfg::ISSUE_BY_KIND ? 1 : 2);
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
      int nq[2] = {0, 0};  // Q loads issued per tile
      int kt = 0, vt = 0;  // K / V tiles issued (ring positions)
      bool ok = true;
      for (int ul = 0; ul < units && ok; ++ul) {
        int qb, h, b;
        unit_of(ul, qb, h, b);
        const int hk = h / (args.heads_q / args.heads_kv);
        const int row0 = qb * ATT_CTA_ROWS;
        for (int j = 0; j < nkv && ok; ++j) {
          // Halfway through a unit, bring the next unit's Q tiles and first
          // K / V tiles into L2: their loads into shared memory can only
          // start when this unit's last S MMAs free the buffers, and would
          // otherwise wait the DRAM latency at the unit boundary.
          if (j == nkv / 2 && ul + 1 < units) {
            int nqb, nh, nb;
            unit_of(ul + 1, nqb, nh, nb);
            const int nhk = nh / (args.heads_q / args.heads_kv);
            att_prefetch_tile_d<D>(&tmQ, args.layout, nqb * ATT_CTA_ROWS, nh, nb);
            att_prefetch_tile_d<D>(&tmQ, args.layout, nqb * ATT_CTA_ROWS + ATT_BM, nh, nb);
            att_prefetch_tile_d<D>(&tmK, args.layout, 0, nhk, nb);
            att_prefetch_tile_d<D>(&tmV, args.layout, 0, nhk, nb);
          }
          // Q_0 before the unit's first K tile, Q_1 after it; each waits for
          // the previous unit's last S_i.
          for (int i = 0; i < 2 && j == 0; ++i) {
            if (i == 1) {
              const int ks = kt % KS;
              if (!(ok = mbar_wait(&k_empty[ks], ((kt / KS) & 1) ^ 1, wd, SITE_ATT_PRODUCER))) break;
              mbar_arrive_expect_tx(&k_full[ks], TB);
              att_load_tile_d<D>(&tmK, &k_full[ks], sK + ks * TB, args.layout, 0, hk, b);
              ++kt;
            }
            if (ul > 0 && !(ok = mbar_wait(&q_empty[i], (ul - 1) & 1, wd, SITE_ATT_PRODUCER))) break;
            mbar_arrive_expect_tx(&q_full[i], TB);
            att_load_tile_d<D>(&tmQ, &q_full[i], sQ + i * TB, args.layout, row0 + i * ATT_BM, h, b);
            ++nq[i];
          }
          if (!ok) break;
          if (j > 0) {
            const int ks = kt % KS;
            if (!(ok = mbar_wait(&k_empty[ks], ((kt / KS) & 1) ^ 1, wd, SITE_ATT_PRODUCER))) break;
            mbar_arrive_expect_tx(&k_full[ks], TB);
            att_load_tile_d<D>(&tmK, &k_full[ks], sK + ks * TB, args.layout, j * ATT_BN, hk, b);
            ++kt;
          }
          const int vs = vt % VS;
          if (!(ok = mbar_wait(&v_empty[vs], ((vt / VS) & 1) ^ 1, wd, SITE_ATT_PRODUCER))) break;
          mbar_arrive_expect_tx(&v_full[vs], TB);
          att_load_tile_d<D>(&tmV, &v_full[vs], sV + vs * TB, args.layout, j * ATT_BN, hk, b);
          ++vt;
        }
      }
      // Wait for the last copy into every buffer before leaving.
      for (int i = 0; i < 2; ++i)
        if (nq[i] > 0) mbar_wait(&q_full[i], (nq[i] - 1) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
      for (int t = (kt > KS ? kt - KS : 0); t < kt; ++t)
        mbar_wait(&k_full[t % KS], (t / KS) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
      for (int t = (vt > VS ? vt - VS : 0); t < vt; ++t)
        mbar_wait(&v_full[t % VS], (t / VS) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
    }
  } else if (warp == 1 || warp == 2) {
    // ---------------------------------------------------------- MMA issuers
    // Two issuing warps (Cfg::ISSUE_BY_KIND: all S / all P.V, else one per
    // Q tile): one thread issues about one tcgen05.mma per 55 SM clocks, so
    // a single issuer could not keep the tensor core fed with N = 64 S MMAs.
    if (elect_one()) {
      // Shared-memory descriptors of the tile bases; a descriptor's low 14
      // bits hold (address >> 4), so the offsets inside a tile are added to
      // it directly (every address stays below 256 KB).
      const uint64_t q_desc0 = sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t k_desc0 = sw128_desc(smem_u32(sK), 16, 1024);
      const uint64_t v_desc0 = sw128_desc(smem_u32(sV), 16384, 1024);
      // The last step of a unit that reads a staged K / V tile.
      auto last_step_of_tile = [&](int n) { return (n & 1) == 1 || n == nst - 1; };
      // Position of a key step: g counts steps across units, n within unit
      // ul; t is the staged K / V tile (ring position) the step reads. Kept
      // incrementally: the issuing thread's index arithmetic sits between
      // MMA groups.
      struct Pos {
        int g, ul, n, t;
      };
      auto advance = [&](Pos& p) {
        ++p.g;
        if (++p.n == nst) {
          p.n = 0;
          ++p.ul;
          p.t = p.ul * nkv;
        } else if ((p.n & 1) == 0) {
          ++p.t;
        }
      };
      // S_i(g) = Q_i K(g)^T: the 64 keys of step n are rows 64 (n % 2) .. +64
      // of the unit's staged K tile n / 2 (8 KB into each 64-column box).
      // Waits for the unit's Q_i (first step), the K tile (first of its two
      // steps) and the slot (P.V of step g - 2).
      auto do_s = [&](int i, const Pos& p) -> bool {
        const int g = p.g, n = p.n, ks = p.t % KS;
        if (n == 0 && !mbar_wait(&q_full[i], p.ul & 1, wd, SITE_ATT_MMA_Q)) return false;
        if ((n & 1) == 0 && !mbar_wait(&k_full[ks], (p.t / KS) & 1, wd, SITE_ATT_MMA_K)) return false;
        if (g >= 2 && !mbar_wait(&pv_done[2 * i + (g & 1)], ((g - 2) >> 1) & 1, wd, SITE_ATT_MMA_PV)) return false;
        tc_fence_after();
        const uint64_t qd = q_desc0 + static_cast<uint32_t>(i * (TB >> 4));
        const uint64_t kd = k_desc0 + static_cast<uint32_t>((ks * TB + (n & 1) * 8192) >> 4);
        const uint32_t d_tmem = tmem_base + i * 128 + (g & 1) * ATT_SN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          umma_f16_ss(d_tmem, qd + off, kd + off, IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[2 * i + (g & 1)]);
        if (n == nst - 1) umma_commit(&q_empty[i]);
        if ((!Cfg::ISSUE_BY_KIND || i == 1) && last_step_of_tile(n)) umma_commit(&k_empty[ks]);
        return true;
      };
      // O_i += P_i(g) V(g): P_i(g) is fp16 pairs in the first 32 columns of
      // slot g % 2; V(g) is rows 64 (n % 2) .. +64 of the unit's staged V
      // tile n / 2. A unit's first P.V starts O_i afresh, once the softmax
      // has read the previous unit's O_i.
      auto do_pv = [&](int i, const Pos& p) -> bool {
        const int g = p.g, n = p.n, vs = p.t % VS;
        if (!mbar_wait(&p_full[2 * i + (g & 1)], (g >> 1) & 1, wd, SITE_ATT_MMA_P)) return false;
        if ((n & 1) == 0 && !mbar_wait(&v_full[vs], (p.t / VS) & 1, wd, SITE_ATT_MMA_V)) return false;
        if (n == 0 && p.ul > 0 && !mbar_wait(&o_empty[i], (p.ul - 1) & 1, wd, SITE_ATT_MMA_O)) return false;
        tc_fence_after();
        const uint64_t vd = v_desc0 + static_cast<uint32_t>((vs * TB + (n & 1) * 8192) >> 4);
        const uint32_t d_tmem = tmem_base + 256 + i * D;
        const uint32_t p_tmem = tmem_base + i * 128 + (g & 1) * ATT_SN;
#pragma unroll
        for (int kk = 0; kk < ATT_SN / 16; ++kk)
          umma_f16_ts(d_tmem, p_tmem + kk * 8, vd + static_cast<uint32_t>(kk * (2048 >> 4)), IDESC_O,
                      (n > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[2 * i + (g & 1)]);
        if (n == nst - 1) umma_commit(&o_full[i]);
        if ((!Cfg::ISSUE_BY_KIND || i == 1) && last_step_of_tile(n)) umma_commit(&v_empty[vs]);
        return true;
      };
      const Pos first{0, 0, 0, 0};
      Pos second = first;
      advance(second);
      bool ok = true;
      if constexpr (Cfg::ISSUE_BY_KIND) {
        // Warp 1: S_0(g), S_1(g) for every step, each into the slot its P.V
        // of step g - 2 frees. Warp 2: P.V_0(g), P.V_1(g) as the P arrive.
        if (warp == 1) {
          ok = do_s(0, first) && (total < 2 || do_s(0, second)) && do_s(1, first) &&
               (total < 2 || do_s(1, second));
          Pos sx = second;
          for (advance(sx); sx.g < total && ok; advance(sx)) ok = do_s(0, sx) && do_s(1, sx);
        } else {
          for (Pos pv = first; pv.g < total && ok; advance(pv)) ok = do_pv(0, pv) && do_pv(1, pv);
        }
      } else {
        // Per step g: this tile's P.V, then S_i(g + 2) into the slot that
        // P.V frees. While this issuer waits for the P.V to complete, the
        // other tile's issuer keeps the tensor core busy.
        const int i = warp - 1;
        ok = do_s(i, first) && (total < 2 || do_s(i, second));
        Pos pv = first, sx = second;
        advance(sx);
        for (; pv.g < total && ok; advance(pv), advance(sx)) {
          ok = do_pv(i, pv);
          if (ok && sx.g < total) ok = do_s(i, sx);
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
    const uint32_t tO = tmem_base + 256 + ti * D + lane_off;
    const float sl2 = args.scale_log2;
    bool ok = true;
    int g = 0;  // key steps done, across units
    for (int ul = 0; ul < units && ok; ++ul) {
      float m = -INFINITY;  // running max, log2 domain (possibly stale by < 8)
      float l = 0.f;
      for (int n = 0; n < nst; ++n, ++g) {
        const int sl = g & 1;
        const uint32_t tSl = tS + sl * ATT_SN;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[2 * ti + sl], (g >> 1) & 1, wd, SITE_ATT_SOFTMAX_S));
        if (!ok) break;
        tc_fence_after();
        float x[64];
        {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(tSl + 0, v0);
          tmem_ld_32x32b_x32(tSl + 32, v1);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            x[i] = __uint_as_float(v0[i]);
            x[32 + i] = __uint_as_float(v1[i]);
          }
        }
        const int valid = args.C - n * ATT_SN;
        if (valid < ATT_SN) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= valid) x[i] = -INFINITY;
        }
        float part;
        if (n == 0) {
          m = att_row_max64(x) * sl2;
          part = att_exp_store64<Cfg::EMU_PER8>(x, sl2, m, tSl);
        } else {
          // Exponentials against the running max, the new row max alongside.
          part = att_exp_store64<Cfg::EMU_PER8>(x, sl2, m, tSl);
          const float mx = att_row_max64(x) * sl2;
          const bool grow = (mx > m + 8.0f);
          if (__any_sync(0xffffffffu, grow)) {
            // Rescale this warp's O rows in TMEM (lanes without growth use
            // 1.0) and redo the exponentials against the new max, once the
            // previous step's O_i += P V (the only MMA that may still write
            // O_i) is done.
            ok = __all_sync(0xffffffffu,
                            mbar_wait(&pv_done[2 * ti + (sl ^ 1)], ((g - 1) >> 1) & 1, wd, SITE_ATT_SOFTMAX_O));
            if (!ok) break;
            tc_fence_after();
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
            part = att_exp_store64<Cfg::EMU_PER8>(x, sl2, m, tSl);
          }
        }
        l += part;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[2 * ti + sl]);
      }
      if (!ok) break;
      // Epilogue of the unit: O_i into registers (then its TMEM columns may
      // take the next unit's first P.V), times 1/l, fp16 stores.
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[ti], ul & 1, wd, SITE_ATT_SOFTMAX_O));
      if (!ok) break;
      tc_fence_after();
      uint32_t o[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t* oc = o + c * 32;
        tmem_ld_32x32b_x32(tO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(oc));
      }
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&o_empty[ti]);
      int qb, h, b;
      unit_of(ul, qb, h, b);
      const int row = qb * ATT_CTA_ROWS + ti * ATT_BM + r;
      const float inv_l = 1.0f / l;
      if (args.lse != nullptr && row < args.R) {
        // m and l share the same (possibly stale) max, so m + log2(l) is the
        // row's log2-sum-exp2 of scale*log2(e)*S; times ln 2 gives the
        // natural-log value (Network.swift createLTerm).
        args.lse[(static_cast<long long>(b) * args.heads_q + h) * args.R + row] =
            (m + log2f(l)) * 0.6931471805599453f;
      }
      if (row < args.R) {
        const long long off = (args.layout == 0)
                                  ? ((static_cast<long long>(b) * args.heads_q + h) * args.R + row) * D
                                  : ((static_cast<long long>(b) * args.R + row) * args.heads_q + h) * D;
        __half* dst = args.O + off;
#pragma unroll
        for (int i = 0; i < D; i += 8) {
          uint4 pk;
          pk.x = pack_half2(__uint_as_float(o[i]) * inv_l, __uint_as_float(o[i + 1]) * inv_l);
          pk.y = pack_half2(__uint_as_float(o[i + 2]) * inv_l, __uint_as_float(o[i + 3]) * inv_l);
          pk.z = pack_half2(__uint_as_float(o[i + 4]) * inv_l, __uint_as_float(o[i + 5]) * inv_l);
          pk.w = pack_half2(__uint_as_float(o[i + 6]) * inv_l, __uint_as_float(o[i + 7]) * inv_l);
          *reinterpret_cast<uint4*>(dst + i) = pk;
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

// Flash-attention forward (non-causal) for sm_100a.
//
// Replaces the reference's generated `attention` kernel
// (Sources/attention/attention.swift:23-382): O = softmax(scale * Q K^T) V
// with an fp32 online softmax in base 2 (the log2(e)*scale factor folded into
// one multiply, as attention.swift:24 folds it into dotScale), fp16 P, fp32 O,
// and a final O * (1/l) epilogue (:354-379).
//
// One CTA per (batch, head, 128-row query tile); head_dim D = 128. 8 warps:
//   warp 0     TMA producer: Q once, then K_j / V_j (128 keys each) into
//              two-stage rings (128-byte-swizzled boxes of 64 x 128).
//   warp 1     TMEM alloc; one elected lane issues tcgen05.mma:
//                S_j = Q K_j^T  (M=128, N=128, K=D) into TMEM S[j%2]
//                O  += P_j V_j  (M=128, N=D,  K=128; V is an MN-major operand)
//              issuing S_{j+1} before O += P_j V_j so QK^T of the next tile
//              overlaps the softmax of the current one.
//   warps 4-7  softmax: thread r owns query row r (TMEM lane r). Per tile it
//              reads its S row (tcgen05.ld), takes the row max in the log2
//              domain, and only when the max grew by more than 8 (a factor of
//              256) rescales its O row in TMEM and its running sum l (lazy
//              rescaling: the stale max cancels in O / l exactly). It then
//              writes P = 2^(s - m) as fp16 into one of two swizzled smem P
//              tiles for the P V MMA; with two P buffers the softmax of tile
//              j+1 waits for P_j V_j only when it has to rescale O.
//              At the end it reads O, multiplies by 1/l and stores fp16.
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
  int* status;
  unsigned long long timeout_ns;
};

constexpr int ATT_D = 128;
constexpr int ATT_BM = 128;  // query rows per CTA
constexpr int ATT_BN = 128;  // keys per tile
constexpr int ATT_THREADS = 256;
constexpr int ATT_TILE_BYTES = 128 * 128 * 2;  // 32 KB: Q, K_j, V_j or P tile
constexpr int ATT_SMEM_BYTES = 7 * ATT_TILE_BYTES + 256 + 1024;  // Q, K[2], V[2], P[2]

enum : int {
  SITE_ATT_PRODUCER = 40,
  SITE_ATT_PRODUCER_DRAIN = 41,
  SITE_ATT_MMA_Q = 42,
  SITE_ATT_MMA_K = 43,
  SITE_ATT_MMA_SFREE = 44,
  SITE_ATT_MMA_P = 45,
  SITE_ATT_MMA_V = 46,
  SITE_ATT_MMA_DRAIN = 47,
  SITE_ATT_SOFTMAX_S = 48,
  SITE_ATT_SOFTMAX_PV = 49,
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
// float (masked scores become ~2e-38).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float kRound = 12582912.0f;  // 1.5 * 2^23
  const float t = x + kRound;
  const float n = t - kRound;
  const float f = x - n;
  const float p = fmaf(fmaf(fmaf(0.05517161f, f, 0.24261114f), f, 0.69326103f), f, 0.99992806f);
  const int ni = __float_as_int(t) - __float_as_int(kRound);
  return __int_as_float(__float_as_int(p) + (ni << 23));
}

// Of every 8 consecutive scores of a row, this many take ex2_poly and the rest
// the hardware ex2.
#ifndef ATT_EMU_PER8
#define ATT_EMU_PER8 2
#endif

// Loads one 128-row x 128-D tile as two 64-wide boxes (D 0..63, 64..127).
__device__ __forceinline__ void att_load_tile(const CUtensorMap* map, uint64_t* bar, uint8_t* dst, int layout,
                                              int row0, int head, int b) {
  if (layout == 0) {  // dims {D, S, H, B}
    tma_load_4d(map, bar, dst, 0, row0, head, b);
    tma_load_4d(map, bar, dst + 16384, 64, row0, head, b);
  } else {  // dims {D, H, S, B}
    tma_load_4d(map, bar, dst, 0, head, row0, b);
    tma_load_4d(map, bar, dst + 16384, 64, head, row0, b);
  }
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    attention_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  constexpr uint32_t IDESC_S = idesc_f16_f32(ATT_BM, ATT_BN, false, false);
  constexpr uint32_t IDESC_O = idesc_f16_f32(ATT_BM, ATT_D, false, true);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + ATT_TILE_BYTES;       // [2]
  uint8_t* sV = smem + 3 * ATT_TILE_BYTES;   // [2]
  uint8_t* sP = smem + 5 * ATT_TILE_BYTES;   // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * ATT_TILE_BYTES);
  uint64_t* q_full = bars;          // 1
  uint64_t* k_full = bars + 1;      // 2
  uint64_t* k_empty = bars + 3;     // 2
  uint64_t* v_full = bars + 5;      // 2
  uint64_t* v_empty = bars + 7;     // 2
  uint64_t* s_full = bars + 9;      // 2
  uint64_t* s_free = bars + 11;     // 2
  uint64_t* p_full = bars + 13;     // 1: P_j written (and O rescaled)
  uint64_t* pv_done = bars + 14;    // 2: P_j V_j finished, per P buffer j%2
  uint64_t* drain = bars + 16;      // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (args.heads_q / args.heads_kv);
  const int nkv = (args.C + ATT_BN - 1) / ATT_BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(drain, 1);
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
  const uint32_t tmem_O = tmem_base + 256;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, ATT_TILE_BYTES);
      att_load_tile(&tmQ, q_full, sQ, args.layout, qt * ATT_BM, h, b);
      int j = 0;
      for (; j < nkv; ++j) {
        const int s = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], ph, wd, SITE_ATT_PRODUCER)) break;
        mbar_arrive_expect_tx(&k_full[s], ATT_TILE_BYTES);
        att_load_tile(&tmK, &k_full[s], sK + s * ATT_TILE_BYTES, args.layout, j * ATT_BN, hk, b);
        if (!mbar_wait(&v_empty[s], ph, wd, SITE_ATT_PRODUCER)) {
          ++j;  // K_j is in flight: drain it below
          break;
        }
        mbar_arrive_expect_tx(&v_full[s], ATT_TILE_BYTES);
        att_load_tile(&tmV, &v_full[s], sV + s * ATT_TILE_BYTES, args.layout, j * ATT_BN, hk, b);
      }
      // Wait for the last copies of every buffer before leaving.
      mbar_wait(q_full, 0, wd, SITE_ATT_PRODUCER_DRAIN);
      for (int i = (j > 2 ? j - 2 : 0); i < j; ++i) {
        mbar_wait(&k_full[i & 1], (i >> 1) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
        mbar_wait(&v_full[i & 1], (i >> 1) & 1, wd, SITE_ATT_PRODUCER_DRAIN);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      bool ok = mbar_wait(q_full, 0, wd, SITE_ATT_MMA_Q);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      for (int j = 0; j <= nkv && ok; ++j) {
        if (j < nkv) {
          const int s = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&k_full[s], ph, wd, SITE_ATT_MMA_K)) break;
          if (!mbar_wait(&s_free[s], ph ^ 1, wd, SITE_ATT_MMA_SFREE)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + s * ATT_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < ATT_D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16_ss(tmem_base + s * 128, sw128_desc(q_addr + off, 16, 1024), sw128_desc(k_addr + off, 16, 1024),
                        IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(&k_empty[s]);
          umma_commit(&s_full[s]);
        }
        if (j >= 1) {
          const int jp = j - 1;
          const int s = jp & 1;
          if (!mbar_wait(p_full, jp & 1, wd, SITE_ATT_MMA_P)) break;
          if (!mbar_wait(&v_full[s], (jp >> 1) & 1, wd, SITE_ATT_MMA_V)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + s * ATT_TILE_BYTES);
          const uint32_t pb_addr = p_addr + (jp & 1) * ATT_TILE_BYTES;
#pragma unroll
          for (int kk = 0; kk < ATT_BN / 16; ++kk) {
            const uint64_t adesc = sw128_desc(pb_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(v_addr + kk * 2048, 16384, 1024);
            umma_f16_ss(tmem_O, adesc, bdesc, IDESC_O, (jp > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&v_empty[s]);
          umma_commit(&pv_done[jp & 1]);
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATT_MMA_DRAIN);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- softmax
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t p_row0 = smem_u32(sP) + r * 128;
    float m = -INFINITY;  // running max, log2 domain (possibly stale by < 8)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], (j >> 1) & 1, wd, SITE_ATT_SOFTMAX_S));
      if (!ok) break;
      tc_fence_after();
      float x[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_base + s * 128 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(v[i]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const int valid = args.C - j * ATT_BN;
      if (valid < ATT_BN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= valid) x[i] = -INFINITY;
      }
      // Row max of the raw scores (scale > 0 commutes with max), eight
      // independent partial maxima so the comparisons pipeline.
      float pm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pm[e] = x[e];
#pragma unroll
      for (int i = 8; i < 128; i += 8)
#pragma unroll
        for (int e = 0; e < 8; ++e) pm[e] = fmaxf(pm[e], x[i + e]);
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) *
                       args.scale_log2;

      const bool grow = (mx > m + 8.0f);
      const float m_new = grow ? mx : m;
      const float factor = grow ? ex2_approx(m - m_new) : 1.0f;
      const bool warp_rescale = j > 0 && __any_sync(0xffffffffu, grow);
      // O may be rescaled only once P_{j-1} V_{j-1} has finished.
      if (warp_rescale) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, wd, SITE_ATT_SOFTMAX_PV));
        if (!ok) break;
        tc_fence_after();
      }
      // P buffer j%2 was last read by P_{j-2} V_{j-2}.
      if (j >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[j & 1], ((j - 2) >> 1) & 1, wd, SITE_ATT_SOFTMAX_PV));
        if (!ok) break;
      }
      if (warp_rescale) {
        // Rescale this warp's O rows in TMEM (lanes without growth use 1.0).
#pragma unroll 1
        for (int c = 0; c < ATT_D / 16; ++c) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_O + (static_cast<uint32_t>(q * 32) << 16) + c * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * factor);
          tmem_st_32x32b_x16(tmem_O + (static_cast<uint32_t>(q * 32) << 16) + c * 16, v);
        }
        tmem_st_wait();
      }
      l *= factor;
      m = m_new;
      // P = 2^(x * scale_log2 - m) as fp16 into the swizzled K-major P tile
      // (two 64-key halves) of buffer j%2: one FFMA + exp per element, eight
      // partial sums so the additions stay independent.
      const uint32_t p_row = p_row0 + (j & 1) * ATT_TILE_BYTES;
      const float neg_m = -m;
      float ls[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) ls[e] = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float arg = fmaf(x[c * 8 + e], args.scale_log2, neg_m);
          p[e] = (e >= 8 - ATT_EMU_PER8) ? ex2_poly(arg) : ex2_approx(arg);
          ls[e] += p[e];
        }
        const uint32_t dst = p_row + (c >> 3) * 16384 + (((c & 7) ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pack_half2(p[0], p[1])),
                     "r"(pack_half2(p[2], p[3])), "r"(pack_half2(p[4], p[5])), "r"(pack_half2(p[6], p[7]))
                     : "memory");
      }
      l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && nkv > 0) {
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&pv_done[(nkv - 1) & 1], ((nkv - 1) >> 1) & 1, wd, SITE_ATT_SOFTMAX_PV));
      if (ok) {
        tc_fence_after();
        const int row = qt * ATT_BM + r;
        const float inv_l = 1.0f / l;
        __half* dst = nullptr;
        if (row < args.R) {
          const long long off = (args.layout == 0)
                                    ? ((static_cast<long long>(b) * args.heads_q + h) * args.R + row) * ATT_D
                                    : ((static_cast<long long>(b) * args.R + row) * args.heads_q + h) * ATT_D;
          dst = args.O + off;
        }
#pragma unroll 1
        for (int c = 0; c < ATT_D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_O + (static_cast<uint32_t>(q * 32) << 16) + c * 32, v);
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

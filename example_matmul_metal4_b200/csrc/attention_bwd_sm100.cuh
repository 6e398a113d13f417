// Flash-attention backward (non-causal, head_dim 128 and 64) for sm_100a.
//
// The reference computes these gradients only on the CPU
// (Sources/attention/Network.swift:205-401): with P = softmax(scale * Q K^T),
//   dV = P^T dO                       (derivativeV, :328-350)
//   dP = dO V^T                       (createDerivativePRow, :205-218)
//   D  = rowsum(dO * O)               (createDTerm, :258-282)
//   dS = P * (dP - D) * scale         (createDerivativeSRow, :220-256)
//   dK = dS^T Q                       (derivativeK, :351-373)
//   dQ = dS K                         (derivativeQ, :375-401)
// Here they run as three launches, none with atomics:
//   attention_bwd_prep_kernel    D per query row, and the forward's
//                                natural-log LSE moved to the log2 domain;
//                                rows padded to a multiple of 128 carry
//                                D = 0 and LSE = +inf (so their P is 0).
//   attention_bwd_dkdv_kernel    one CTA per (batch, kv head, 128 key rows):
//                                K_j, V_j stay in shared memory while every
//                                query tile of every query head of the group
//                                streams past; dK_j and dV_j accumulate in
//                                TMEM across the whole group.
//   attention_bwd_dq_kernel      one CTA per (batch, query head, 128 query
//                                rows): Q_i, dO_i stay, K_j / V_j stream;
//                                dQ_i accumulates in TMEM.
// Both main kernels recompute P from S and the stored LSE rather than
// reading it. Each streamed 128-row tile is processed as two 64-column
// halves ("units") through two TMEM buffers, so the tensor core computes one
// unit's S / dP while an element-wise warpgroup turns the other unit's S / dP
// into P / dS:
//   buffer b (units of half b):  S-shaped product in 64 columns, then dP in
//                                the next 64; the element-wise warpgroup of
//                                buffer b writes P (or dS) as fp16 pairs over
//                                the first 32 columns of each, where the
//                                accumulating MMAs read them as their A
//                                operand.
// The next unit of a buffer overwrites those fp16 pairs, so its S / dP MMAs
// are issued only after the commit of the MMAs that read them has completed
// (buf_free[b], an mbarrier), never on the strength of issue order. Two
// threads issue: warp 1 the S / dP MMAs (N = 64), warp 2 the accumulating
// ones (N = D), each in unit order, so accumulation order is fixed and the
// results are deterministic.
//
// TMEM columns (512), dK/dV kernel: [0,128) buffer 0 | [128,256) buffer 1 |
// [256,256+D) dV | [256+D,256+2D) dK. dQ kernel: [0,128) buffer 0 |
// [128,256) buffer 1 | [256,256+D) dQ.
#pragma once

#include "attention_sm100.cuh"

namespace mm4 {

struct AttnBwdArgs {
  int batch, heads_q, heads_kv, R, C, R_pad;
  int layout;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  const float* lse2;  // [B][Hq][R_pad] log2-domain LSE (+inf on pad rows)
  const float* dvec;  // [B][Hq][R_pad] D = rowsum(dO * O) (0 on pad rows)
  __half* dQ;
  __half* dK;
  __half* dV;
  int* status;
  unsigned long long timeout_ns;
};

constexpr int ATB_THREADS = 384;  // warp 0 TMA, warps 1-2 MMA, warps 4-7 / 8-11 element-wise (buffer 0 / 1)
constexpr int ATB_STAGES = 2;
constexpr int ATB_VEC_BYTES = ATT_BM * 4;  // one tile's LSE or D values
template <int D>
struct AtbCfg {
  static constexpr int TILE_BYTES = 128 * D * 2;  // one 128-row tile of head dim D
  static constexpr int DKDV_SMEM = 2 * TILE_BYTES + ATB_STAGES * (2 * TILE_BYTES + 2 * ATB_VEC_BYTES) + 256 + 1024;
  static constexpr int DQ_SMEM = 2 * TILE_BYTES + ATB_STAGES * 2 * TILE_BYTES + 256 + 1024;
  // Of every 8 exponentials of the element-wise step, this many take the
  // FMA-pipe cubic ex2_poly2 and the rest MUFU (B4 H16 S4096 on one B200:
  // D = 128 1.676 ms with 0, 1.693 with 2; D = 64 1.392 ms with 2, 1.415 with 0).
  static constexpr int EMU_PER8 = (D == 64) ? 2 : 0;
};

enum : int {
  SITE_ATB_PRODUCER = 90,
  SITE_ATB_PRODUCER_DRAIN = 91,
  SITE_ATB_MMA_FIXED = 92,
  SITE_ATB_MMA_STREAM = 93,
  SITE_ATB_MMA_P = 94,
  SITE_ATB_MMA_DRAIN = 95,
  SITE_ATB_EW_S = 96,
  SITE_ATB_EW_ACC = 97,
  SITE_ATB_MMA_FREE = 98,
};

__device__ __forceinline__ long long attn_row_offset(int layout, int b, int heads, int S, int h, int row, int D) {
  return layout == 0 ? ((static_cast<long long>(b) * heads + h) * S + row) * D
                     : ((static_cast<long long>(b) * S + row) * heads + h) * D;
}

// D and the log2-domain LSE for every (batch, query head, padded row); one
// warp per row, D / 32 elements per lane.
template <int D>
__global__ void __launch_bounds__(256) attention_bwd_prep_kernel(const __half* __restrict__ O,
                                                                 const __half* __restrict__ dO,
                                                                 const float* __restrict__ lse, float* lse2,
                                                                 float* dvec, int batch, int heads, int R, int R_pad,
                                                                 int layout) {
  const long long total = static_cast<long long>(batch) * heads * R_pad;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += warps) {
    const int row = static_cast<int>(w % R_pad);
    const long long bh = w / R_pad;
    const int h = static_cast<int>(bh % heads);
    const int b = static_cast<int>(bh / heads);
    float dot = 0.f;
    if (row < R) {
      const long long off = attn_row_offset(layout, b, heads, R, h, row, D) + lane * (D / 32);
#pragma unroll
      for (int k = 0; k < D / 32; k += 2) {
        const float2 o = __half22float2(*reinterpret_cast<const __half2*>(O + off + k));
        const float2 g = __half22float2(*reinterpret_cast<const __half2*>(dO + off + k));
        dot += o.x * g.x + o.y * g.y;
      }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
    if (lane == 0) {
      dvec[w] = dot;
      lse2[w] = row < R ? lse[bh * R + row] * 1.4426950408889634f : INFINITY;
    }
  }
}

// The element-wise step of one unit is split by columns between the two
// element-wise warpgroups: warpgroup w takes columns [32 w, 32 w + 32) of the
// unit's S (or S^T) and dP (or dP^T), and writes its fp16 pairs over the
// first 16 of those columns, which it alone reads. The accumulating MMAs
// find their A operand (K = 64) at column offsets 0, 8, 32, 40.
//
// P for the 32 columns at c0 of this thread's S row: 2^(s * sl2 - lse2),
// zero where !valid(c). EMU of every 8 exponentials on the FMA pipe.
template <int EMU, typename LseF, typename ValidF>
__device__ __forceinline__ void atb_p32(uint32_t tS, int c0, float sl2, LseF lse2_of, ValidF valid,
                                        float2 (&p)[16]) {
  uint32_t vs[32];
  tmem_ld_32x32b_x32(tS + c0, vs);
  tmem_ld_wait();
  const float2 sc = make_float2(sl2, sl2);
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int c = c0 + 2 * e;
    const float2 a = ffma2(make_float2(__uint_as_float(vs[2 * e]), __uint_as_float(vs[2 * e + 1])), sc,
                           make_float2(-lse2_of(c), -lse2_of(c + 1)));
    float2 pv;
    if ((e & 3) * 2 >= 8 - EMU) {
      pv = ex2_poly2(a);
    } else {
      pv.x = ex2_approx(a.x);
      pv.y = ex2_approx(a.y);
    }
    if (!valid(c)) pv.x = 0.f;
    if (!valid(c + 1)) pv.y = 0.f;
    p[e] = pv;
  }
}

// dS = P * (dP - D) * scale = P * (dP * scale - D * scale) for the same 32
// columns, read from this thread's dP row at tdP + c0; fp16 pairs out.
template <typename DF>
__device__ __forceinline__ void atb_ds32(uint32_t tdP, int c0, float scale, DF d_of, const float2 (&p)[16],
                                         uint32_t (&pd)[16]) {
  uint32_t vp[32];
  tmem_ld_32x32b_x32(tdP + c0, vp);
  tmem_ld_wait();
  const float2 ds = make_float2(scale, scale);
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int c = c0 + 2 * e;
    const float2 t = ffma2(make_float2(__uint_as_float(vp[2 * e]), __uint_as_float(vp[2 * e + 1])), ds,
                           make_float2(-d_of(c) * scale, -d_of(c + 1) * scale));
    const float2 dv = ffma2(p[e], t, make_float2(0.f, 0.f));
    pd[e] = pack_half2(dv.x, dv.y);
  }
}

// Reads a D-column fp32 accumulator row from TMEM and stores it as fp16.
template <int D>
__device__ __forceinline__ void atb_store_row(uint32_t taddr, __half* dst) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(taddr + c * 32, v);
    tmem_ld_wait();
    if (dst) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 pk;
        pk.x = pack_half2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
        pk.y = pack_half2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
        pk.z = pack_half2(__uint_as_float(v[i + 4]), __uint_as_float(v[i + 5]));
        pk.w = pack_half2(__uint_as_float(v[i + 6]), __uint_as_float(v[i + 7]));
        *reinterpret_cast<uint4*>(dst + c * 32 + i) = pk;
      }
    }
  }
}

// S-shaped MMA of one unit (M = 128, N = 64, K = D): D[tmem] = A_tile *
// B_rows^T, A a [128 rows][D] tile and B 64 rows of one, both stored as D/64
// 64-wide 128-byte-swizzled boxes; `b_addr` points at the unit's first row
// (tile base + 64 * 128 B for the second half).
// The descriptors are built once per call: a descriptor's low 14 bits hold
// (address >> 4), so the k-step offsets are added to it directly.
template <int D>
__device__ __forceinline__ void atb_mma_nt_unit(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr) {
  constexpr uint32_t IDESC = idesc_f16_f32(ATT_BM, ATT_BN / 2, false, false);
  const uint64_t da = sw128_desc(a_addr, 16, 1024);
  const uint64_t db = sw128_desc(b_addr, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
    umma_f16_ss(d_tmem, da + off, db + off, IDESC, kk > 0 ? 1u : 0u);
  }
}

// Accumulating MMA of one unit (M = 128, N = D, K = 64): D[tmem] (+)=
// A[tmem, fp16 pairs at column offsets 0, 8, 32, 40 (see atb_p32)] * B, B
// the unit's 64 rows of a [rows][D] tile read MN-major (`b_addr` at the
// unit's first row).
template <int D>
__device__ __forceinline__ void atb_mma_tn_unit(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr, bool acc) {
  constexpr uint32_t IDESC = idesc_f16_f32(ATT_BM, D, false, true);
  const uint64_t db = sw128_desc(b_addr, 16384, 1024);
#pragma unroll
  for (int kk = 0; kk < ATT_BN / 32; ++kk)
    umma_f16_ts(d_tmem, a_tmem + (kk >> 1) * 32 + (kk & 1) * 8, db + static_cast<uint32_t>(kk * (2048 >> 4)),
                IDESC, (acc || kk > 0) ? 1u : 0u);
}

template <int D>
__global__ void __launch_bounds__(ATB_THREADS, 1)
    attention_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                              const AttnBwdArgs args) {
  constexpr int TB = AtbCfg<D>::TILE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sK = smem;
  uint8_t* sV = sK + TB;
  uint8_t* sQ = sV + TB;                      // [STAGES]
  uint8_t* sdO = sQ + ATB_STAGES * TB;        // [STAGES]
  float* sL = reinterpret_cast<float*>(sdO + ATB_STAGES * TB);  // [STAGES][128]
  float* sD = sL + ATB_STAGES * ATT_BM;                                      // [STAGES][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sD + ATB_STAGES * ATT_BM);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;                 // STAGES
  uint64_t* q_empty = q_full + ATB_STAGES;     // STAGES
  uint64_t* s_full = q_empty + ATB_STAGES;     // 2: a unit's S^T in buffer b
  uint64_t* dp_full = s_full + 2;              // 2: its dP^T
  uint64_t* p_full = dp_full + 2;              // 2: its P^T (both element-wise warpgroups)
  uint64_t* ds_full = p_full + 2;              // 2: its dS^T
  uint64_t* free_s = ds_full + 2;              // 2: dV += P^T dO read buffer b's P^T
  uint64_t* free_dp = free_s + 2;              // 2: dK += dS^T Q read its dS^T
  uint64_t* acc_full = free_dp + 2;            // dK, dV complete
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int kv0 = blockIdx.x * ATT_BN;
  const int group = args.heads_q / args.heads_kv;
  const int nq = args.R_pad / ATT_BM;
  const int iters = group * nq;   // streamed Q / dO tiles
  const int units = 2 * iters;    // unit u: half u & 1 of tile u >> 1

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&p_full[i], 2 * ATT_BM);
      mbar_init(&ds_full[i], 2 * ATT_BM);
      mbar_init(&free_s[i], 1);
      mbar_init(&free_dp[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 2);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(kv_full, 2 * TB);
      att_load_tile_d<D>(&tmK, kv_full, sK, args.layout, kv0, hk, b);
      att_load_tile_d<D>(&tmV, kv_full, sV, args.layout, kv0, hk, b);
      int issued = 0;
      for (int n = 0; n < iters; ++n) {
        const int s = n % ATB_STAGES;
        if (!mbar_wait(&q_empty[s], ((n / ATB_STAGES) & 1) ^ 1, wd, SITE_ATB_PRODUCER)) break;
        const int hq = hk * group + n / nq;
        const int i = n % nq;
        mbar_arrive_expect_tx(&q_full[s], 2 * TB + 2 * ATB_VEC_BYTES);
        att_load_tile_d<D>(&tmQ, &q_full[s], sQ + s * TB, args.layout, i * ATT_BM, hq, b);
        att_load_tile_d<D>(&tmdO, &q_full[s], sdO + s * TB, args.layout, i * ATT_BM, hq, b);
        const long long voff = (static_cast<long long>(b) * args.heads_q + hq) * args.R_pad + i * ATT_BM;
        bulk_load(sL + s * ATT_BM, args.lse2 + voff, ATB_VEC_BYTES, &q_full[s]);
        bulk_load(sD + s * ATT_BM, args.dvec + voff, ATB_VEC_BYTES, &q_full[s]);
        issued = n + 1;
      }
      mbar_wait(kv_full, 0, wd, SITE_ATB_PRODUCER_DRAIN);
      for (int n = (issued > ATB_STAGES ? issued - ATB_STAGES : 0); n < issued; ++n)
        mbar_wait(&q_full[n % ATB_STAGES], (n / ATB_STAGES) & 1, wd, SITE_ATB_PRODUCER_DRAIN);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues every unit's S^T, dP^T (N = 64), warp 2 the accumulating
    // dV, dK MMAs (N = D) in unit order: one thread issues about one
    // tcgen05.mma per 55 SM clocks, too few for the unit's 24 MMAs. Each
    // half of a buffer is handed back separately: S^T of unit u + 2 follows
    // dV += P^T dO of unit u, dP^T follows dK += dS^T Q.
    if (elect_one()) {
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, wd, SITE_ATB_MMA_FIXED);
      for (int u = 0; u < units && ok; ++u) {
        const int n = u >> 1, hf = u & 1, s = n % ATB_STAGES;
        const uint32_t par = static_cast<uint32_t>(n & 1), prev = par ^ 1u;
        const uint32_t rows = static_cast<uint32_t>(hf) * 8192u;  // the unit's 64 query rows
        const uint32_t buf = tmem_base + hf * 128;
        if (warp == 1) {
          if (hf == 0 && !mbar_wait(&q_full[s], (n / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
          if (u >= 2 && !mbar_wait(&free_s[hf], prev, wd, SITE_ATB_MMA_FREE)) break;
          tc_fence_after();
          atb_mma_nt_unit<D>(buf, k_addr, smem_u32(sQ + s * TB) + rows);  // S^T = K_j Q^T
          umma_commit(&s_full[hf]);
          if (u >= 2 && !mbar_wait(&free_dp[hf], prev, wd, SITE_ATB_MMA_FREE)) break;
          tc_fence_after();
          atb_mma_nt_unit<D>(buf + 64, v_addr, smem_u32(sdO + s * TB) + rows);  // dP^T = V_j dO^T
          umma_commit(&dp_full[hf]);
        } else {
          if (hf == 0 && !mbar_wait(&q_full[s], (n / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
          if (!mbar_wait(&p_full[hf], par, wd, SITE_ATB_MMA_P)) break;
          tc_fence_after();
          atb_mma_tn_unit<D>(tmem_base + 256, buf, smem_u32(sdO + s * TB) + rows, u > 0);  // dV += P^T dO
          umma_commit(&free_s[hf]);
          if (!mbar_wait(&ds_full[hf], par, wd, SITE_ATB_MMA_P)) break;
          tc_fence_after();
          atb_mma_tn_unit<D>(tmem_base + 256 + D, buf + 64, smem_u32(sQ + s * TB) + rows, u > 0);  // dK += dS^T Q
          umma_commit(&free_dp[hf]);
          if (hf == 1) umma_commit(&q_empty[s]);
        }
      }
      if (warp == 2) umma_commit(acc_full);
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATB_MMA_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ P^T, dS^T and the epilogue
    // Both warpgroups work on every unit, warpgroup w on its columns
    // [32 w, 32 w + 32) (query rows of the unit); P^T is released first so
    // dV += P^T dO can start while dS^T is formed.
    const int w = (warp - 4) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;    // key row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const int c0 = 32 * w;
    bool ok = true;
    for (int u = 0; u < units; ++u) {
      const int n = u >> 1, hf = u & 1, s = n % ATB_STAGES;
      const uint32_t tS = tmem_base + hf * 128 + lane_off;
      // The stage's LSE / D vectors arrive by bulk copy on q_full[s]; waiting
      // on that phase too makes them visible here. It cannot have moved on:
      // the stage is refilled only after this tile's last dS^T is consumed.
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[hf], n & 1, wd, SITE_ATB_EW_S) &&
                                       mbar_wait(&q_full[s], (n / ATB_STAGES) & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      const float* L = sL + s * ATT_BM + hf * 64;
      const float* Dv = sD + s * ATT_BM + hf * 64;
      float2 p[16];
      atb_p32<AtbCfg<D>::EMU_PER8>(tS, c0, args.scale_log2, [&](int c) { return L[c]; }, [](int) { return true; }, p);
      {
        uint32_t pp[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) pp[e] = pack_half2(p[e].x, p[e].y);
        tmem_st_32x32b_x16(tS + c0, pp);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[hf]);
      ok = __all_sync(0xffffffffu, mbar_wait(&dp_full[hf], n & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      uint32_t pd[16];
      atb_ds32(tS + 64, c0, args.scale, [&](int c) { return Dv[c]; }, p, pd);
      tmem_st_32x32b_x16(tS + 64 + c0, pd);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&ds_full[hf]);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(acc_full, 0, wd, SITE_ATB_EW_ACC))) {
      tc_fence_after();
      const int row = kv0 + r;
      const bool live = row < args.C;
      const long long off = attn_row_offset(args.layout, b, args.heads_kv, args.C, hk, live ? row : 0, D);
      // warpgroup 0 stores dV, warpgroup 1 dK
      if (w == 0)
        atb_store_row<D>(tmem_base + 256 + lane_off, live ? args.dV + off : nullptr);
      else
        atb_store_row<D>(tmem_base + 256 + D + lane_off, live ? args.dK + off : nullptr);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int D>
__global__ void __launch_bounds__(ATB_THREADS, 1)
    attention_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                            const AttnBwdArgs args) {
  constexpr int TB = AtbCfg<D>::TILE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + TB;
  uint8_t* sK = sdO + TB;                  // [STAGES]
  uint8_t* sV = sK + ATB_STAGES * TB;      // [STAGES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ATB_STAGES * TB);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // STAGES
  uint64_t* kv_empty = kv_full + ATB_STAGES;   // STAGES
  uint64_t* s_full = kv_empty + ATB_STAGES;    // 2: a unit's S in buffer b
  uint64_t* dp_full = s_full + 2;              // 2: its dP
  uint64_t* ds_full = dp_full + 2;             // 2: its dS (both element-wise warpgroups)
  uint64_t* buf_free = ds_full + 2;            // 2: dQ += dS K read buffer b's dS
  uint64_t* acc_full = buf_free + 2;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = blockIdx.x * ATT_BM;
  const int hk = h / (args.heads_q / args.heads_kv);
  const int nkv = (args.C + ATT_BN - 1) / ATT_BN;
  const int units = 2 * nkv;  // unit u: key half u & 1 of tile u >> 1

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&ds_full[i], 2 * ATT_BM);
      mbar_init(&buf_free[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 2);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(q_full, 2 * TB);
      att_load_tile_d<D>(&tmQ, q_full, sQ, args.layout, q0, h, b);
      att_load_tile_d<D>(&tmdO, q_full, sdO, args.layout, q0, h, b);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % ATB_STAGES;
        if (!mbar_wait(&kv_empty[s], ((j / ATB_STAGES) & 1) ^ 1, wd, SITE_ATB_PRODUCER)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * TB);
        att_load_tile_d<D>(&tmK, &kv_full[s], sK + s * TB, args.layout, j * ATT_BN, hk, b);
        att_load_tile_d<D>(&tmV, &kv_full[s], sV + s * TB, args.layout, j * ATT_BN, hk, b);
        issued = j + 1;
      }
      mbar_wait(q_full, 0, wd, SITE_ATB_PRODUCER_DRAIN);
      for (int j = (issued > ATB_STAGES ? issued - ATB_STAGES : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % ATB_STAGES], (j / ATB_STAGES) & 1, wd, SITE_ATB_PRODUCER_DRAIN);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 1 issues every unit's S, dP (N = 64), warp 2 the accumulating dQ
    // MMAs (N = D) in unit order.
    if (elect_one()) {
      const uint32_t q_addr = smem_u32(sQ), g_addr = smem_u32(sdO);
      bool ok = mbar_wait(q_full, 0, wd, SITE_ATB_MMA_FIXED);
      for (int u = 0; u < units && ok; ++u) {
        const int j = u >> 1, hf = u & 1, s = j % ATB_STAGES;
        const uint32_t rows = static_cast<uint32_t>(hf) * 8192u;  // the unit's 64 key rows
        const uint32_t buf = tmem_base + hf * 128;
        if (warp == 1) {
          // Unit u reuses buffer hf: its S overwrites the dS unit u - 2's dQ
          // MMAs read.
          if (u >= 2 && !mbar_wait(&buf_free[hf], ((u - 2) >> 1) & 1, wd, SITE_ATB_MMA_FREE)) break;
          if (hf == 0 && !mbar_wait(&kv_full[s], (j / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
          tc_fence_after();
          atb_mma_nt_unit<D>(buf, q_addr, smem_u32(sK + s * TB) + rows);  // S = Q_i K^T
          umma_commit(&s_full[hf]);
          atb_mma_nt_unit<D>(buf + 64, g_addr, smem_u32(sV + s * TB) + rows);  // dP = dO_i V^T
          umma_commit(&dp_full[hf]);
        } else {
          if (!mbar_wait(&ds_full[hf], j & 1, wd, SITE_ATB_MMA_P)) break;
          if (hf == 0 && !mbar_wait(&kv_full[s], (j / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
          tc_fence_after();
          atb_mma_tn_unit<D>(tmem_base + 256, buf, smem_u32(sK + s * TB) + rows, u > 0);  // dQ += dS K
          umma_commit(&buf_free[hf]);
          if (hf == 1) umma_commit(&kv_empty[s]);
        }
      }
      if (warp == 2) umma_commit(acc_full);
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATB_MMA_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dS and the epilogue
    // Both warpgroups work on every unit, warpgroup w on its columns
    // [32 w, 32 w + 32) (keys of the unit); P stays in registers.
    const int w = (warp - 4) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;    // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const int c0 = 32 * w;
    const long long voff = (static_cast<long long>(b) * args.heads_q + h) * args.R_pad + q0 + r;
    const float lse2 = args.lse2[voff];
    const float dterm = args.dvec[voff];
    bool ok = true;
    for (int u = 0; u < units; ++u) {
      const int j = u >> 1, hf = u & 1;
      const uint32_t tS = tmem_base + hf * 128 + lane_off;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[hf], j & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      const int valid = args.C - j * ATT_BN - hf * 64;  // key columns of this unit inside C
      float2 p[16];
      atb_p32<AtbCfg<D>::EMU_PER8>(tS, c0, args.scale_log2, [&](int) { return lse2; }, [&](int c) { return c < valid; }, p);
      ok = __all_sync(0xffffffffu, mbar_wait(&dp_full[hf], j & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      // dS over this warpgroup's S columns (the dQ MMA reads it there).
      uint32_t pd[16];
      atb_ds32(tS + 64, c0, args.scale, [&](int) { return dterm; }, p, pd);
      tmem_st_32x32b_x16(tS + c0, pd);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&ds_full[hf]);
    }
    if (ok && w == 0 && __all_sync(0xffffffffu, mbar_wait(acc_full, 0, wd, SITE_ATB_EW_ACC))) {
      tc_fence_after();
      const int row = q0 + r;
      const bool live = row < args.R;
      const long long off = attn_row_offset(args.layout, b, args.heads_q, args.R, h, live ? row : 0, D);
      atb_store_row<D>(tmem_base + 256 + lane_off, live ? args.dQ + off : nullptr);
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

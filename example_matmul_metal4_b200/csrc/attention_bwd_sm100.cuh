// Flash-attention backward (non-causal, head_dim 128) for sm_100a.
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
// reading it. Their tensor-core steps are tcgen05.mma with fp32 TMEM
// accumulators; the element-wise step (P, dS) runs in four warps, one TMEM
// lane (one row of S^T or S) per thread, and writes P / dS as fp16 pairs back
// over the S / dP columns they came from, where the next MMAs read them as
// their A operand (the forward kernel's P-over-S scheme: the MMAs of one
// issuing thread execute in issue order, so the next S overwrites P only
// after the MMAs that read it).
//
// TMEM columns (512), dK/dV kernel: [0,128) S^T then P^T | [128,256) dP^T
// then dS^T | [256,384) dV | [384,512) dK. dQ kernel: [0,128) S then dS |
// [128,256) dP | [256,384) dQ.
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

constexpr int ATB_THREADS = 256;  // warp 0 TMA, warp 1 MMA, warps 4-7 element-wise + epilogue
constexpr int ATB_STAGES = 2;
constexpr int ATB_VEC_BYTES = ATT_BM * 4;  // one tile's LSE or D values
constexpr int ATB_DKDV_SMEM =
    2 * ATT_TILE_BYTES + ATB_STAGES * (2 * ATT_TILE_BYTES + 2 * ATB_VEC_BYTES) + 256 + 1024;
constexpr int ATB_DQ_SMEM = 2 * ATT_TILE_BYTES + ATB_STAGES * 2 * ATT_TILE_BYTES + 256 + 1024;

enum : int {
  SITE_ATB_PRODUCER = 90,
  SITE_ATB_PRODUCER_DRAIN = 91,
  SITE_ATB_MMA_FIXED = 92,
  SITE_ATB_MMA_STREAM = 93,
  SITE_ATB_MMA_P = 94,
  SITE_ATB_MMA_DRAIN = 95,
  SITE_ATB_EW_S = 96,
  SITE_ATB_EW_ACC = 97,
};

__device__ __forceinline__ long long attn_row_offset(int layout, int b, int heads, int S, int h, int row) {
  return layout == 0 ? ((static_cast<long long>(b) * heads + h) * S + row) * ATT_D
                     : ((static_cast<long long>(b) * S + row) * heads + h) * ATT_D;
}

// D and the log2-domain LSE for every (batch, query head, padded row); one
// warp per row.
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
      const long long off = attn_row_offset(layout, b, heads, R, h, row) + lane * 4;
      const uint2 ov = *reinterpret_cast<const uint2*>(O + off);
      const uint2 gv = *reinterpret_cast<const uint2*>(dO + off);
      const float2 o0 = __half22float2(*reinterpret_cast<const __half2*>(&ov.x));
      const float2 o1 = __half22float2(*reinterpret_cast<const __half2*>(&ov.y));
      const float2 g0 = __half22float2(*reinterpret_cast<const __half2*>(&gv.x));
      const float2 g1 = __half22float2(*reinterpret_cast<const __half2*>(&gv.y));
      dot = o0.x * g0.x + o0.y * g0.y + o1.x * g1.x + o1.y * g1.y;
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, s);
    if (lane == 0) {
      dvec[w] = dot;
      lse2[w] = row < R ? lse[bh * R + row] * 1.4426950408889634f : INFINITY;
    }
  }
}

// One 64-column half of a thread's S / dP row pair: P = 2^(s * scale_log2 -
// lse2), dS = P * (dP - D) * scale, packed as fp16 pairs. Column c uses
// lse2_of(c) / d_of(c) and is zeroed when !valid(c).
template <typename LseF, typename DF, typename ValidF>
__device__ __forceinline__ void atb_elementwise_half(uint32_t tS, uint32_t tP, int half, float sl2, float scale,
                                                     LseF lse2_of, DF d_of, ValidF valid, uint32_t (&pp)[32],
                                                     uint32_t (&pd)[32]) {
#pragma unroll
  for (int sub = 0; sub < 2; ++sub) {
    const int c0 = half * 64 + sub * 32;
    uint32_t vs[32], vp[32];
    tmem_ld_32x32b_x32(tS + c0, vs);
    tmem_ld_32x32b_x32(tP + c0, vp);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int c = c0 + 2 * e;
      float p0 = ex2_approx(__uint_as_float(vs[2 * e]) * sl2 - lse2_of(c));
      float p1 = ex2_approx(__uint_as_float(vs[2 * e + 1]) * sl2 - lse2_of(c + 1));
      if (!valid(c)) p0 = 0.f;
      if (!valid(c + 1)) p1 = 0.f;
      const float d0 = p0 * (__uint_as_float(vp[2 * e]) - d_of(c)) * scale;
      const float d1 = p1 * (__uint_as_float(vp[2 * e + 1]) - d_of(c + 1)) * scale;
      pp[sub * 16 + e] = pack_half2(p0, p1);
      pd[sub * 16 + e] = pack_half2(d0, d1);
    }
  }
}

// Reads a 128-column fp32 accumulator row from TMEM and stores it as fp16.
__device__ __forceinline__ void atb_store_row(uint32_t taddr, __half* dst) {
#pragma unroll 1
  for (int c = 0; c < ATT_D / 32; ++c) {
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

// S-shaped MMA (M = 128, N = 128, K = D): D[tmem] = A_tile * B_tile^T, both
// tiles [128 rows][128 D] as two 64-wide 128-byte-swizzled boxes.
__device__ __forceinline__ void atb_mma_nt(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr) {
  constexpr uint32_t IDESC_S = idesc_f16_f32(ATT_BM, ATT_BN, false, false);
#pragma unroll
  for (int kk = 0; kk < ATT_D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
    umma_f16_ss(d_tmem, sw128_desc(a_addr + off, 16, 1024), sw128_desc(b_addr + off, 16, 1024), IDESC_S,
                kk > 0 ? 1u : 0u);
  }
}

// PV-shaped MMA (M = 128, N = D, K = 128): D[tmem] (+)= A[tmem, fp16 pairs in
// 64 columns] * B_tile, B a [128 K rows][128 D] tile read MN-major.
__device__ __forceinline__ void atb_mma_tn(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_addr, bool acc) {
  constexpr uint32_t IDESC_O = idesc_f16_f32(ATT_BM, ATT_D, false, true);
#pragma unroll
  for (int kk = 0; kk < ATT_BN / 16; ++kk)
    umma_f16_ts(d_tmem, a_tmem + kk * 8, sw128_desc(b_addr + kk * 2048, 16384, 1024), IDESC_O,
                (acc || kk > 0) ? 1u : 0u);
}

__global__ void __launch_bounds__(ATB_THREADS, 1)
    attention_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                              const AttnBwdArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sK = smem;
  uint8_t* sV = sK + ATT_TILE_BYTES;
  uint8_t* sQ = sV + ATT_TILE_BYTES;                      // [STAGES]
  uint8_t* sdO = sQ + ATB_STAGES * ATT_TILE_BYTES;        // [STAGES]
  float* sL = reinterpret_cast<float*>(sdO + ATB_STAGES * ATT_TILE_BYTES);  // [STAGES][128]
  float* sD = sL + ATB_STAGES * ATT_BM;                                      // [STAGES][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sD + ATB_STAGES * ATT_BM);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;                 // STAGES
  uint64_t* q_empty = q_full + ATB_STAGES;     // STAGES
  uint64_t* s_full = q_empty + ATB_STAGES;     // S^T, dP^T in TMEM
  uint64_t* p_full = s_full + 1;               // P^T, dS^T in TMEM
  uint64_t* acc_full = p_full + 1;             // dK, dV complete
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
  const int iters = group * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, ATT_BM);
    mbar_init(acc_full, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(kv_full, 2 * ATT_TILE_BYTES);
      att_load_tile(&tmK, kv_full, sK, args.layout, kv0, hk, b);
      att_load_tile(&tmV, kv_full, sV, args.layout, kv0, hk, b);
      int issued = 0;
      for (int n = 0; n < iters; ++n) {
        const int s = n % ATB_STAGES;
        if (!mbar_wait(&q_empty[s], ((n / ATB_STAGES) & 1) ^ 1, wd, SITE_ATB_PRODUCER)) break;
        const int hq = hk * group + n / nq;
        const int i = n % nq;
        mbar_arrive_expect_tx(&q_full[s], 2 * ATT_TILE_BYTES + 2 * ATB_VEC_BYTES);
        att_load_tile(&tmQ, &q_full[s], sQ + s * ATT_TILE_BYTES, args.layout, i * ATT_BM, hq, b);
        att_load_tile(&tmdO, &q_full[s], sdO + s * ATT_TILE_BYTES, args.layout, i * ATT_BM, hq, b);
        const long long voff = (static_cast<long long>(b) * args.heads_q + hq) * args.R_pad + i * ATT_BM;
        bulk_load(sL + s * ATT_BM, args.lse2 + voff, ATB_VEC_BYTES, &q_full[s]);
        bulk_load(sD + s * ATT_BM, args.dvec + voff, ATB_VEC_BYTES, &q_full[s]);
        issued = n + 1;
      }
      mbar_wait(kv_full, 0, wd, SITE_ATB_PRODUCER_DRAIN);
      for (int n = (issued > ATB_STAGES ? issued - ATB_STAGES : 0); n < issued; ++n)
        mbar_wait(&q_full[n % ATB_STAGES], (n / ATB_STAGES) & 1, wd, SITE_ATB_PRODUCER_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      bool ok = mbar_wait(kv_full, 0, wd, SITE_ATB_MMA_FIXED);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      for (int n = 0; n < iters && ok; ++n) {
        const int s = n % ATB_STAGES;
        if (!mbar_wait(&q_full[s], (n / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + s * ATT_TILE_BYTES);
        const uint32_t g_addr = smem_u32(sdO + s * ATT_TILE_BYTES);
        atb_mma_nt(tmem_base + 0, k_addr, q_addr);    // S^T = K_j Q_i^T
        atb_mma_nt(tmem_base + 128, v_addr, g_addr);  // dP^T = V_j dO_i^T
        umma_commit(s_full);
        if (!mbar_wait(p_full, n & 1, wd, SITE_ATB_MMA_P)) break;
        tc_fence_after();
        atb_mma_tn(tmem_base + 256, tmem_base + 0, g_addr, n > 0);    // dV += P^T dO_i
        atb_mma_tn(tmem_base + 384, tmem_base + 128, q_addr, n > 0);  // dK += dS^T Q_i
        umma_commit(&q_empty[s]);
      }
      umma_commit(acc_full);
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATB_MMA_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ P^T, dS^T and the epilogue
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // key row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tS = tmem_base + lane_off;
    const uint32_t tP = tmem_base + 128 + lane_off;
    bool ok = true;
    for (int n = 0; n < iters; ++n) {
      const int s = n % ATB_STAGES;
      // The stage's LSE / D vectors arrive by bulk copy on q_full[s]; waiting
      // on that phase too makes them visible here. It cannot have moved on:
      // the stage is refilled only after this iteration's p_full.
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, n & 1, wd, SITE_ATB_EW_S) &&
                                       mbar_wait(&q_full[s], (n / ATB_STAGES) & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      const float* L = sL + s * ATT_BM;
      const float* Dv = sD + s * ATT_BM;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t pp[32], pd[32];
        atb_elementwise_half(
            tS, tP, half, args.scale_log2, args.scale, [&](int c) { return L[c]; }, [&](int c) { return Dv[c]; },
            [](int) { return true; }, pp, pd);
        tmem_st_32x32b_x32(tS + half * 32, pp);
        tmem_st_32x32b_x32(tP + half * 32, pd);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(acc_full, 0, wd, SITE_ATB_EW_ACC))) {
      tc_fence_after();
      const int row = kv0 + r;
      const bool live = row < args.C;
      const long long off = attn_row_offset(args.layout, b, args.heads_kv, args.C, hk, live ? row : 0);
      atb_store_row(tmem_base + 256 + lane_off, live ? args.dV + off : nullptr);
      atb_store_row(tmem_base + 384 + lane_off, live ? args.dK + off : nullptr);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

__global__ void __launch_bounds__(ATB_THREADS, 1)
    attention_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                            const AttnBwdArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + ATT_TILE_BYTES;
  uint8_t* sK = sdO + ATT_TILE_BYTES;                  // [STAGES]
  uint8_t* sV = sK + ATB_STAGES * ATT_TILE_BYTES;      // [STAGES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ATB_STAGES * ATT_TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                // STAGES
  uint64_t* kv_empty = kv_full + ATB_STAGES;   // STAGES
  uint64_t* s_full = kv_empty + ATB_STAGES;
  uint64_t* p_full = s_full + 1;
  uint64_t* acc_full = p_full + 1;
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

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ATB_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, ATT_BM);
    mbar_init(acc_full, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(q_full, 2 * ATT_TILE_BYTES);
      att_load_tile(&tmQ, q_full, sQ, args.layout, q0, h, b);
      att_load_tile(&tmdO, q_full, sdO, args.layout, q0, h, b);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % ATB_STAGES;
        if (!mbar_wait(&kv_empty[s], ((j / ATB_STAGES) & 1) ^ 1, wd, SITE_ATB_PRODUCER)) break;
        mbar_arrive_expect_tx(&kv_full[s], 2 * ATT_TILE_BYTES);
        att_load_tile(&tmK, &kv_full[s], sK + s * ATT_TILE_BYTES, args.layout, j * ATT_BN, hk, b);
        att_load_tile(&tmV, &kv_full[s], sV + s * ATT_TILE_BYTES, args.layout, j * ATT_BN, hk, b);
        issued = j + 1;
      }
      mbar_wait(q_full, 0, wd, SITE_ATB_PRODUCER_DRAIN);
      for (int j = (issued > ATB_STAGES ? issued - ATB_STAGES : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % ATB_STAGES], (j / ATB_STAGES) & 1, wd, SITE_ATB_PRODUCER_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      bool ok = mbar_wait(q_full, 0, wd, SITE_ATB_MMA_FIXED);
      const uint32_t q_addr = smem_u32(sQ), g_addr = smem_u32(sdO);
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % ATB_STAGES;
        if (!mbar_wait(&kv_full[s], (j / ATB_STAGES) & 1, wd, SITE_ATB_MMA_STREAM)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * ATT_TILE_BYTES);
        const uint32_t v_addr = smem_u32(sV + s * ATT_TILE_BYTES);
        atb_mma_nt(tmem_base + 0, q_addr, k_addr);    // S = Q_i K_j^T
        atb_mma_nt(tmem_base + 128, g_addr, v_addr);  // dP = dO_i V_j^T
        umma_commit(s_full);
        if (!mbar_wait(p_full, j & 1, wd, SITE_ATB_MMA_P)) break;
        tc_fence_after();
        atb_mma_tn(tmem_base + 256, tmem_base + 0, k_addr, j > 0);  // dQ += dS K_j
        umma_commit(&kv_empty[s]);
      }
      umma_commit(acc_full);
      umma_commit(drain);
      mbar_wait(drain, 0, wd, SITE_ATB_MMA_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dS and the epilogue
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tS = tmem_base + lane_off;
    const uint32_t tP = tmem_base + 128 + lane_off;
    const long long voff = (static_cast<long long>(b) * args.heads_q + h) * args.R_pad + q0 + r;
    const float lse2 = args.lse2[voff];
    const float dterm = args.dvec[voff];
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, wd, SITE_ATB_EW_S));
      if (!ok) break;
      tc_fence_after();
      const int valid = args.C - j * ATT_BN;  // key columns of this tile inside C
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t pp[32], pd[32];
        atb_elementwise_half(
            tS, tP, half, args.scale_log2, args.scale, [&](int) { return lse2; }, [&](int) { return dterm; },
            [&](int c) { return c < valid; }, pp, pd);
        tmem_st_32x32b_x32(tS + half * 32, pd);  // dS over S; P is not needed here
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(acc_full, 0, wd, SITE_ATB_EW_ACC))) {
      tc_fence_after();
      const int row = q0 + r;
      const bool live = row < args.R;
      const long long off = attn_row_offset(args.layout, b, args.heads_q, args.R, h, live ? row : 0);
      atb_store_row(tmem_base + 256 + lane_off, live ? args.dQ + off : nullptr);
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

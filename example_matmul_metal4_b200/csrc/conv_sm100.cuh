// Implicit-GEMM convolution (conv2d and conv3d, NDHWC) for sm_100a.
//
// Replaces the reference's conv kernels: the conv2d tensor op
// (ConvolutionShared.swift:4631-4836), the padded conv2d probe
// (convolution2d_padding.swift:109-210) and the conv3d depth-slice kernels
// (ConvolutionShared.swift:4431-4591, :4282-4429), which the reference runs
// as N*OD*KD host-orchestrated launches with fp16 read-modify-write of the
// output between them. Here a conv3d is ONE launch: the depth taps are part
// of the K loop and the accumulator stays fp32 in TMEM until the epilogue.
//
// GEMM view: M = N*OD*OH*OW output pixels, N = Cout, K = taps x Cin with Cin
// padded to 64 per tap, so every 64-wide k-block is one filter tap and one
// 64-channel slab: kb = tap * ceil(Cin/64) + cb.
//
// CTA = 10 warps (one CTA per SM, persistent over output tiles):
//   warp 0     weights producer (TMA) when the weights are 16-byte pitched
//   warp 1     TMEM alloc + tcgen05.mma issuer        (shared with the GEMM)
//   warps 2-5  epilogue: bias, fp16, NDHWC store      (shared with the GEMM)
//   For stride-1 convolutions with 16-byte-pitched channels, warp 0 also
//   loads the activations by TMA: a tile is a TH x TW rectangle of output
//   pixels (TW*TH = 128) of one (n, oz) plane, so each tap's A operand is one
//   5-D box {64 channels, TW, TH, 1, 1} of the NDHWC input at the tap-shifted
//   origin, with out-of-range (padding) coordinates zero-filled by TMA.
//   Otherwise:
//   warps 6-9  activation gather: each thread owns one 16-byte channel chunk
//              of 8 tile rows and copies it with cp.async (zero-filled when
//              the tap falls in the padding or past Cin). Replaces the
//              reference's clamp + set_offsets padding rule
//              (AGENTS.md:76-84): out-of-range taps simply read zeros.
// With 16-byte-aligned channels and TMA weights, the gather threads arrive on
// a stage's mbarrier with cp.async.mbarrier.arrive.noinc (the arrival fires
// when the thread's copies land), so up to STAGES stages are in flight with
// no producer-side waits; the MMA thread issues fence.proxy.async after its
// wait so the tensor core (async proxy) observes the cp.async writes. Shapes
// that need ordinary shared-memory stores (unaligned channels or gathered
// weights) complete their writes, fence, and arrive synchronously.
#pragma once

#include "gemm_sm100.cuh"

namespace mm4 {

struct ConvGeom {
  int N, D, H, W, C, O;
  int KD, KH, KW;
  int SZ, SY, SX, DZ, DY, DX;
  int PF, PT, PL;  // front / top / left padding
  int OD, OH, OW;
  int ncb;         // ceil(C / 64)
  int taps;        // KD*KH*KW
  int w_layout;    // mm4 weight layout id (for the gathered-weights path)
  int x_vec;       // C % 8 == 0 and x 16-byte aligned: 16-byte cp.async
  const __half* x;
  const __half* w;
};

constexpr int CONV_THREADS = 320;
constexpr int CONV_GATHER_THREADS = 128;
constexpr int CONV_GATHER_T0 = 192;  // first gather thread (warp 6)

enum : int {
  SITE_CONV_GATHER_EMPTY = 20,
  SITE_CONV_WTMA_EMPTY = 21,
  SITE_CONV_WTMA_DRAIN = 22,
};

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Arrives on the mbarrier once all cp.async issued so far by this thread have
// landed; counts as one of the barrier's expected arrivals (.noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Offset of weight element (oc, tap, ic) for the 2-D/3-D layouts; tap is the
// flattened (kd, kh, kw) index.
__device__ __forceinline__ long long conv_weight_offset(const ConvGeom& g, int oc, int tap, int ic) {
  switch (g.w_layout) {
    case 0:  // HWIO
    case 3:  // DHWIO
      return (static_cast<long long>(tap) * g.C + ic) * g.O + oc;
    default:  // OHWI / ODHWI
      return (static_cast<long long>(oc) * g.taps + tap) * g.C + ic;
  }
}

// Tile origin (in input coordinates, before the tap offset) of an output
// rectangle tile when activations are TMA-fed (stride 1).
struct ConvTileOrigin {
  int n, z, y, x;
};

__device__ __forceinline__ ConvTileOrigin conv_tile_origin(const GemmArgs& a, const ConvGeom& g, int mt) {
  int t = mt;
  const int twi = t % a.rm_tiles_w;
  t /= a.rm_tiles_w;
  const int thi = t % a.rm_tiles_h;
  t /= a.rm_tiles_h;
  const int oz = t % a.rm_od;
  ConvTileOrigin o;
  o.n = t / a.rm_od;
  o.z = oz - g.PF;
  o.y = thi * a.rm_th - g.PT;
  o.x = twi * a.rm_tw - g.PL;
  return o;
}

// How the activations reach shared memory.
enum : int {
  CONV_A_GATHER = 0,  // cp.async gather warps (any stride / channel pitch)
  CONV_A_RECT = 1,    // TMA 5-D box over a TH x TW output rectangle (stride 1)
  CONV_A_IM2COL = 2,  // TMA im2col: 128 consecutive output pixels (stride 1)
};

template <int BN, bool B_TMA, bool B_MN, int A_MODE>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    conv_sm100_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                      const GemmArgs args, const ConvGeom g) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool A_TMA = A_MODE != CONV_A_GATHER;

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
  const Watchdog wd{args.status, args.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], A_TMA ? 1 : CONV_GATHER_THREADS + (B_TMA ? 1 : 0));
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ weights via TMA
    if (B_TMA && elect_one()) {
      tma_prefetch_desc(&tmW);
      if (A_TMA) tma_prefetch_desc(&tmX);
      uint32_t fills = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < args.num_units && ok; u += gridDim.x) {
        const GemmUnit w = gemm_decode_unit(args, u);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(fills % STAGES);
          const uint32_t ph = (fills / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, wd, SITE_CONV_WTMA_EMPTY)) {
            ok = false;
            break;
          }
          const int tap = kb / g.ncb;
          const int cb = kb - tap * g.ncb;
          uint8_t* sB = ring + s * Cfg::STAGE_BYTES + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[s], A_TMA ? Cfg::STAGE_BYTES : Cfg::B_BYTES);
          if (A_TMA) {
            const int kd = tap / (g.KH * g.KW);
            const int khw = tap - kd * (g.KH * g.KW);
            const int kh = khw / g.KW;
            const int kw = khw - kh * g.KW;
            if (A_MODE == CONV_A_RECT) {
              // Activation box {64 ch, TW, TH, 1, 1}: the output rectangle's
              // input footprint for this tap; padding taps read zeros (OOB fill).
              const ConvTileOrigin o = conv_tile_origin(args, g, w.mt);
              tma_load_5d(&tmX, &full[s], ring + s * Cfg::STAGE_BYTES, cb * 64, o.x + kw * g.DX, o.y + kh * g.DY,
                          o.z + kd * g.DZ, o.n);
            } else {
              // im2col: the tile is output pixels [128 mt, 128 mt + 128) in
              // (n, oz, oy, ox) order; the load starts at the first pixel's
              // window origin and walks the window box, this tap's offset
              // added; padding and pixels past the end read zeros.
              const int m0 = w.mt * GEMM_BM;
              const int ox = m0 % g.OW;
              const int r1 = m0 / g.OW;
              const int oy = r1 % g.OH;
              const int r2 = r1 / g.OH;
              const int oz = r2 % g.OD;
              const int n = r2 / g.OD;
              tma_load_5d_im2col(&tmX, &full[s], ring + s * Cfg::STAGE_BYTES, cb * 64, ox - g.PL, oy - g.PT,
                                 oz - g.PF, n, static_cast<uint16_t>(kw * g.DX), static_cast<uint16_t>(kh * g.DY),
                                 static_cast<uint16_t>(kd * g.DZ));
            }
          }
          if (!B_MN) {
            // [Cout][taps][Cin]: box 64(Cin) x 1(tap) x BN(Cout)
            tma_load_3d(&tmW, &full[s], sB, cb * 64, tap, w.nt * BN);
          } else {
            // [taps][Cin][Cout]: box 64(Cout) x 64(Cin) x 1(tap), BN/64 boxes
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(&tmW, &full[s], sB + j * 8192, w.nt * BN + 64 * j, cb * 64, tap);
          }
          ++fills;
        }
      }
      const uint32_t first = fills > STAGES ? fills - STAGES : 0u;
      for (uint32_t i = first; i < fills; ++i) {
        if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, wd, SITE_CONV_WTMA_DRAIN)) break;
      }
    }
  } else if (warp == 1) {
    if (elect_one())
      mma_role<BN, false, B_MN, STAGES, Cfg::STAGE_BYTES, Cfg::A_BYTES, !A_TMA>(args, ring, full, empty, tmem_full,
                                                                           tmem_empty, drain, tmem_base, wd);
  } else if (warp < 6) {
    epilogue_role<BN, MODE_DIRECT_F16>(args, tmem_full, tmem_empty, tmem_base, s_vote, s_last, nullptr, wd, warp,
                                       lane);
  } else if (!A_TMA) {
    // ------------------------------------------------ activation gather
    const int gt = threadIdx.x - CONV_GATHER_T0;  // 0..127
    const int j = gt & 7;                          // 16-byte channel chunk within the 128-byte row
    const int rg = gt >> 3;                        // rows rg, rg+16, ..., rg+112
    const long long m_total = static_cast<long long>(g.N) * g.OD * g.OH * g.OW;
    // Launch-uniform: activations by 16-byte cp.async and weights by TMA.
    const bool fast = B_TMA && g.x_vec;
    uint32_t fills = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < args.num_units && ok; u += gridDim.x) {
      const GemmUnit w = gemm_decode_unit(args, u);
      // Per-row input origin of the 8 tile rows this thread fills.
      int rn[8], rz[8], ry[8], rx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const long long p = static_cast<long long>(w.mt) * GEMM_BM + rg + 16 * i;
        if (p < m_total) {
          long long t = p;
          const int ow = static_cast<int>(t % g.OW);
          t /= g.OW;
          const int oh = static_cast<int>(t % g.OH);
          t /= g.OH;
          const int oz = static_cast<int>(t % g.OD);
          rn[i] = static_cast<int>(t / g.OD);
          rz[i] = oz * g.SZ - g.PF;
          ry[i] = oh * g.SY - g.PT;
          rx[i] = ow * g.SX - g.PL;
        } else {
          rn[i] = -1;
          rz[i] = ry[i] = rx[i] = 0;
        }
      }
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        const int s = static_cast<int>(fills % STAGES);
        const uint32_t ph = (fills / STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, wd, SITE_CONV_GATHER_EMPTY)) {
          ok = false;
          break;
        }
        const int tap = kb / g.ncb;
        const int cb = kb - tap * g.ncb;
        const int kd = tap / (g.KH * g.KW);
        const int khw = tap - kd * (g.KH * g.KW);
        const int kh = khw / g.KW;
        const int kw = khw - kh * g.KW;
        const int c = cb * 64 + j * 8;
        uint8_t* sA = ring + s * Cfg::STAGE_BYTES;
        const uint32_t sA_addr = smem_u32(sA);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = rg + 16 * i;
          const uint32_t dst = sA_addr + r * 128 + ((j ^ (r & 7)) << 4);
          const int iz = rz[i] + kd * g.DZ;
          const int ih = ry[i] + kh * g.DY;
          const int iw = rx[i] + kw * g.DX;
          const bool inside = rn[i] >= 0 && iz >= 0 && iz < g.D && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
          const long long pix = inside ? (((static_cast<long long>(rn[i]) * g.D + iz) * g.H + ih) * g.W + iw) : 0;
          if (g.x_vec) {
            const bool v = inside && c < g.C;
            cp_async_16(dst, v ? static_cast<const void*>(g.x + pix * g.C + c) : static_cast<const void*>(g.x),
                        v ? 16u : 0u);
          } else {
            uint32_t h[4] = {0u, 0u, 0u, 0u};
            if (inside) {
              const unsigned short* xs = reinterpret_cast<const unsigned short*>(g.x) + pix * g.C;
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const unsigned short val = (c + e < g.C) ? xs[c + e] : static_cast<unsigned short>(0);
                h[e >> 1] |= static_cast<uint32_t>(val) << ((e & 1) * 16);
              }
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                         "r"(h[3])
                         : "memory");
          }
        }
        if (!B_TMA) {
          // Gathered weights (pitch not 16-byte aligned): K-major [BN][64].
          const uint32_t sB_addr = sA_addr + Cfg::A_BYTES;
          const unsigned short* ws = reinterpret_cast<const unsigned short*>(g.w);
#pragma unroll 1
          for (int q = gt; q < BN * 8; q += CONV_GATHER_THREADS) {
            const int n = q >> 3;
            const int jj = q & 7;
            const int oc = w.nt * BN + n;
            const int ic0 = cb * 64 + jj * 8;
            uint32_t h[4] = {0u, 0u, 0u, 0u};
            if (oc < g.O) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const unsigned short val =
                    (ic0 + e < g.C) ? ws[conv_weight_offset(g, oc, tap, ic0 + e)] : static_cast<unsigned short>(0);
                h[e >> 1] |= static_cast<uint32_t>(val) << ((e & 1) * 16);
              }
            }
            const uint32_t dst = sB_addr + n * 128 + ((jj ^ (n & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                         "r"(h[3])
                         : "memory");
          }
        }
        if (fast) {
          // The hardware arrives once this thread's copies have landed; the
          // MMA thread fences the async proxy after its wait.
          cp_async_arrive_noinc(&full[s]);
        } else {
          // Ordinary st.shared writes (and any cp.async) complete here.
          cp_async_wait_all();
          fence_proxy_async_smem();
          mbar_arrive(&full[s]);
        }
        ++fills;
      }
    }
    // Never leave with copies in flight (also on the abort path).
    cp_async_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// Weight layout permutation (HBM-bound copy, one thread per element).
__global__ void permute_weights_kernel(int from, int to, int O, int C, int KD, int KH, int KW,
                                       const unsigned short* __restrict__ src, unsigned short* __restrict__ dst) {
  const long long total = static_cast<long long>(O) * C * KD * KH * KW;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // i enumerates the destination layout; decode (oc, kd, kh, kw, ic) from it.
    long long t = i;
    int oc, ic, kd, kh, kw;
    switch (to) {
      case 0:
      case 3:  // [KD][KH][KW][C][O]
        oc = static_cast<int>(t % O); t /= O;
        ic = static_cast<int>(t % C); t /= C;
        kw = static_cast<int>(t % KW); t /= KW;
        kh = static_cast<int>(t % KH); t /= KH;
        kd = static_cast<int>(t);
        break;
      case 1:
      case 4:  // [O][KD][KH][KW][C]
        ic = static_cast<int>(t % C); t /= C;
        kw = static_cast<int>(t % KW); t /= KW;
        kh = static_cast<int>(t % KH); t /= KH;
        kd = static_cast<int>(t % KD); t /= KD;
        oc = static_cast<int>(t);
        break;
      default:  // [O][C][KD][KH][KW]
        kw = static_cast<int>(t % KW); t /= KW;
        kh = static_cast<int>(t % KH); t /= KH;
        kd = static_cast<int>(t % KD); t /= KD;
        ic = static_cast<int>(t % C); t /= C;
        oc = static_cast<int>(t);
        break;
    }
    long long s;
    switch (from) {
      case 0:
      case 3: s = ((((static_cast<long long>(kd) * KH + kh) * KW + kw) * C + ic) * O) + oc; break;
      case 1:
      case 4: s = ((((static_cast<long long>(oc) * KD + kd) * KH + kh) * KW + kw) * C) + ic; break;
      default: s = ((((static_cast<long long>(oc) * C + ic) * KD + kd) * KH + kh) * KW) + kw; break;
    }
    dst[i] = src[s];
  }
}

}  // namespace mm4

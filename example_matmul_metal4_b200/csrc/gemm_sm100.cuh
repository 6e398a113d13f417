// Persistent warp-specialised GEMM for sm_100a: C = A * B (+ bias).
//
// Replaces the generated `matmul` kernel and the `reduce_sum_2` split-K
// reduction of the reference (Sources/matmul/matmul.swift:239-296, :298-311).
//
// CTA = 6 warps, one CTA per SM, persistent over work units:
//   warp 0     TMA producer: one elected lane streams A/B k-blocks (64 wide)
//              into a STAGES-deep ring of 128-byte-swizzled smem tiles.
//   warp 1     allocates TMEM; one elected lane issues tcgen05.mma
//              (M=128, N=BN, K=16 per instruction) into one of two TMEM
//              accumulators and commits each stage back to the producer.
//   warps 2-5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//              32*(w%4)..+31, one output row per thread), add bias, round to
//              fp16, store. With two accumulators the epilogue of one tile
//              overlaps the main loop of the next.
//
// Split-K (MODE_SPLITK*): a work unit is (k-split, tile). Each unit adds its
// fp32 partial into an L2-resident fp32 workspace with vector atomics, then
// bumps a per-tile arrival counter; the unit that arrives last reads the
// summed tile back, adds bias, writes the output and re-zeroes the workspace
// and counter, so the workspace is clean for the next launch. The vector
// reductions are fire-and-forget (red.global.add.v4.f32). The fp32
// partials never round-trip through fp16 (the reference keeps fp16 partials,
// matmul.swift:248, :298-311), and the K tail is applied exactly once (the
// reference applies it in every split, matmul.swift:266-277).
//
// K tails need no special code: TMA zero-fills coordinates past K, so a
// partial last k-block contributes zeros (replaces the dynamic_length_v op,
// matmul.swift:271-277 and README.md:50-52).
#pragma once

#include "mm4_ptx.cuh"

namespace mm4 {

enum GemmMode : int {
  MODE_DIRECT_F16 = 0,  // splits == 1: fp16 output + bias
  MODE_SPLITK_F16 = 1,  // splits > 1: workspace reduce, fp16 output + bias
  MODE_DIRECT_F32 = 2,  // splits == 1: fp32 output, no bias (K-shard partial)
  MODE_SPLITK_F32 = 3,  // splits > 1: workspace reduce, fp32 output, no bias
};

// Multi-GPU split-K: each rank runs the same plan on its own K shard; the
// ranks' fp32 partials meet in the epilogue over peer memory (one kernel per
// GPU, no separate collective). The split-K scratch stays rank-local; each
// rank's exchange buffer holds two staging halves (by run parity) of one
// slot per rank, and every other rank maps it. Per slice (a 128-row half
// tile x one split's row range):
//   1. on a rank that does not own the slice (the owner is the root, or
//      slice % world in the spread mode), the CTA that completes the slice's
//      rank-local sum pushes the rows into its own slot of the owner's
//      staging half for this run (peer stores, posted over NVLink as soon as
//      the rows are final), re-zeroes the scratch rows and raises
//      ready[slice][rank] on the owner;
//   2. the owner's CTA for the slice waits for the other ranks' flags, reads
//      their rows from its own staging (local memory) and its own rows from
//      its scratch, sums them in rank order, adds bias, rounds, stores the
//      rows into the root's C (and raises done[slice] on the root when it is
//      not the root itself); at its next launch it raises consumed[slice] on
//      every rank;
//   3. a rank overwrites its slot of a staging half (two runs later) only
//      after the owner consumed it; the root's launch ends once every slice
//      is in C.
// Cross-GPU traffic is peer stores (and C stores) plus release/acquire flags
// that carry the run index + 1 (no remote atomics, nothing to reset).
constexpr int MM4_MAX_GROUP = 8;
struct SplitKGroupArgs {
  int world;                     // ranks (<= 1: single GPU)
  int rank, root;
  int owner_mode;                // 0: the root owns every slice; 1: slice % world (spread)
  int num_slices;                // half tiles x splits
  unsigned long long epoch;      // run index, the same on every rank
  float* stage[MM4_MAX_GROUP];   // rank r's staging half for this run: [world slots][rows][ws_ld] fp32 (peer-mapped)
  long long slot_floats;         // floats per slot (one rank's partials)
  unsigned long long* ready[MM4_MAX_GROUP];     // rank r: [num_slices][world]
  unsigned long long* consumed[MM4_MAX_GROUP];  // rank r: [num_slices]
  unsigned long long* done;      // root: [num_slices]
  __half* c_root;                // root's C [M][N] fp16 (peer-mapped)
};

__device__ __forceinline__ int group_owner(const SplitKGroupArgs& g, int slice) {
  return g.owner_mode == 0 ? g.root : slice % g.world;
}

struct GemmArgs {
  int M, N, K;
  int num_m_tiles, num_n_tiles, num_tiles;
  int splits, kb_total, num_units;
  int group_m;            // raster: tiles are walked in groups of group_m M-tiles
  const __half* bias;     // [N] or null
  __half* C;              // [M][N] fp16 output (F16 modes)
  float* C32;             // [M][N] fp32 output (F32 modes)
  float* ws;              // [num_m_tiles*128][ws_ld] fp32, split-K only
  unsigned long long* counters;  // one arrival count per 128-row half tile, split-K only
  int ws_ld;
  int coop_finalize;      // split-K: all units co-resident (cooperative launch), slices finalized in parallel
  // Split-K, deterministic mode (0: off): split s stores its partial into
  // ws + s * det_split_floats instead of reducing it into ws, and the
  // finalize sums the splits in order, so every run gives the same bits.
  long long det_split_floats;
  // Output row map of the direct epilogue. 0: tile row r is output row
  // mt*128 + r (GEMM). 1: a tile is a rm_th x rm_tw rectangle of output
  // pixels of one (n, oz) plane (convolution with TMA-fed activations).
  // 2: tile rows are virtual pixels of rows rm_vw wide (output width plus
  // the filter's kw overhang); virtual pixel v is output pixel
  // (v / rm_vw) * rm_ow + v % rm_vw when v % rm_vw < rm_ow and
  // v / rm_vw < rm_vrows, otherwise it is not stored.
  int rowmap;
  int rm_tw, rm_th, rm_tiles_w, rm_tiles_h, rm_od, rm_oh, rm_ow;
  int rm_vw, rm_vrows;
  int* status;
  unsigned long long timeout_ns;
  SplitKGroupArgs grp;    // multi-GPU split-K (grp.world > 1), cooperative finalize only
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

// Split-K epilogue staging: per epilogue warp a 32 x 32 fp32 block, rows
// padded to 36 floats so both the row-wise writes and the transposed reads
// are free of bank conflicts.
constexpr int EPI_STAGE_LD = 36;
constexpr int EPI_STAGE_BYTES = 4 * 32 * EPI_STAGE_LD * 4;

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 512) ? 2 : (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int ACC_BUFS = (BN == 512) ? 1 : 2;  // TMEM has 512 fp32 columns
  static constexpr int TMEM_COLS = ACC_BUFS * BN;
  static constexpr int N_INSTR = BN < 256 ? BN : 256;    // UMMA N per instruction
  static constexpr int N_HALVES = BN / N_INSTR;
  static constexpr int B_BOX_N = BN < 256 ? BN : 256;    // K-major B: TMA box rows
  // ring + split-K staging + barriers/slots + alignment slack
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_STAGE_BYTES + 256 + 1024;
};

// Wait-site ids recorded with MM4_ERR_TIMEOUT.
enum : int {
  SITE_GEMM_PRODUCER_EMPTY = 1,
  SITE_GEMM_PRODUCER_DRAIN = 2,
  SITE_GEMM_MMA_TMEM_EMPTY = 3,
  SITE_GEMM_MMA_FULL = 4,
  SITE_GEMM_MMA_DRAIN = 5,
  SITE_GEMM_EPI_TMEM_FULL = 6,
  SITE_GEMM_EPI_TILE_RENDEZVOUS = 7,
  SITE_GEMM_GROUP_FLAGS = 8,
  SITE_GEMM_GROUP_DONE = 9,
  SITE_GEMM_GROUP_SCRATCH = 10,
};

struct GemmUnit {
  int mt, nt, tile, split, kb0, kb1;
};

__device__ __forceinline__ GemmUnit gemm_decode_unit(const GemmArgs& a, int u) {
  GemmUnit w;
  if (a.splits > 1) {
    // Split-K: N-tile-major, then split, then M-tile. With the grid at
    // splits * num_m_tiles CTAs (pairs) each one keeps its (split, M-tile)
    // and walks the N-tiles, so its A k-slab is re-read from L2 and the
    // reduction of one N-tile overlaps the main loop of the next; all units
    // of one N-tile run together and share their B k-slabs in L2.
    const int per_n = a.splits * a.num_m_tiles;
    w.nt = u / per_n;
    const int r = u - w.nt * per_n;
    w.split = r / a.num_m_tiles;
    w.mt = r - w.split * a.num_m_tiles;
  } else {
    // Grouped raster: walk group_m M-tiles down a column of N-tiles.
    w.split = 0;
    const int group_size = a.group_m * a.num_n_tiles;
    const int group = u / group_size;
    const int first_m = group * a.group_m;
    const int gm = min(a.num_m_tiles - first_m, a.group_m);
    const int r = u - group * group_size;
    w.mt = first_m + r % gm;
    w.nt = r / gm;
  }
  w.tile = w.mt * a.num_n_tiles + w.nt;
  w.kb0 = static_cast<int>((static_cast<long long>(w.split) * a.kb_total) / a.splits);
  w.kb1 = static_cast<int>((static_cast<long long>(w.split + 1) * a.kb_total) / a.splits);
  return w;
}

// Multi-GPU split-K finalize of one slice (see SplitKGroupArgs), run by the
// 128 epilogue threads of the CTA that completed the slice's rank-local sum.
template <int BN>
__device__ __forceinline__ void group_finalize(const GemmArgs& args, int ctr_tile, int split, int row_base,
                                               int col0, int r_begin, int r_end, int ethread, const Watchdog& wd) {
  const SplitKGroupArgs& g = args.grp;
  const int slice = ctr_tile * args.splits + split;
  const int owner = group_owner(g, slice);
  const unsigned long long tag = g.epoch + 1ull;
  constexpr int TPR = BN / 4;     // threads per row (float4 each)
  constexpr int RPI = 128 / TPR;  // rows per iteration
  const int tr = ethread / TPR;
  const int gc = col0 + (ethread % TPR) * 4;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // 1. A rank that does not own the slice pushes it into its slot of the
  //    owner's staging half (free: group_unit_start checked it): rows
  //    scratch -> owner, scratch re-zeroed, flag on the owner. The owner
  //    reads its own rows straight from its scratch in step 2.
  if (owner != g.rank) {
    float* stage = g.stage[owner] + g.rank * g.slot_floats;
    for (int rr0 = r_begin + tr; rr0 < r_end; rr0 += 4 * RPI) {
      float4 v[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int rr = rr0 + b * RPI;
        if (rr < r_end) v[b] = __ldcg(reinterpret_cast<const float4*>(args.ws + static_cast<size_t>(row_base + rr) * args.ws_ld + gc));
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int rr = rr0 + b * RPI;
        if (rr >= r_end) break;
        const size_t off = static_cast<size_t>(row_base + rr) * args.ws_ld + gc;
        __stcg(reinterpret_cast<float4*>(args.ws + off), zero);
        __stcg(reinterpret_cast<float4*>(stage + off), v[b]);
      }
    }
    fence_acq_rel_sys();    // this thread's peer stores, before the barrier
    named_barrier(1, 128);  // orders every thread's stores before the release
    if (ethread == 0) st_release_sys_u64(g.ready[owner] + static_cast<size_t>(slice) * g.world + g.rank, tag);
    return;
  }
  // 2. Owner: one thread per other rank polls that rank's flag; then every
  //    rank's rows (its slot of this rank's staging, this rank's own from its
  //    scratch; all loads of a row batch in flight at once), summed in rank
  //    order, bias, fp16 into the root's C; this rank's scratch rows
  //    re-zeroed.
  const bool ok = ethread >= g.world || ethread == g.rank ||
                  wait_all_ge_sys_u64(g.ready[g.rank] + static_cast<size_t>(slice) * g.world + ethread, 1, tag, wd,
                                      SITE_GEMM_GROUP_FLAGS);
  if (!named_barrier_and(1, 128, ok)) return;
  float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
  if (args.bias != nullptr) {
    if (gc + 0 < args.N) b0 = __half2float(args.bias[gc + 0]);
    if (gc + 1 < args.N) b1 = __half2float(args.bias[gc + 1]);
    if (gc + 2 < args.N) b2 = __half2float(args.bias[gc + 2]);
    if (gc + 3 < args.N) b3 = __half2float(args.bias[gc + 3]);
  }
  const bool vec = (args.N & 3) == 0 && (reinterpret_cast<uintptr_t>(g.c_root) & 7u) == 0;
  constexpr int RB = 2;  // rows per batch
  for (int rr0 = r_begin + tr; rr0 < r_end; rr0 += RB * RPI) {
    // Every (source, row) load of a batch is issued before any is used: one
    // NVLink round trip per batch, not one per source.
    float4 v[MM4_MAX_GROUP][RB];
#pragma unroll
    for (int src = 0; src < MM4_MAX_GROUP; ++src) {
#pragma unroll
      for (int b = 0; b < RB; ++b) {
        const int rr = rr0 + b * RPI;
        if (src < g.world && rr < r_end) {
          const float* from = src == g.rank ? args.ws : g.stage[g.rank] + src * g.slot_floats;
          v[src][b] = __ldcg(reinterpret_cast<const float4*>(from + static_cast<size_t>(row_base + rr) * args.ws_ld + gc));
        }
      }
    }
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      const int rr = rr0 + b * RPI;
      if (rr < r_end) __stcg(reinterpret_cast<float4*>(args.ws + static_cast<size_t>(row_base + rr) * args.ws_ld + gc), zero);
    }
    float4 acc[RB];
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      acc[b] = v[0][b];
#pragma unroll
      for (int src = 1; src < MM4_MAX_GROUP; ++src) {
        if (src < g.world) {
          acc[b].x += v[src][b].x;
          acc[b].y += v[src][b].y;
          acc[b].z += v[src][b].z;
          acc[b].w += v[src][b].w;
        }
      }
    }
#pragma unroll
    for (int b = 0; b < RB; ++b) {
      const int rr = rr0 + b * RPI;
      const int grow = row_base + rr;
      if (rr >= r_end || grow >= args.M) continue;
      __half* c = g.c_root + static_cast<size_t>(grow) * args.N + gc;
      const float o0 = acc[b].x + b0, o1 = acc[b].y + b1, o2 = acc[b].z + b2, o3 = acc[b].w + b3;
      if (vec && gc + 4 <= args.N) {
        uint2 pk;
        pk.x = pack_half2(o0, o1);
        pk.y = pack_half2(o2, o3);
        *reinterpret_cast<uint2*>(c) = pk;
      } else {
        if (gc + 0 < args.N) c[0] = __float2half_rn(o0);
        if (gc + 1 < args.N) c[1] = __float2half_rn(o1);
        if (gc + 2 < args.N) c[2] = __float2half_rn(o2);
        if (gc + 3 < args.N) c[3] = __float2half_rn(o3);
      }
    }
  }
  // 3. The root may finish once its C rows are in (the CTA barrier orders
  //    every thread's stores before the release). The ranks learn that their
  //    staging was consumed from the next launch (group_unit_start).
  if (g.rank != g.root) {
    named_barrier(1, 128);
    if (ethread == 0) st_release_sys_u64(g.done + slice, tag);
  }
}

// Multi-GPU split-K, at the start of a unit, while the epilogue warps wait for
// the main loop (off the critical path):
//   - the slice this CTA owned in the previous run was read by then (the
//     launch boundary orders those loads): tell every rank it may reuse that
//     staging half (consumed = previous run index + 1);
//   - this CTA's staging half for this run was last written two runs ago:
//     wait until its owner has consumed it.
template <bool PAIR>
__device__ __forceinline__ bool group_unit_start(const GemmArgs& args, const GemmUnit& w, uint32_t rank,
                                                 int ethread, const Watchdog& wd) {
  const SplitKGroupArgs& g = args.grp;
  const int ct = PAIR ? 2 * w.tile + static_cast<int>(rank) : w.tile;
  const int slice = ct * args.splits + w.split;
  if (g.epoch >= 1 && group_owner(g, slice) == g.rank && ethread < g.world)
    st_release_sys_u64(g.consumed[ethread] + slice, g.epoch);
  const bool ok = g.epoch < 2 || ethread != 0 ||
                  wait_all_ge_sys_u64(g.consumed[g.rank] + slice, 1, g.epoch - 1ull, wd, SITE_GEMM_GROUP_SCRATCH);
  return named_barrier_and(1, 128, ok);
}

// All four epilogue warps agree on whether to proceed (every thread reaches
// the two named barriers whatever its own wait returned, so none can hang).
__device__ __forceinline__ bool epi_consensus(bool ok, int q, int lane, volatile int* s_vote) {
  const int v = __all_sync(0xffffffffu, ok) ? 1 : 0;
  if (lane == 0) s_vote[q] = v;
  named_barrier(1, 128);
  const bool all = (s_vote[0] & s_vote[1] & s_vote[2] & s_vote[3]) != 0;
  named_barrier(1, 128);
  return all;
}


// ---------------------------------------------------------------------------
// MMA issuer role (one elected thread). Consumes `kb1 - kb0` ring stages per
// work unit into one of two TMEM accumulators. PROXY_FENCE is set when the
// ring is filled by ordinary (generic-proxy) stores instead of TMA.
// ---------------------------------------------------------------------------
template <int BN, bool A_MN, bool B_MN, int STAGES, int STAGE_BYTES, int A_BYTES, bool PROXY_FENCE>
__device__ __forceinline__ void mma_role(const GemmArgs& args, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                         uint64_t* tmem_full, uint64_t* tmem_empty, uint64_t* drain,
                                         uint32_t tmem_base, const Watchdog& wd) {
  using Cfg = GemmCfg<BN>;
  constexpr uint32_t IDESC = idesc_f16_f32(GEMM_BM, Cfg::N_INSTR, A_MN, B_MN);
  // Byte offset of the second N half of the B tile (BN = 512).
  constexpr uint32_t B_HALF = B_MN ? (Cfg::N_INSTR / 64) * 8192u : Cfg::N_INSTR * 128u;
  uint32_t consumed = 0;
  uint32_t tiles_done = 0;
  bool ok = true;
  for (int u = blockIdx.x; u < args.num_units && ok; u += gridDim.x) {
    const GemmUnit w = gemm_decode_unit(args, u);
    const uint32_t acc = tiles_done % Cfg::ACC_BUFS;
    const uint32_t aph = (tiles_done / Cfg::ACC_BUFS) & 1u;
    if (!mbar_wait(&tmem_empty[acc], aph ^ 1u, wd, SITE_GEMM_MMA_TMEM_EMPTY)) break;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + acc * BN;
    for (int kb = w.kb0; kb < w.kb1; ++kb) {
      const int s = static_cast<int>(consumed % STAGES);
      const uint32_t ph = (consumed / STAGES) & 1u;
      if (!mbar_wait(&full[s], ph, wd, SITE_GEMM_MMA_FULL)) {
        ok = false;
        break;
      }
      if (PROXY_FENCE) fence_proxy_async_smem();
      tc_fence_after();
      const uint32_t a_base = smem_u32(ring + s * STAGE_BYTES);
      const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
        const uint64_t adesc =
            A_MN ? sw128_desc(a_base + kk * 2048, 8192, 1024) : sw128_desc(a_base + kk * 32, 16, 1024);
#pragma unroll
        for (int hh = 0; hh < Cfg::N_HALVES; ++hh) {
          const uint32_t bb = b_base + hh * B_HALF;
          const uint64_t bdesc = B_MN ? sw128_desc(bb + kk * 2048, 8192, 1024) : sw128_desc(bb + kk * 32, 16, 1024);
          umma_f16_ss(d_tmem + hh * Cfg::N_INSTR, adesc, bdesc, IDESC, (kb > w.kb0 || kk > 0) ? 1u : 0u);
        }
      }
      umma_commit(&empty[s]);
      ++consumed;
    }
    if (!ok) break;
    umma_commit(&tmem_full[acc]);
    ++tiles_done;
  }
  // All issued MMAs must finish before TMEM is released.
  umma_commit(drain);
  mbar_wait(drain, 0, wd, SITE_GEMM_MMA_DRAIN);
}

// ---------------------------------------------------------------------------
// Epilogue role (warps 2-5 of the CTA, 128 threads: thread 64 + i).
// ---------------------------------------------------------------------------
// PAIR: the CTA is one half (rank 0 = leader, 1 = peer) of a 2-CTA cluster
// computing 256-row tiles with cta_group::2; its accumulator holds rows
// rank*128..+127 of the tile, and it hands TMEM back to the leader's MMA
// thread through the leader's tmem_empty barrier.
template <int BN, int MODE, bool PAIR = false>
__device__ __forceinline__ void epilogue_role(const GemmArgs& args, uint64_t* tmem_full, uint64_t* tmem_empty,
                                              uint32_t tmem_base, volatile int* s_vote, volatile int* s_last,
                                              float* stage, const Watchdog& wd, int warp, int lane,
                                              uint32_t rank = 0) {
  constexpr bool SPLITK = (MODE == MODE_SPLITK_F16 || MODE == MODE_SPLITK_F32);
  constexpr bool OUT_F32 = (MODE == MODE_DIRECT_F32 || MODE == MODE_SPLITK_F32);
  constexpr int ACC_BUFS = (BN == 512) ? 1 : 2;
  constexpr int TILE_M = PAIR ? 2 * GEMM_BM : GEMM_BM;
  const int q = warp & 3;  // TMEM lane quarter this warp may access
  const int row_in_tile = q * 32 + lane;
  const int ethread = threadIdx.x - 64;  // 0..127
  const int u0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ustep = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  uint32_t tiles_done = 0;
  for (int u = u0; u < args.num_units; u += ustep) {
    const GemmUnit w = gemm_decode_unit(args, u);
    const uint32_t acc = tiles_done % ACC_BUFS;
    const uint32_t aph = (tiles_done / ACC_BUFS) & 1u;
    if constexpr (SPLITK) {
      if (args.grp.world > 1 && !group_unit_start<PAIR>(args, w, rank, ethread, wd)) break;
    }
    bool ok = mbar_wait(&tmem_full[acc], aph, wd, SITE_GEMM_EPI_TMEM_FULL);
    if (!epi_consensus(ok, q, lane, s_vote)) break;
    tc_fence_after();
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
    const int row_base = w.mt * TILE_M + static_cast<int>(rank) * GEMM_BM;  // this CTA's first tile row
    int row = row_base + row_in_tile;
    bool row_ok = row < args.M;
    if (args.rowmap == 1) {
      int t = w.mt;
      const int twi = t % args.rm_tiles_w;
      t /= args.rm_tiles_w;
      const int thi = t % args.rm_tiles_h;
      t /= args.rm_tiles_h;
      const int oz = t % args.rm_od;
      const int n = t / args.rm_od;
      const int oh = thi * args.rm_th + row_in_tile / args.rm_tw;
      const int ow = twi * args.rm_tw + row_in_tile % args.rm_tw;
      row_ok = oh < args.rm_oh && ow < args.rm_ow;
      row = ((n * args.rm_od + oz) * args.rm_oh + oh) * args.rm_ow + ow;
    } else if (args.rowmap == 2) {
      const int xv = row % args.rm_vw;
      const int line = row / args.rm_vw;
      row_ok = xv < args.rm_ow && line < args.rm_vrows;
      row = line * args.rm_ow + xv;
    }
    const int col0 = w.nt * BN;

    // Split-K: each split starts at a different 32-column chunk, so the
    // splits of a tile do not all reduce into the same lines at once.
    const int rot = SPLITK ? w.split & (BN / 32 - 1) : 0;
#pragma unroll 1
    for (int ci = 0; ci < BN / 32; ++ci) {
      const int c = (ci + rot) & (BN / 32 - 1);
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r);
      tmem_ld_wait();
      if (ci == BN / 32 - 1) {
        tc_fence_before();
        if (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[acc]), 0));
        else
          mbar_arrive(&tmem_empty[acc]);
      }
      const int cbase = col0 + c * 32;
      if constexpr (SPLITK) {
        // Transpose the warp's 32 rows x 32 columns through shared memory so
        // that each red instruction covers four whole 128-byte rows (eight
        // lanes per row) instead of 32 half-used sectors.
        float* wst = stage + q * (32 * EPI_STAGE_LD);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<uint4*>(wst + lane * EPI_STAGE_LD + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        __syncwarp();
        const int sub_r = lane >> 3;
        const int sub_c = (lane & 7) * 4;
        float* dst = args.ws + static_cast<size_t>(row_base + q * 32 + sub_r) * args.ws_ld + cbase + sub_c;
        if (args.det_split_floats != 0) {
          dst += w.split * args.det_split_floats;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            __stcg(reinterpret_cast<float4*>(dst + static_cast<size_t>(k * 4) * args.ws_ld),
                   *reinterpret_cast<const float4*>(wst + (k * 4 + sub_r) * EPI_STAGE_LD + sub_c));
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 v = *reinterpret_cast<const float4*>(wst + (k * 4 + sub_r) * EPI_STAGE_LD + sub_c);
            red_add_v4_f32(dst + static_cast<size_t>(k * 4) * args.ws_ld, v.x, v.y, v.z, v.w);
          }
        }
        __syncwarp();
      } else if constexpr (OUT_F32) {
        if (row_ok) {
          float* dst = args.C32 + static_cast<size_t>(row) * args.N + cbase;
          const bool vec = (cbase + 32 <= args.N) && ((args.N & 3) == 0) &&
                           ((reinterpret_cast<uintptr_t>(args.C32) & 15u) == 0);
          if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
            for (int j = 0; j < 32; ++j)
              if (cbase + j < args.N) dst[j] = __uint_as_float(r[j]);
          }
        }
      } else {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (args.bias != nullptr) {
          if (cbase + 32 <= args.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += __half2float(args.bias[cbase + j]);
          } else {
            for (int j = 0; j < 32; ++j)
              if (cbase + j < args.N) v[j] += __half2float(args.bias[cbase + j]);
          }
        }
        if (row_ok) {
          __half* dst = args.C + static_cast<size_t>(row) * args.N + cbase;
          const bool vec = (cbase + 32 <= args.N) && ((args.N & 7) == 0) &&
                           ((reinterpret_cast<uintptr_t>(args.C) & 15u) == 0);
          if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 pk;
              pk.x = pack_half2(v[j], v[j + 1]);
              pk.y = pack_half2(v[j + 2], v[j + 3]);
              pk.z = pack_half2(v[j + 4], v[j + 5]);
              pk.w = pack_half2(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4*>(dst + j) = pk;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (cbase + j < args.N) dst[j] = __float2half_rn(v[j]);
          }
        }
      }
    }

    if constexpr (SPLITK) {
      // Publish this unit's partial, then count arrivals for the tile. The
      // 64-bit arrival counters only grow: the launch's arrivals for a tile
      // are the values [e * splits, (e + 1) * splits) for some e, so no reset
      // is needed between launches.
      __threadfence();
      named_barrier(1, 128);
      const int ctr_tile = PAIR ? 2 * w.tile + static_cast<int>(rank) : w.tile;  // per 128-row half
      unsigned long long* arrive_ctr = &args.counters[ctr_tile];
      if (ethread == 0) {
        const unsigned long long splits = static_cast<unsigned long long>(args.splits);
        const unsigned long long prev = atomicAdd(arrive_ctr, 1ull);
        if (!args.coop_finalize) {
          *s_last = (prev % splits == splits - 1) ? 1 : 0;
        } else {
          // All units are co-resident (cooperative launch): wait, bounded,
          // until every split of this tile has published its partial.
          const unsigned long long target = (prev / splits + 1) * splits;
          int ok = 1;
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          while (*reinterpret_cast<volatile unsigned long long*>(arrive_ctr) < target) {
            if ((++spins & 63u) == 0 &&
                (aborted(wd.status) || globaltimer_ns() - t0 > wd.limit_ns)) {
              record_error(wd.status, MM4_ERR_TIMEOUT, SITE_GEMM_EPI_TILE_RENDEZVOUS);
              ok = 0;
              break;
            }
          }
          *s_last = ok;
        }
      }
      named_barrier(1, 128);
      int r_begin = 0, r_end = 0;  // tile rows this CTA finalizes
      if (*s_last) {
        if (args.coop_finalize) {
          r_begin = (w.split * GEMM_BM) / args.splits;
          r_end = ((w.split + 1) * GEMM_BM) / args.splits;
        } else {
          r_end = GEMM_BM;
        }
      }
      if (args.grp.world > 1) {
        // Multi-GPU: the rank-local sum of this slice joins the other ranks'.
        if (*s_last) {
          __threadfence();
          group_finalize<BN>(args, ctr_tile, w.split, row_base, col0, r_begin, r_end, ethread, wd);
        }
        r_end = r_begin;
      }
      if (r_end > r_begin) {
        __threadfence();
        // Sum is complete: add bias, round, store; re-zero the workspace rows.
        constexpr int TPR = BN / 4;          // threads per row (float4 each)
        constexpr int RPI = 128 / TPR;       // rows per iteration
        const int tr = ethread / TPR;
        const int tc = (ethread % TPR) * 4;
        const int gc = col0 + tc;
        float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        if (!OUT_F32 && args.bias != nullptr) {
          if (gc + 0 < args.N) b0 = __half2float(args.bias[gc + 0]);
          if (gc + 1 < args.N) b1 = __half2float(args.bias[gc + 1]);
          if (gc + 2 < args.N) b2 = __half2float(args.bias[gc + 2]);
          if (gc + 3 < args.N) b3 = __half2float(args.bias[gc + 3]);
        }
        // Up to four rows per thread in flight: all loads first, then the
        // stores, so the L2 round trips overlap.
        for (int rr0 = r_begin + tr; rr0 < r_end; rr0 += 4 * RPI) {
          float4 s4v[4];
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
            const int rr = rr0 + bb * RPI;
            if (rr >= r_end) continue;
            const float* src = args.ws + static_cast<size_t>(row_base + rr) * args.ws_ld + gc;
            if (args.det_split_floats != 0) {
              // The splits' partials, summed in split order.
              float4 acc = __ldcg(reinterpret_cast<const float4*>(src));
              for (int sp = 1; sp < args.splits; ++sp) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(src + sp * args.det_split_floats));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
              }
              s4v[bb] = acc;
            } else {
              s4v[bb] = __ldcg(reinterpret_cast<const float4*>(src));
            }
          }
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
          const int rr = rr0 + bb * RPI;
          if (rr >= r_end) break;
          const int grow = row_base + rr;
          if (args.det_split_floats == 0)
            __stcg(reinterpret_cast<float4*>(args.ws + static_cast<size_t>(grow) * args.ws_ld + gc),
                   make_float4(0.f, 0.f, 0.f, 0.f));
          if (grow >= args.M) continue;
          const float4 s4 = s4v[bb];
          const float o0 = s4.x + b0, o1 = s4.y + b1, o2 = s4.z + b2, o3 = s4.w + b3;
          if constexpr (OUT_F32) {
            float* dst = args.C32 + static_cast<size_t>(grow) * args.N + gc;
            if (gc + 4 <= args.N && (args.N & 3) == 0 && (reinterpret_cast<uintptr_t>(args.C32) & 15u) == 0) {
              *reinterpret_cast<float4*>(dst) = make_float4(o0, o1, o2, o3);
            } else {
              if (gc + 0 < args.N) dst[0] = o0;
              if (gc + 1 < args.N) dst[1] = o1;
              if (gc + 2 < args.N) dst[2] = o2;
              if (gc + 3 < args.N) dst[3] = o3;
            }
          } else {
            __half* dst = args.C + static_cast<size_t>(grow) * args.N + gc;
            if (gc + 4 <= args.N && (args.N & 3) == 0 && (reinterpret_cast<uintptr_t>(args.C) & 7u) == 0) {
              uint2 pk;
              pk.x = pack_half2(o0, o1);
              pk.y = pack_half2(o2, o3);
              *reinterpret_cast<uint2*>(dst) = pk;
            } else {
              if (gc + 0 < args.N) dst[0] = __float2half_rn(o0);
              if (gc + 1 < args.N) dst[1] = __float2half_rn(o1);
              if (gc + 2 < args.N) dst[2] = __float2half_rn(o2);
              if (gc + 3 < args.N) dst[3] = __float2half_rn(o3);
            }
          }
          }
        }
      }
    }
    ++tiles_done;
  }
  if constexpr (SPLITK) {
    // Multi-GPU root: the launch ends only once every slice of C is written.
    // Slices other ranks own; spread over every epilogue thread of every root
    // CTA, one flag each.
    if (args.grp.world > 1 && args.grp.rank == args.grp.root && args.grp.owner_mode != 0) {
      const int stride = static_cast<int>(gridDim.x) * 128;
      for (int sl = static_cast<int>(blockIdx.x) + ethread * static_cast<int>(gridDim.x); sl < args.grp.num_slices;
           sl += stride) {
        if (group_owner(args.grp, sl) == args.grp.rank) continue;
        if (aborted(wd.status) ||
            !wait_all_ge_sys_u64(args.grp.done + sl, 1, args.grp.epoch + 1ull, wd, SITE_GEMM_GROUP_DONE))
          break;
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int MODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* ring = smem;
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + EPI_STAGE_BYTES);
  uint64_t* full = bars;                  // [STAGES]
  uint64_t* empty = bars + STAGES;        // [STAGES]
  uint64_t* tmem_full = bars + 2 * STAGES;   // [2]
  uint64_t* tmem_empty = tmem_full + 2;      // [2]
  uint64_t* drain = tmem_empty + 2;          // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_vote = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [4]
  volatile int* s_last = s_vote + 4;                                       // [1]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Watchdog wd{args.status, args.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
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
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      uint32_t fills = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < args.num_units && ok; u += gridDim.x) {
        const GemmUnit w = gemm_decode_unit(args, u);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          const int s = static_cast<int>(fills % STAGES);
          const uint32_t ph = (fills / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, wd, SITE_GEMM_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* sA = ring + s * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
          const int k0 = kb * GEMM_BK;
          if (!A_MN) {
            tma_load_2d(&tmA, &full[s], sA, k0, w.mt * GEMM_BM);
          } else {
            tma_load_2d(&tmA, &full[s], sA, w.mt * GEMM_BM, k0);
            tma_load_2d(&tmA, &full[s], sA + 8192, w.mt * GEMM_BM + 64, k0);
          }
          if (!B_MN) {
#pragma unroll
            for (int j = 0; j < BN / Cfg::B_BOX_N; ++j)
              tma_load_2d(&tmB, &full[s], sB + j * Cfg::B_BOX_N * 128, k0, w.nt * BN + j * Cfg::B_BOX_N);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(&tmB, &full[s], sB + j * 8192, w.nt * BN + 64 * j, k0);
          }
          ++fills;
        }
      }
      // Never leave with copies in flight: wait for the last fill of each stage.
      const uint32_t first = fills > STAGES ? fills - STAGES : 0u;
      for (uint32_t i = first; i < fills; ++i) {
        if (!mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, wd, SITE_GEMM_PRODUCER_DRAIN)) break;
      }
    }
  } else if (warp == 1) {
    if (elect_one())
      mma_role<BN, A_MN, B_MN, STAGES, Cfg::STAGE_BYTES, Cfg::A_BYTES, false>(args, ring, full, empty, tmem_full,
                                                                           tmem_empty, drain, tmem_base, wd);
  } else {
    epilogue_role<BN, MODE>(args, tmem_full, tmem_empty, tmem_base, s_vote, s_last, epi_stage, wd, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace mm4

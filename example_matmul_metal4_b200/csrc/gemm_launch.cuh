// Host-side launch of the GEMM kernel instances, shared by the GEMM entry
// points (mm4_gemm.cu) and the allocation-free split-K entry (mm4_noalloc.cu).
#pragma once

#include <cstring>

#include "gemm_sm100.cuh"
#include "gemm_sm100_pair.cuh"
#include "mm4_gemm_plan.h"
#include "mm4_internal.h"

namespace mm4 {

// TMA descriptors of A and B for the plan's tile shape.
inline mm4_status gemm_build_maps(const mm4_gemm_plan* p, const void* A, const void* B, CUtensorMap* ta,
                                  CUtensorMap* tb) {
  const mm4_gemm_desc& d = p->d;
  mm4_status rc;
  if (!d.transpose_left) {  // A [M][K]: box 64(K) x 128(M)
    const uint64_t dims[2] = {static_cast<uint64_t>(d.K), static_cast<uint64_t>(d.M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.K) * 2};
    const uint32_t box[2] = {64, 128};
    rc = encode_tiled(ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {  // A [K][M]: box 64(M) x 64(K), two per stage
    const uint64_t dims[2] = {static_cast<uint64_t>(d.M), static_cast<uint64_t>(d.K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.M) * 2};
    const uint32_t box[2] = {64, 64};
    rc = encode_tiled(ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc != MM4_OK) return rc;
  if (d.transpose_right) {  // B [N][K]: box 64(K) x rows(N)
    const uint64_t dims[2] = {static_cast<uint64_t>(d.K), static_cast<uint64_t>(d.N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.K) * 2};
    const uint32_t rows = p->pair ? 128u : static_cast<uint32_t>(p->bn < 256 ? p->bn : 256);
    const uint32_t box[2] = {64, rows};
    rc = encode_tiled(tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {  // B [K][N]: box 64(N) x 64(K)
    const uint64_t dims[2] = {static_cast<uint64_t>(d.N), static_cast<uint64_t>(d.K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.N) * 2};
    const uint32_t box[2] = {64, 64};
    rc = encode_tiled(tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  return rc;
}

// Launches `kern` (grid 1-D) with an optional 2-CTA cluster and an optional
// cooperative guarantee (all CTAs co-resident). A cooperative launch that the
// device refuses is retried without it, with args.coop_finalize cleared.
template <typename Kern>
mm4_status gemm_launch(Kern kern, int smem, int grid, bool pair, const CUtensorMap& ta, const CUtensorMap& tb,
                       const GemmArgs& args, cudaStream_t st) {
  mm4_status rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (rc != MM4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pair) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 2;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (args.coop_finalize) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, args);
  if (e != cudaSuccess && args.coop_finalize) {
    cudaGetLastError();
    GemmArgs fallback = args;
    fallback.coop_finalize = 0;
    cfg.numAttrs = pair ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, ta, tb, fallback);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemm kernel launch");
  return MM4_OK;
}

template <int BN, bool AMN, bool BMN, int MODE>
mm4_status gemm_launch_instance(bool pair, int grid, const CUtensorMap& ta, const CUtensorMap& tb,
                                const GemmArgs& args, cudaStream_t st) {
  if (pair) {
    if constexpr (BN == 256 || BN == 512)
      return gemm_launch(gemm_sm100_pair_kernel<BN, AMN, BMN, MODE>, PairCfg<BN>::SMEM_BYTES, grid, true, ta, tb,
                         args, st);
    return fail(MM4_ERR_UNSUPPORTED, "no CTA-pair GEMM instance for BN=%d", BN);
  }
  return gemm_launch(gemm_sm100_kernel<BN, AMN, BMN, MODE>, GemmCfg<BN>::SMEM_BYTES, grid, false, ta, tb, args, st);
}

template <int BN, bool AMN, bool BMN>
mm4_status gemm_launch_mode(int mode, bool pair, int grid, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& args, cudaStream_t st) {
  if constexpr (BN == 512) {  // BN = 512 is a split-K-only tile
    if (mode == MODE_SPLITK_F16)
      return gemm_launch_instance<BN, AMN, BMN, MODE_SPLITK_F16>(pair, grid, ta, tb, args, st);
    return gemm_launch_instance<BN, AMN, BMN, MODE_SPLITK_F32>(pair, grid, ta, tb, args, st);
  } else {
    switch (mode) {
      case MODE_DIRECT_F16: return gemm_launch_instance<BN, AMN, BMN, MODE_DIRECT_F16>(pair, grid, ta, tb, args, st);
      case MODE_SPLITK_F16: return gemm_launch_instance<BN, AMN, BMN, MODE_SPLITK_F16>(pair, grid, ta, tb, args, st);
      case MODE_DIRECT_F32: return gemm_launch_instance<BN, AMN, BMN, MODE_DIRECT_F32>(pair, grid, ta, tb, args, st);
      default: return gemm_launch_instance<BN, AMN, BMN, MODE_SPLITK_F32>(pair, grid, ta, tb, args, st);
    }
  }
}

template <int BN>
mm4_status gemm_launch_majors(bool amn, bool bmn, int mode, bool pair, int grid, const CUtensorMap& ta,
                              const CUtensorMap& tb, const GemmArgs& args, cudaStream_t st) {
  if (!amn && !bmn) return gemm_launch_mode<BN, false, false>(mode, pair, grid, ta, tb, args, st);
  if (!amn && bmn) return gemm_launch_mode<BN, false, true>(mode, pair, grid, ta, tb, args, st);
  if (amn && !bmn) return gemm_launch_mode<BN, true, false>(mode, pair, grid, ta, tb, args, st);
  return gemm_launch_mode<BN, true, true>(mode, pair, grid, ta, tb, args, st);
}

// Fills the shape part of GemmArgs from the plan.
inline void gemm_plan_args(const mm4_gemm_plan* p, GemmArgs* a) {
  a->M = p->d.M;
  a->N = p->d.N;
  a->K = p->d.K;
  a->num_m_tiles = p->num_m_tiles;
  a->num_n_tiles = p->num_n_tiles;
  a->num_tiles = p->num_tiles;
  a->splits = p->splits;
  a->kb_total = p->kb_total;
  a->num_units = p->num_tiles * p->splits;
  a->group_m = 8;
  a->ws_ld = p->num_n_tiles * p->bn;
}

// Grid for the plan: one CTA (or CTA pair) per work unit, at most one per SM.
// Split-K plans get one CTA (pair) per (split, M-tile) when that fits, so each
// walks the N-tiles of its k-slab (see gemm_decode_unit).
inline int gemm_grid(const mm4_gemm_plan* p, int num_units, int sm_count) {
  int slots = p->pair ? sm_count / 2 : sm_count;
  int want = num_units;
  if (p->splits > 1) want = std::min(want, p->splits * p->num_m_tiles);
  const int n = std::min(want, slots);
  return p->pair ? 2 * n : n;
}

inline mm4_status gemm_dispatch(const mm4_gemm_plan* p, int mode, const CUtensorMap& ta, const CUtensorMap& tb,
                                const GemmArgs& args, int grid, cudaStream_t st) {
  const bool amn = p->d.transpose_left != 0;
  const bool bmn = p->d.transpose_right == 0;
  if (p->bn == 512) return gemm_launch_majors<512>(amn, bmn, mode, p->pair, grid, ta, tb, args, st);
  if (p->bn == 256) return gemm_launch_majors<256>(amn, bmn, mode, p->pair, grid, ta, tb, args, st);
  return gemm_launch_majors<128>(amn, bmn, mode, false, grid, ta, tb, args, st);
}

}  // namespace mm4

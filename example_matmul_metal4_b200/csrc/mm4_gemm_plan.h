// Host-side GEMM plan record shared by the GEMM entry points.
#pragma once

#include <cstddef>

#include <cuda_runtime.h>

#include "mm4.h"

struct mm4_gemm_plan {
  mm4_gemm_desc d;
  bool tensor_core;  // false: reduced-alignment SIMT kernel
  bool pair;         // 2-CTA cluster kernel (cta_group::2), 256-row tiles
  int bn;            // tile N (per CTA for one-CTA tiles, per pair otherwise)
  int splits;
  int kb_total;
  int num_m_tiles, num_n_tiles, num_tiles;
  size_t ws_bytes;
  size_t ws_counter_offset;
  long long det_split_floats;  // split-K deterministic mode: floats per split's partial (0: off)
  char name[96];
};

namespace mm4 {
struct SplitKGroupArgs;
// Tensor-core GEMM launch (mm4_gemm.cu): fp16 C with bias, or fp32 C32 partial
// when C32 is set; `grp` joins a multi-GPU split-K group.
mm4_status gemm_run_tc(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias, void* C, float* C32,
                       void* ws, size_t ws_bytes, cudaStream_t st, const SplitKGroupArgs* grp = nullptr);
}  // namespace mm4

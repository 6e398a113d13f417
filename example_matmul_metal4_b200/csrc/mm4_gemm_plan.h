// Host-side GEMM plan record shared by the GEMM entry points.
#pragma once

#include <cstddef>

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
  char name[96];
};

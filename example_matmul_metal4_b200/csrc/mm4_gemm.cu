// GEMM plans and dispatch: the sm_100a replacement for the reference's
// runtime-generated matmul kernel + reduce_sum_2 dispatch
// (Sources/matmul/matmul.swift:18-329 generator, :345-511 run()).
//
// The reference compiles one MSL kernel per (shape, tile, options) at run
// time; mm4 instead selects one of a fixed set of template instances
// (BN x operand majors x epilogue mode) when the plan is created.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <new>

#include "gemm_simt.cuh"
#include "gemm_sm100.cuh"
#include "mm4_gemm_plan.h"
#include "mm4_internal.h"

using namespace mm4;


namespace {

template <int BN, bool AMN, bool BMN, int MODE>
mm4_status launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tapf, const GemmArgs& args,
                     int grid,
                     cudaStream_t st) {
  auto kern = gemm_sm100_kernel<BN, AMN, BMN, MODE>;
  constexpr int smem = GemmCfg<BN>::SMEM_BYTES;
  mm4_status rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (rc != MM4_OK) return rc;
  if (args.coop_finalize) {
    // Every work unit has its own co-resident CTA; the launch fails (rather
    // than deadlocks) if the grid cannot be co-resident.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tapf, args);
    if (e == cudaSuccess) return MM4_OK;
    cudaGetLastError();
    GemmArgs fallback = args;
    fallback.coop_finalize = 0;
    kern<<<grid, GEMM_THREADS, smem, st>>>(ta, tb, tapf, fallback);
  } else {
    kern<<<grid, GEMM_THREADS, smem, st>>>(ta, tb, tapf, args);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_sm100_kernel launch");
  return MM4_OK;
}

template <int BN, bool AMN, bool BMN>
mm4_status launch_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tapf,
                       const GemmArgs& args, int grid,
                       cudaStream_t st) {
  if constexpr (BN == 512) {  // BN = 512 is a split-K-only tile
    if (mode == MODE_SPLITK_F16) return launch_tc<BN, AMN, BMN, MODE_SPLITK_F16>(ta, tb, tapf, args, grid, st);
    return launch_tc<BN, AMN, BMN, MODE_SPLITK_F32>(ta, tb, tapf, args, grid, st);
  }
  switch (mode) {
    case MODE_DIRECT_F16: return launch_tc<BN, AMN, BMN, MODE_DIRECT_F16>(ta, tb, tapf, args, grid, st);
    case MODE_SPLITK_F16: return launch_tc<BN, AMN, BMN, MODE_SPLITK_F16>(ta, tb, tapf, args, grid, st);
    case MODE_DIRECT_F32: return launch_tc<BN, AMN, BMN, MODE_DIRECT_F32>(ta, tb, tapf, args, grid, st);
    default: return launch_tc<BN, AMN, BMN, MODE_SPLITK_F32>(ta, tb, tapf, args, grid, st);
  }
}

template <int BN>
mm4_status launch_bn(bool amn, bool bmn, int mode, const CUtensorMap& ta, const CUtensorMap& tb,
                     const CUtensorMap& tapf,
                     const GemmArgs& args, int grid, cudaStream_t st) {
  if (!amn && !bmn) return launch_mode<BN, false, false>(mode, ta, tb, tapf, args, grid, st);
  if (!amn && bmn) return launch_mode<BN, false, true>(mode, ta, tb, tapf, args, grid, st);
  if (amn && !bmn) return launch_mode<BN, true, false>(mode, ta, tb, tapf, args, grid, st);
  return launch_mode<BN, true, true>(mode, ta, tb, tapf, args, grid, st);
}

// Element strides of A(m, k) and B(k, n) for the reference's transpose flags.
void operand_strides(const mm4_gemm_desc& d, long long* a_sm, long long* a_sk, long long* b_sk, long long* b_sn) {
  if (!d.transpose_left) {  // A [M][K]
    *a_sm = d.K;
    *a_sk = 1;
  } else {  // A [K][M]
    *a_sm = 1;
    *a_sk = d.M;
  }
  if (d.transpose_right) {  // B [N][K]
    *b_sn = d.K;
    *b_sk = 1;
  } else {  // B [K][N]
    *b_sn = 1;
    *b_sk = d.N;
  }
}

mm4_status run_simt(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias, void* C, bool out_f32,
                    cudaStream_t st) {
  long long a_sm, a_sk, b_sk, b_sn;
  operand_strides(p->d, &a_sm, &a_sk, &b_sk, &b_sn);
  dim3 grid((p->d.N + 63) / 64, (p->d.M + 63) / 64);
  if (out_f32) {
    gemm_simt_kernel<true><<<grid, 256, 0, st>>>(static_cast<const __half*>(A), a_sm, a_sk,
                                                  static_cast<const __half*>(B), b_sk, b_sn, nullptr, C, p->d.M,
                                                  p->d.N, p->d.K);
  } else {
    gemm_simt_kernel<false><<<grid, 256, 0, st>>>(static_cast<const __half*>(A), a_sm, a_sk,
                                                   static_cast<const __half*>(B), b_sk, b_sn,
                                                   static_cast<const __half*>(bias), C, p->d.M, p->d.N, p->d.K);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm_simt_kernel launch");
  return MM4_OK;
}

mm4_status build_maps(const mm4_gemm_plan* p, const void* A, const void* B, CUtensorMap* ta, CUtensorMap* tb,
                      CUtensorMap* tapf) {
  const mm4_gemm_desc& d = p->d;
  mm4_status rc;
  if (!d.transpose_left && p->splits > 1) {  // A [M][K] L2-prefetch map: box 256(K) x 128(M), unswizzled
    const uint64_t dims[2] = {static_cast<uint64_t>(d.K), static_cast<uint64_t>(d.M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.K) * 2};
    const uint32_t box[2] = {256, 128};
    rc = encode_tiled(tapf, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != MM4_OK) return rc;
  }
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
  if (d.transpose_right) {  // B [N][K]: box 64(K) x BN(N)
    const uint64_t dims[2] = {static_cast<uint64_t>(d.K), static_cast<uint64_t>(d.N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.K) * 2};
    const uint32_t box[2] = {64, static_cast<uint32_t>(p->bn < 256 ? p->bn : 256)};
    rc = encode_tiled(tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {  // B [K][N]: box 64(N) x 64(K), BN/64 per stage
    const uint64_t dims[2] = {static_cast<uint64_t>(d.N), static_cast<uint64_t>(d.K)};
    const uint64_t strides[1] = {static_cast<uint64_t>(d.N) * 2};
    const uint32_t box[2] = {64, 64};
    rc = encode_tiled(tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  return rc;
}

mm4_status run_tc(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias, void* C, float* C32,
                  void* ws, size_t ws_bytes, cudaStream_t st) {
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* status = nullptr;
  rc = status_word(&status);
  if (rc != MM4_OK) return rc;

  CUtensorMap ta, tb, tapf;
  memset(&tapf, 0, sizeof(tapf));
  rc = build_maps(p, A, B, &ta, &tb, &tapf);
  if (rc != MM4_OK) return rc;

  const bool out_f32 = (C32 != nullptr);
  GemmArgs args{};
  args.M = p->d.M;
  args.N = p->d.N;
  args.K = p->d.K;
  args.num_m_tiles = p->num_m_tiles;
  args.num_n_tiles = p->num_n_tiles;
  args.num_tiles = p->num_tiles;
  args.splits = p->splits;
  args.kb_total = p->kb_total;
  args.num_units = p->num_tiles * p->splits;
  args.group_m = 8;
  args.bias = out_f32 ? nullptr : static_cast<const __half*>(bias);
  args.C = static_cast<__half*>(C);
  args.C32 = C32;
  args.status = status;
  args.timeout_ns = wait_timeout_ns();
  int mode;
  if (p->splits > 1) {
    if (!ws) return fail(MM4_ERR_WORKSPACE, "split_k=%d needs a workspace of %zu bytes", p->splits, p->ws_bytes);
    if (ws_bytes < p->ws_bytes)
      return fail(MM4_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", ws_bytes, p->ws_bytes);
    if (!aligned16(ws)) return fail(MM4_ERR_WORKSPACE, "workspace must be 16-byte aligned");
    args.ws = static_cast<float*>(ws);
    args.ws_ld = p->num_n_tiles * p->bn;
    args.counters = reinterpret_cast<int*>(static_cast<char*>(ws) + p->ws_counter_offset);
    args.coop_finalize = (args.num_units <= info.sm_count) ? 1 : 0;
    mode = out_f32 ? MODE_SPLITK_F32 : MODE_SPLITK_F16;
  } else {
    mode = out_f32 ? MODE_DIRECT_F32 : MODE_DIRECT_F16;
  }
  const int grid = std::min(args.num_units, info.sm_count);
  const bool amn = p->d.transpose_left != 0;
  const bool bmn = p->d.transpose_right == 0;
  if (p->bn == 512) return launch_bn<512>(amn, bmn, mode, ta, tb, tapf, args, grid, st);
  if (p->bn == 256) return launch_bn<256>(amn, bmn, mode, ta, tb, tapf, args, grid, st);
  return launch_bn<128>(amn, bmn, mode, ta, tb, tapf, args, grid, st);
}

mm4_status validate(const mm4_gemm_desc* d) {
  if (!d) return fail(MM4_ERR_INVALID, "null gemm descriptor");
  if (d->M <= 0 || d->N <= 0 || d->K <= 0)
    return fail(MM4_ERR_INVALID, "GEMM dimensions must be positive (M=%d N=%d K=%d)", d->M, d->N, d->K);
  if (d->split_k < 0 || d->block_m < 0 || d->block_n < 0 || d->block_k < 0 || d->cooperative_simdgroups < 0 ||
      d->preemptive_simdgroups < 0)
    return fail(MM4_ERR_INVALID, "GEMM build options must be non-negative");
  if ((d->transpose_left != 0 && d->transpose_left != 1) || (d->transpose_right != 0 && d->transpose_right != 1))
    return fail(MM4_ERR_INVALID, "transpose flags must be 0 or 1");
  return MM4_OK;
}

}  // namespace

extern "C" {

mm4_status mm4_gemm_plan_create(mm4_gemm_plan** out, const mm4_gemm_desc* desc) {
  if (!out) return fail(MM4_ERR_INVALID, "null plan pointer");
  *out = nullptr;
  mm4_status rc = validate(desc);
  if (rc != MM4_OK) return rc;
  mm4_gemm_plan* p = new (std::nothrow) mm4_gemm_plan();
  if (!p) return fail(MM4_ERR_INVALID, "out of host memory");
  p->d = *desc;
  const mm4_gemm_desc& d = p->d;
  // TMA needs 16-byte global row pitches: the contiguous dimension of every
  // operand must be a multiple of 8 fp16 elements.
  const bool a_ok = d.transpose_left ? (d.M % 8 == 0) : (d.K % 8 == 0);
  const bool b_ok = d.transpose_right ? (d.K % 8 == 0) : (d.N % 8 == 0);
  p->tensor_core = a_ok && b_ok;
  // Split-K runs few, K-heavy units: a 128 x 512 tile (one TMEM-wide
  // accumulator) reads each A k-slab once per 512 columns. Otherwise 128 x 256
  // with a double-buffered accumulator, or 128 x 128 for narrow N.
  p->kb_total = (d.K + GEMM_BK - 1) / GEMM_BK;
  p->splits = std::max(1, std::min(d.split_k, p->kb_total));
  if (!p->tensor_core) p->splits = 1;
  p->bn = (d.N <= 128) ? 128 : 256;
  if (p->splits > 1 && d.N > 256) p->bn = 512;
  p->num_m_tiles = (d.M + GEMM_BM - 1) / GEMM_BM;
  p->num_n_tiles = (d.N + p->bn - 1) / p->bn;
  p->num_tiles = p->num_m_tiles * p->num_n_tiles;
  p->ws_bytes = 0;
  p->ws_counter_offset = 0;
  if (p->splits > 1) {
    const size_t acc = static_cast<size_t>(p->num_m_tiles) * GEMM_BM * p->num_n_tiles * p->bn * sizeof(float);
    p->ws_counter_offset = acc;
    p->ws_bytes = (acc + static_cast<size_t>(p->num_tiles) * 2 * sizeof(int) + 255) & ~static_cast<size_t>(255);
  }
  if (p->tensor_core)
    snprintf(p->name, sizeof(p->name), "gemm_sm100<BN=%d,%s%s,%s>", p->bn, d.transpose_left ? "A:MN" : "A:K",
             d.transpose_right ? ",B:K" : ",B:MN", p->splits > 1 ? "splitk" : "direct");
  else
    snprintf(p->name, sizeof(p->name), "gemm_simt<unaligned>");
  *out = p;
  return MM4_OK;
}

void mm4_gemm_plan_destroy(mm4_gemm_plan* plan) { delete plan; }

size_t mm4_gemm_workspace_size(const mm4_gemm_plan* plan) { return plan ? plan->ws_bytes : 0; }

const char* mm4_gemm_plan_kernel_name(const mm4_gemm_plan* plan) { return plan ? plan->name : ""; }

mm4_status mm4_gemm_run(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias, void* C,
                        void* workspace, size_t workspace_bytes, mm4_stream_t stream, int duplicated_count) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!A || !B || !C) return fail(MM4_ERR_INVALID, "null A/B/C pointer");
  if (p->d.bias && !bias) return fail(MM4_ERR_INVALID, "plan has bias but bias pointer is null");
  if (!p->d.bias) bias = nullptr;
  if (duplicated_count < 1) return fail(MM4_ERR_INVALID, "duplicated_count must be >= 1");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tc = p->tensor_core && aligned16(A) && aligned16(B);
  for (int i = 0; i < duplicated_count; ++i) {
    mm4_status rc;
    if (tc) {
      rc = run_tc(p, A, B, bias, C, nullptr, workspace, workspace_bytes, st);
    } else {
      DeviceInfo info;
      rc = current_device(&info);
      if (rc == MM4_OK) rc = run_simt(p, A, B, bias, C, false, st);
    }
    if (rc != MM4_OK) return rc;
  }
  return MM4_OK;
}

mm4_status mm4_gemm_partial_run(const mm4_gemm_plan* p, const void* A, const void* B, float* C32, void* workspace,
                                size_t workspace_bytes, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!A || !B || !C32) return fail(MM4_ERR_INVALID, "null A/B/C32 pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->tensor_core && aligned16(A) && aligned16(B))
    return run_tc(p, A, B, nullptr, nullptr, C32, workspace, workspace_bytes, st);
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  return run_simt(p, A, B, nullptr, C32, true, st);
}

mm4_status mm4_splitk_finalize(int32_t M, int32_t N, const float* C32, const void* bias, void* C,
                               mm4_stream_t stream) {
  if (M <= 0 || N <= 0) return fail(MM4_ERR_INVALID, "finalize dimensions must be positive");
  if (!C32 || !C) return fail(MM4_ERR_INVALID, "null C32/C pointer");
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  const size_t total = static_cast<size_t>(M) * N;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, static_cast<size_t>(info.sm_count) * 8));
  splitk_finalize_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      M, N, C32, static_cast<const __half*>(bias), static_cast<__half*>(C));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "splitk_finalize_kernel launch");
  return MM4_OK;
}

}  // extern "C"

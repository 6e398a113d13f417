// GEMM plans and dispatch: the sm_100a replacement for the reference's
// runtime-generated matmul kernel + reduce_sum_2 dispatch
// (Sources/matmul/matmul.swift:18-329 generator, :345-511 run()).
//
// The reference compiles one MSL kernel per (shape, tile, options) at run
// time; mm4 instead selects one of a fixed set of template instances
// (BN x operand majors x epilogue mode) when the plan is created.
#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <new>

#include "gemm_launch.cuh"
#include "gemm_simt.cuh"

using namespace mm4;


namespace {

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

// MM4_SPLITK_COOPERATIVE=0 selects the last-arriver finalize even where every
// work unit fits on the device at once (profilers that replay kernels may not
// support cooperative launches of clusters).
// MM4_SPLITK_DETERMINISTIC=1, read when a plan is created: split-K partials
// are stored one slice per split and summed in split order (bitwise
// reproducible runs; splits x the partial bytes of workspace, and more
// traffic than the default in-L2 reduction). Single-GPU plans only.
bool deterministic_splitk_requested() {
  const char* v = std::getenv("MM4_SPLITK_DETERMINISTIC");
  return v && v[0] == '1';
}

bool cooperative_finalize_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MM4_SPLITK_COOPERATIVE");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace

namespace mm4 {

// Tensor-core launch shared by the entry points; `grp` (may be null) joins a
// multi-GPU split-K group, which needs the cooperative finalize.
mm4_status gemm_run_tc(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias, void* C, float* C32,
                       void* ws, size_t ws_bytes, cudaStream_t st, const SplitKGroupArgs* grp) {
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* status = nullptr;
  rc = status_word(&status);
  if (rc != MM4_OK) return rc;

  CUtensorMap ta, tb;
  rc = gemm_build_maps(p, A, B, &ta, &tb);
  if (rc != MM4_OK) return rc;

  const bool out_f32 = (C32 != nullptr);
  GemmArgs args{};
  gemm_plan_args(p, &args);
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
    args.counters = reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + p->ws_counter_offset);
    args.det_split_floats = p->det_split_floats;
    // The cooperative finalize has every split of a tile meet in the
    // epilogue, so it needs all CTAs co-resident and no two splits of one
    // tile on the same CTA (pair): one CTA (pair) per (split, M-tile).
    const int grid = gemm_grid(p, args.num_units, info.sm_count);
    const int slots = p->pair ? grid / 2 : grid;
    args.coop_finalize =
        (grid <= info.sm_count && slots == p->splits * p->num_m_tiles && cooperative_finalize_enabled()) ? 1 : 0;
    mode = out_f32 ? MODE_SPLITK_F32 : MODE_SPLITK_F16;
  } else {
    mode = out_f32 ? MODE_DIRECT_F32 : MODE_DIRECT_F16;
  }
  if (grp && grp->world > 1) {
    if (p->det_split_floats != 0)
      return fail(MM4_ERR_UNSUPPORTED, "the deterministic split-K mode is single-GPU only");
    if (p->splits < 2 || out_f32)
      return fail(MM4_ERR_UNSUPPORTED, "a multi-GPU split-K group needs a split-K plan (split_k >= 2)");
    if (!args.coop_finalize)
      return fail(MM4_ERR_UNSUPPORTED,
                  "a multi-GPU split-K group needs one CTA (pair) per (split, M-tile) resident at once: %d x %d "
                  "%s does not fit this device's %d SMs (or MM4_SPLITK_COOPERATIVE=0)",
                  p->splits, p->num_m_tiles, p->pair ? "CTA pairs" : "CTAs", info.sm_count);
    args.grp = *grp;
  }
  return gemm_dispatch(p, mode, ta, tb, args, gemm_grid(p, args.num_units, info.sm_count), st);
}

}  // namespace mm4

namespace {

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

// SM count the tile choice assumes (B200); plans are made without touching a
// device, launches size their grids from the device's own count.
constexpr int kPlanSmCount = 148;

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
  p->kb_total = (d.K + GEMM_BK - 1) / GEMM_BK;
  p->splits = std::max(1, std::min(d.split_k, p->kb_total));
  if (!p->tensor_core) p->splits = 1;
  // Tile choice. CTA pairs (cta_group::2, 256-row tiles, each CTA staging half
  // of B) when M and N are both at least 256, otherwise one CTA with 128 x 256
  // (128 x 128 for narrow N); the adjustments below cover small problems and
  // split-K.
  p->pair = p->tensor_core && d.M >= 256 && d.N >= 256;
  p->bn = (d.N <= 128) ? 128 : 256;
  if (p->splits == 1 && p->tensor_core) {
    // Small problems: tiles that fill the SMs matter more than the pair's
    // lower shared-memory traffic. Use one-CTA tiles when 256 x 256 pair tiles
    // leave most SMs idle, and 128 x 128 tiles when 128 x 256 would too.
    const long long pair_tiles = static_cast<long long>((d.M + 255) / 256) * ((d.N + 255) / 256);
    if (p->pair && 2 * pair_tiles < kPlanSmCount) p->pair = false;
    const long long tiles256 = static_cast<long long>((d.M + 127) / 128) * ((d.N + 255) / 256);
    if (!p->pair && tiles256 < kPlanSmCount) p->bn = 128;
  }
  // Split-K with N > 256: 512-column tiles (all of TMEM, one accumulator)
  // read the fewest bytes per output, so they win when every (split, tile)
  // unit gets its own CTA (pair). When units outnumber the CTAs, CTA pairs use
  // 256 x 256 tiles with two accumulators so one tile's reduction overlaps the
  // next tile's main loop.
  if (p->splits > 1 && d.N > 256) {
    p->bn = 512;
    if (p->pair) {
      const int m_tiles = (d.M + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
      const long long units512 = static_cast<long long>(m_tiles) * ((d.N + 511) / 512) * p->splits;
      if (units512 > kPlanSmCount / 2) p->bn = 256;
    }
  }
  p->num_m_tiles = (d.M + (p->pair ? 2 * GEMM_BM : GEMM_BM) - 1) / (p->pair ? 2 * GEMM_BM : GEMM_BM);
  p->num_n_tiles = (d.N + p->bn - 1) / p->bn;
  p->num_tiles = p->num_m_tiles * p->num_n_tiles;
  p->ws_bytes = 0;
  p->ws_counter_offset = 0;
  p->det_split_floats = 0;
  if (p->splits > 1) {
    const int tile_m = p->pair ? 2 * GEMM_BM : GEMM_BM;
    size_t acc = static_cast<size_t>(p->num_m_tiles) * tile_m * p->num_n_tiles * p->bn * sizeof(float);
    if (deterministic_splitk_requested() && p->tensor_core) {
      // One partial slice per split, summed in split order by the finalize.
      p->det_split_floats = static_cast<long long>(acc / sizeof(float));
      acc *= static_cast<size_t>(p->splits);
    }
    p->ws_counter_offset = acc;
    // one 64-bit arrival counter per 128-row half tile
    const size_t counters = static_cast<size_t>(p->num_tiles) * (p->pair ? 2 : 1) * sizeof(unsigned long long);
    p->ws_bytes = (acc + counters + 255) & ~static_cast<size_t>(255);
  }
  if (p->tensor_core)
    snprintf(p->name, sizeof(p->name), "gemm_sm100%s<BM=%d,BN=%d,%s%s,%s>", p->pair ? "_pair" : "",
             p->pair ? 2 * GEMM_BM : GEMM_BM, p->bn, d.transpose_left ? "A:MN" : "A:K",
             d.transpose_right ? ",B:K" : ",B:MN",
             p->splits > 1 ? (p->det_split_floats != 0 ? "splitk-deterministic" : "splitk") : "direct");
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
      rc = gemm_run_tc(p, A, B, bias, C, nullptr, workspace, workspace_bytes, st);
    } else {
      DeviceInfo info;
      rc = current_device(&info);
      if (rc == MM4_OK) rc = run_simt(p, A, B, bias, C, false, st);
    }
    if (rc != MM4_OK) return rc;
  }
  return MM4_OK;
}

mm4_status mm4_gemm_run_host(const mm4_gemm_plan* p, const void* hA, const void* hB, const void* hbias, void* hC,
                             void* dA, void* dB, void* dbias, void* dC, void* workspace, size_t workspace_bytes,
                             int32_t chunks, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!hA || !hB || !hC || !dA || !dB || !dC) return fail(MM4_ERR_INVALID, "null buffer pointer");
  if (p->d.bias && (!hbias || !dbias)) return fail(MM4_ERR_INVALID, "plan has bias but a bias pointer is null");
  const mm4_gemm_desc& d = p->d;
  const size_t a_row = static_cast<size_t>(d.K) * 2, c_row = static_cast<size_t>(d.N) * 2;
  // Chunks of whole 256-row blocks of A and C; A must be [M][K] for its rows
  // to be contiguous (otherwise one chunk).
  int n = chunks > 0 ? chunks : 16;
  const int blocks = (d.M + 255) / 256;
  if (d.transpose_left) n = 1;
  n = std::max(1, std::min(std::min(n, kHostMaxChunks), blocks));
  const int rows_per = (blocks + n - 1) / n * 256;
  n = (d.M + rows_per - 1) / rows_per;
  // Plans of the chunk heights (all but the last share one).
  mm4_gemm_plan* sub[2] = {nullptr, nullptr};
  auto cleanup = [&]() {
    for (auto*& q : sub)
      if (q) {
        mm4_gemm_plan_destroy(q);
        q = nullptr;
      }
  };
  const int last_rows = d.M - (n - 1) * rows_per;
  for (int i = 0; i < 2; ++i) {
    mm4_gemm_desc sd = d;
    sd.M = i == 0 ? std::min(rows_per, d.M) : last_rows;
    mm4_status rc = mm4_gemm_plan_create(&sub[i], &sd);
    if (rc == MM4_OK && (sub[i]->det_split_floats != 0) != (p->det_split_floats != 0))
      rc = fail(MM4_ERR_INVALID, "MM4_SPLITK_DETERMINISTIC changed since the plan was created");
    if (rc != MM4_OK) {
      cleanup();
      return rc;
    }
  }
  // The block plans run on the whole plan's workspace, shifted so that their
  // split-K arrival counters are the whole plan's counters and their partials
  // lie inside its partial area. Counters then stay multiples of the split
  // count whichever plan ran last, and the partial area keeps its invariant
  // (zero-filled, or overwritten whole in the deterministic mode).
  auto block_ws = [&](const mm4_gemm_plan* q, void** w, size_t* bytes) {
    *w = workspace;
    *bytes = workspace_bytes;
    if (!workspace || q->ws_bytes == 0 || p->ws_bytes == 0 || q->ws_counter_offset >= p->ws_counter_offset) return;
    const size_t delta = p->ws_counter_offset - q->ws_counter_offset;
    *w = static_cast<char*>(workspace) + delta;
    *bytes = workspace_bytes > delta ? workspace_bytes - delta : 0;
  };
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cleanup();
    return cuda_fail(e, "cudaGetDevice");
  }
  std::lock_guard<std::mutex> lock(host_pipe_mutex());
  HostPipe* hp = nullptr;
  mm4_status rc = host_pipe(dev, &hp);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto at = [](const void* base, size_t off) { return static_cast<char*>(const_cast<void*>(base)) + off; };
  auto run = [&]() -> mm4_status {
    if (rc != MM4_OK) return rc;
    MM4_CUDA_TRY(cudaEventRecord(hp->start, st));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->in, hp->start, 0));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->start, 0));
    // B and bias first: every chunk needs them whole.
    const size_t b_bytes = static_cast<size_t>(d.K) * d.N * 2;
    MM4_CUDA_TRY(cudaMemcpyAsync(dB, hB, b_bytes, cudaMemcpyHostToDevice, hp->in));
    if (d.bias) MM4_CUDA_TRY(cudaMemcpyAsync(dbias, hbias, c_row, cudaMemcpyHostToDevice, hp->in));
    for (int c = 0; c < n; ++c) {
      const int m0 = c * rows_per, rows = c == n - 1 ? last_rows : rows_per;
      const size_t ao = d.transpose_left ? 0 : static_cast<size_t>(m0) * a_row;
      const size_t an = d.transpose_left ? static_cast<size_t>(d.K) * d.M * 2 : static_cast<size_t>(rows) * a_row;
      MM4_CUDA_TRY(cudaMemcpyAsync(at(dA, ao), at(hA, ao), an, cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaEventRecord(hp->loaded[c], hp->in));
      MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->loaded[c], 0));
      const size_t co = static_cast<size_t>(m0) * c_row;
      const mm4_gemm_plan* q = c == n - 1 ? sub[1] : sub[0];
      void* qws = nullptr;
      size_t qws_bytes = 0;
      block_ws(q, &qws, &qws_bytes);
      mm4_status r = mm4_gemm_run(q, at(dA, ao), dB, d.bias ? dbias : nullptr, at(dC, co), qws, qws_bytes, stream, 1);
      if (r != MM4_OK) return r;
      MM4_CUDA_TRY(cudaEventRecord(hp->done[c], st));
      MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->done[c], 0));
      MM4_CUDA_TRY(cudaMemcpyAsync(at(hC, co), at(dC, co), static_cast<size_t>(rows) * c_row,
                                   cudaMemcpyDeviceToHost, hp->out));
    }
    MM4_CUDA_TRY(cudaEventRecord(hp->end, hp->out));
    MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->end, 0));
    return MM4_OK;
  };
  rc = run();
  if (rc != MM4_OK) host_pipe_join(hp, st);
  cleanup();
  return rc;
}

mm4_status mm4_gemm_partial_run(const mm4_gemm_plan* p, const void* A, const void* B, float* C32, void* workspace,
                                size_t workspace_bytes, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!A || !B || !C32) return fail(MM4_ERR_INVALID, "null A/B/C32 pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->tensor_core && aligned16(A) && aligned16(B))
    return gemm_run_tc(p, A, B, nullptr, nullptr, C32, workspace, workspace_bytes, st);
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

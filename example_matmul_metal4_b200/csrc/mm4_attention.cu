// Attention plans and dispatch: replaces the reference's attention
// createSource + run(...) (Sources/attention/attention.swift:23-382, :398-541).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "attention_bwd_sm100.cuh"
#include "attention_sm100.cuh"
#include "mm4_internal.h"

using namespace mm4;

struct mm4_attention_plan {
  mm4_attention_desc d;
  float scale;
  char name[96];
};

namespace {

mm4_status encode_attn_map(CUtensorMap* map, const void* base, int layout, int D, int S, int H, int B) {
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  if (layout == MM4_ATTN_BHSD) {  // [B][H][S][D]
    dims[0] = D; dims[1] = S; dims[2] = H; dims[3] = B;
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(S) * D * 2;
    strides[2] = static_cast<uint64_t>(H) * S * D * 2;
    box[0] = 64; box[1] = 128; box[2] = 1; box[3] = 1;
  } else {  // [B][S][H][D]
    dims[0] = D; dims[1] = H; dims[2] = S; dims[3] = B;
    strides[0] = static_cast<uint64_t>(D) * 2;
    strides[1] = static_cast<uint64_t>(H) * D * 2;
    strides[2] = static_cast<uint64_t>(S) * H * D * 2;
    box[0] = 64; box[1] = 1; box[2] = 128; box[3] = 1;
  }
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

extern "C" {

mm4_status mm4_attention_plan_create(mm4_attention_plan** out, const mm4_attention_desc* d) {
  if (!out) return fail(MM4_ERR_INVALID, "null plan pointer");
  *out = nullptr;
  if (!d) return fail(MM4_ERR_INVALID, "null attention descriptor");
  if (d->batch <= 0 || d->heads_q <= 0 || d->heads_kv <= 0 || d->rows <= 0 || d->columns <= 0 || d->head_dim <= 0)
    return fail(MM4_ERR_INVALID, "attention dimensions must be positive");
  if (d->heads_q % d->heads_kv != 0)
    return fail(MM4_ERR_INVALID, "heads_kv (%d) must divide heads_q (%d)", d->heads_kv, d->heads_q);
  if (d->layout != MM4_ATTN_BHSD && d->layout != MM4_ATTN_BSHD)
    return fail(MM4_ERR_INVALID, "unknown attention layout %d", d->layout);
  if (d->head_dim != 128 && d->head_dim != 64)
    return fail(MM4_ERR_UNSUPPORTED, "head_dim %d: this build implements head_dim 128 and 64", d->head_dim);
  if (!(d->scale >= 0.f) && !(d->scale < 0.f)) return fail(MM4_ERR_INVALID, "scale is NaN");
  mm4_attention_plan* p = new (std::nothrow) mm4_attention_plan();
  if (!p) return fail(MM4_ERR_INVALID, "out of host memory");
  p->d = *d;
  p->scale = d->scale > 0.f ? d->scale : 1.0f / std::sqrt(static_cast<float>(d->head_dim));
  snprintf(p->name, sizeof(p->name), "attention_fwd_sm100<D=128,%s>", d->layout == MM4_ATTN_BHSD ? "BHSD" : "BSHD");
  *out = p;
  return MM4_OK;
}

void mm4_attention_plan_destroy(mm4_attention_plan* plan) { delete plan; }

const char* mm4_attention_plan_kernel_name(const mm4_attention_plan* plan) { return plan ? plan->name : ""; }

}  // extern "C"

namespace {

template <int D>
mm4_status launch_forward(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnArgs& args,
                          const mm4_attention_desc& d, int sm_count, cudaStream_t st, int duplicated_count) {
  const void* kern = reinterpret_cast<const void*>(attention_fwd_sm100_kernel<D>);
  constexpr int smem = AttFwdCfg<D>::SMEM_BYTES;
  mm4_status rc = ensure_smem_attr(kern, smem);
  if (rc != MM4_OK) return rc;
  {
    // The kernel moves registers between warpgroups (setmaxnreg); that only
    // completes if the launch allocates at least ATT_REGS_NEEDED per thread.
    static int launch_regs = -1;
    if (launch_regs < 0) {
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(attention_fwd_sm100_kernel)");
      launch_regs = fa.numRegs;
    }
    if (launch_regs < ATT_REGS_NEEDED)
      return fail(MM4_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, needs %d", launch_regs,
                  ATT_REGS_NEEDED);
  }
  // Persistent: one CTA per SM at most, each walking units (batch, head,
  // 256 query rows) gridDim.x apart.
  const long long units = static_cast<long long>(args.q_blocks) * d.heads_q * d.batch;
  if (units > 0x7fffffffLL) return fail(MM4_ERR_UNSUPPORTED, "too many query blocks for one launch");
  const dim3 grid(static_cast<unsigned>(std::min<long long>(units, sm_count)));
  for (int i = 0; i < duplicated_count; ++i) {
    attention_fwd_sm100_kernel<D><<<grid, ATT_THREADS, smem, st>>>(tq, tk, tv, args);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "attention_fwd_sm100_kernel launch");
  }
  return MM4_OK;
}

mm4_status attention_forward(const mm4_attention_plan* p, const void* Q, const void* K, const void* V, void* O,
                             float* lse, cudaStream_t st, int duplicated_count) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!Q || !K || !V || !O) return fail(MM4_ERR_INVALID, "null Q/K/V/O pointer");
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return fail(MM4_ERR_INVALID, "Q, K, V and O must be 16-byte aligned");
  if (duplicated_count < 1) return fail(MM4_ERR_INVALID, "duplicated_count must be >= 1");
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* status = nullptr;
  rc = status_word(&status);
  if (rc != MM4_OK) return rc;
  const mm4_attention_desc& d = p->d;
  CUtensorMap tq, tk, tv;
  rc = encode_attn_map(&tq, Q, d.layout, d.head_dim, d.rows, d.heads_q, d.batch);
  if (rc == MM4_OK) rc = encode_attn_map(&tk, K, d.layout, d.head_dim, d.columns, d.heads_kv, d.batch);
  if (rc == MM4_OK) rc = encode_attn_map(&tv, V, d.layout, d.head_dim, d.columns, d.heads_kv, d.batch);
  if (rc != MM4_OK) return rc;

  AttnArgs args{};
  args.batch = d.batch;
  args.heads_q = d.heads_q;
  args.heads_kv = d.heads_kv;
  args.R = d.rows;
  args.C = d.columns;
  args.layout = d.layout;
  args.q_blocks = (d.rows + ATT_CTA_ROWS - 1) / ATT_CTA_ROWS;
  args.num_units = static_cast<int>(std::min<long long>(
      static_cast<long long>(args.q_blocks) * d.heads_q * d.batch, 0x7fffffffLL));
  args.scale_log2 = p->scale * 1.4426950408889634f;
  args.O = static_cast<__half*>(O);
  args.lse = lse;
  args.status = status;
  args.timeout_ns = wait_timeout_ns();

  if (d.head_dim == 128) return launch_forward<128>(tq, tk, tv, args, d, info.sm_count, st, duplicated_count);
  return launch_forward<64>(tq, tk, tv, args, d, info.sm_count, st, duplicated_count);
}

template <int D>
mm4_status launch_backward(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                           const AttnBwdArgs& args, const mm4_attention_desc& d, const void* O, const void* dO,
                           const float* lse, cudaStream_t st, int sm_count) {
  const long long rows_total = static_cast<long long>(d.batch) * d.heads_q * args.R_pad;
  const int prep_grid = static_cast<int>(std::min<long long>((rows_total + 7) / 8, 16ll * sm_count));
  attention_bwd_prep_kernel<D><<<prep_grid, 256, 0, st>>>(static_cast<const __half*>(O),
                                                           static_cast<const __half*>(dO), lse,
                                                           const_cast<float*>(args.lse2), const_cast<float*>(args.dvec),
                                                           d.batch, d.heads_q, d.rows, args.R_pad, d.layout);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_bwd_prep_kernel launch");

  dim3 grid_kv((d.columns + ATT_BN - 1) / ATT_BN, d.heads_kv, d.batch);
  dim3 grid_q(args.R_pad / ATT_BM, d.heads_q, d.batch);
  if (grid_kv.y > 65535 || grid_kv.z > 65535 || grid_q.y > 65535)
    return fail(MM4_ERR_UNSUPPORTED, "too many heads or batches for one launch");
  constexpr int dkdv_smem = AtbCfg<D>::DKDV_SMEM;
  constexpr int dq_smem = AtbCfg<D>::DQ_SMEM;
  mm4_status rc = ensure_smem_attr(reinterpret_cast<const void*>(attention_bwd_dkdv_kernel<D>), dkdv_smem);
  if (rc == MM4_OK) rc = ensure_smem_attr(reinterpret_cast<const void*>(attention_bwd_dq_kernel<D>), dq_smem);
  if (rc != MM4_OK) return rc;
  attention_bwd_dkdv_kernel<D><<<grid_kv, ATB_THREADS, dkdv_smem, st>>>(tq, tk, tv, tdo, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_bwd_dkdv_kernel launch");
  attention_bwd_dq_kernel<D><<<grid_q, ATB_THREADS, dq_smem, st>>>(tq, tk, tv, tdo, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention_bwd_dq_kernel launch");
  return MM4_OK;
}

int padded_rows(const mm4_attention_desc& d) { return (d.rows + ATT_BM - 1) / ATT_BM * ATT_BM; }

size_t bwd_workspace_bytes(const mm4_attention_desc& d) {
  return 2 * static_cast<size_t>(d.batch) * d.heads_q * padded_rows(d) * sizeof(float);
}

}  // namespace

extern "C" {

mm4_status mm4_attention_fwd(const mm4_attention_plan* p, const void* Q, const void* K, const void* V, void* O,
                             mm4_stream_t stream, int duplicated_count) {
  return attention_forward(p, Q, K, V, O, nullptr, static_cast<cudaStream_t>(stream), duplicated_count);
}

mm4_status mm4_attention_fwd_lse(const mm4_attention_plan* p, const void* Q, const void* K, const void* V, void* O,
                                 float* lse, mm4_stream_t stream) {
  if (!lse) return fail(MM4_ERR_INVALID, "null lse pointer");
  return attention_forward(p, Q, K, V, O, lse, static_cast<cudaStream_t>(stream), 1);
}

mm4_status mm4_attention_fwd_host(const mm4_attention_plan* p, const void* hQ, const void* hK, const void* hV,
                                  void* hO, void* dQ, void* dK, void* dV, void* dO, int32_t chunks,
                                  mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!hQ || !hK || !hV || !hO || !dQ || !dK || !dV || !dO) return fail(MM4_ERR_INVALID, "null buffer pointer");
  const mm4_attention_desc& d = p->d;
  const int group = d.heads_q / d.heads_kv;
  // Pieces that a chunk may hold whole: a key/value head with its query heads
  // ([B][H][S][D]), or a batch element ([B][S][H][D]).
  const bool bhsd = d.layout == MM4_ATTN_BHSD;
  const long long pieces = bhsd ? static_cast<long long>(d.batch) * d.heads_kv : d.batch;
  const size_t elt = 2;
  const size_t q_piece = (bhsd ? static_cast<size_t>(group) : static_cast<size_t>(d.heads_q)) * d.rows * d.head_dim * elt;
  const size_t kv_piece = (bhsd ? 1 : static_cast<size_t>(d.heads_kv)) * d.columns * d.head_dim * elt;
  int n = chunks > 0 ? chunks : 16;
  n = static_cast<int>(std::min<long long>(std::min(n, kHostMaxChunks), pieces));
  int dev = -1;
  MM4_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(host_pipe_mutex());
  HostPipe* hp = nullptr;
  mm4_status rc = host_pipe(dev, &hp);
  if (rc != MM4_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto run = [&]() -> mm4_status {
    MM4_CUDA_TRY(cudaEventRecord(hp->start, st));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->in, hp->start, 0));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->start, 0));
    auto at = [](const void* base, size_t off) { return static_cast<char*>(const_cast<void*>(base)) + off; };
    for (int c = 0; c < n; ++c) {
      const long long p0 = c * pieces / n, p1 = (c + 1) * pieces / n, np = p1 - p0;
      const size_t qo = static_cast<size_t>(p0) * q_piece, qn = static_cast<size_t>(np) * q_piece;
      const size_t ko = static_cast<size_t>(p0) * kv_piece, kn = static_cast<size_t>(np) * kv_piece;
      MM4_CUDA_TRY(cudaMemcpyAsync(at(dQ, qo), at(hQ, qo), qn, cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaMemcpyAsync(at(dK, ko), at(hK, ko), kn, cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaMemcpyAsync(at(dV, ko), at(hV, ko), kn, cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaEventRecord(hp->loaded[c], hp->in));
      MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->loaded[c], 0));
      // The chunk as a problem of its own: its (batch, head) units are
      // computed exactly as in the whole problem.
      mm4_attention_plan sub = *p;
      if (bhsd) {
        sub.d.batch = 1;
        sub.d.heads_q = static_cast<int32_t>(np * group);
        sub.d.heads_kv = static_cast<int32_t>(np);
      } else {
        sub.d.batch = static_cast<int32_t>(np);
      }
      mm4_status r = attention_forward(&sub, at(dQ, qo), at(dK, ko), at(dV, ko), at(dO, qo), nullptr, st, 1);
      if (r != MM4_OK) return r;
      MM4_CUDA_TRY(cudaEventRecord(hp->done[c], st));
      MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->done[c], 0));
      MM4_CUDA_TRY(cudaMemcpyAsync(at(hO, qo), at(dO, qo), qn, cudaMemcpyDeviceToHost, hp->out));
    }
    MM4_CUDA_TRY(cudaEventRecord(hp->end, hp->out));
    MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->end, 0));
    return MM4_OK;
  };
  rc = run();
  if (rc != MM4_OK) host_pipe_join(hp, st);
  return rc;
}

size_t mm4_attention_bwd_workspace_size(const mm4_attention_plan* p) { return p ? bwd_workspace_bytes(p->d) : 0; }

mm4_status mm4_attention_bwd(const mm4_attention_plan* p, const void* Q, const void* K, const void* V, const void* O,
                             const void* dO, const float* lse, void* dQ, void* dK, void* dV, void* workspace,
                             size_t workspace_bytes, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!Q || !K || !V || !O || !dO || !lse || !dQ || !dK || !dV)
    return fail(MM4_ERR_INVALID, "null tensor pointer");
  const void* ptrs[] = {Q, K, V, O, dO, dQ, dK, dV};
  for (const void* q : ptrs)
    if (!aligned16(q)) return fail(MM4_ERR_INVALID, "Q, K, V, O, dO, dQ, dK and dV must be 16-byte aligned");
  const mm4_attention_desc& d = p->d;
  const size_t need = bwd_workspace_bytes(d);
  if (!workspace || workspace_bytes < need)
    return fail(MM4_ERR_WORKSPACE, "attention backward needs a %zu-byte workspace", need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return fail(MM4_ERR_INVALID, "workspace must be 16-byte aligned");
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* status = nullptr;
  rc = status_word(&status);
  if (rc != MM4_OK) return rc;
  CUtensorMap tq, tk, tv, tdo;
  rc = encode_attn_map(&tq, Q, d.layout, d.head_dim, d.rows, d.heads_q, d.batch);
  if (rc == MM4_OK) rc = encode_attn_map(&tdo, dO, d.layout, d.head_dim, d.rows, d.heads_q, d.batch);
  if (rc == MM4_OK) rc = encode_attn_map(&tk, K, d.layout, d.head_dim, d.columns, d.heads_kv, d.batch);
  if (rc == MM4_OK) rc = encode_attn_map(&tv, V, d.layout, d.head_dim, d.columns, d.heads_kv, d.batch);
  if (rc != MM4_OK) return rc;

  const int R_pad = padded_rows(d);
  float* lse2 = static_cast<float*>(workspace);
  float* dvec = lse2 + static_cast<size_t>(d.batch) * d.heads_q * R_pad;
  AttnBwdArgs args{};
  args.batch = d.batch;
  args.heads_q = d.heads_q;
  args.heads_kv = d.heads_kv;
  args.R = d.rows;
  args.C = d.columns;
  args.R_pad = R_pad;
  args.layout = d.layout;
  args.scale = p->scale;
  args.scale_log2 = p->scale * 1.4426950408889634f;
  args.lse2 = lse2;
  args.dvec = dvec;
  args.dQ = static_cast<__half*>(dQ);
  args.dK = static_cast<__half*>(dK);
  args.dV = static_cast<__half*>(dV);
  args.status = status;
  args.timeout_ns = wait_timeout_ns();

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d.head_dim == 128) return launch_backward<128>(tq, tk, tv, tdo, args, d, O, dO, lse, st, info.sm_count);
  return launch_backward<64>(tq, tk, tv, tdo, args, d, O, dO, lse, st, info.sm_count);
}

mm4_status mm4_attention_bwd_host(const mm4_attention_plan* p, const void* const* host_in, void* const* host_out,
                                  void* const* dev_in, void* const* dev_out, void* workspace, size_t workspace_bytes,
                                  int32_t chunks, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!host_in || !host_out || !dev_in || !dev_out) return fail(MM4_ERR_INVALID, "null buffer array");
  for (int i = 0; i < 6; ++i)
    if (!host_in[i] || !dev_in[i]) return fail(MM4_ERR_INVALID, "null input buffer %d", i);
  for (int i = 0; i < 3; ++i)
    if (!host_out[i] || !dev_out[i]) return fail(MM4_ERR_INVALID, "null output buffer %d", i);
  const mm4_attention_desc& d = p->d;
  const size_t need = bwd_workspace_bytes(d);
  if (!workspace || workspace_bytes < need)
    return fail(MM4_ERR_WORKSPACE, "attention backward needs a %zu-byte workspace", need);
  const int group = d.heads_q / d.heads_kv;
  const bool bhsd = d.layout == MM4_ATTN_BHSD;
  const long long pieces = bhsd ? static_cast<long long>(d.batch) * d.heads_kv : d.batch;
  const size_t qh = bhsd ? static_cast<size_t>(group) : static_cast<size_t>(d.heads_q);   // query heads per piece
  const size_t kh = bhsd ? 1 : static_cast<size_t>(d.heads_kv);                           // key/value heads per piece
  const size_t q_piece = qh * d.rows * d.head_dim * 2, kv_piece = kh * d.columns * d.head_dim * 2;
  const size_t l_piece = qh * d.rows * sizeof(float);
  const size_t w_piece = 2 * qh * padded_rows(d) * sizeof(float);
  int n = chunks > 0 ? chunks : 16;
  n = static_cast<int>(std::min<long long>(std::min(n, kHostMaxChunks), pieces));
  int dev = -1;
  MM4_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(host_pipe_mutex());
  HostPipe* hp = nullptr;
  mm4_status rc = host_pipe(dev, &hp);
  if (rc != MM4_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto run = [&]() -> mm4_status {
    MM4_CUDA_TRY(cudaEventRecord(hp->start, st));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->in, hp->start, 0));
    MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->start, 0));
    auto at = [](const void* base, size_t off) { return static_cast<char*>(const_cast<void*>(base)) + off; };
    for (int c = 0; c < n; ++c) {
      const long long p0 = c * pieces / n, p1 = (c + 1) * pieces / n, np = p1 - p0;
      // Offsets and sizes of the chunk in Q / O / dO (and dQ), K / V (and dK, dV), lse.
      const size_t qo = p0 * q_piece, qn = np * q_piece, ko = p0 * kv_piece, kn = np * kv_piece;
      const size_t lo = p0 * l_piece, ln = np * l_piece;
      const size_t in_off[6] = {qo, ko, ko, qo, qo, lo}, in_len[6] = {qn, kn, kn, qn, qn, ln};
      for (int i = 0; i < 6; ++i)
        MM4_CUDA_TRY(cudaMemcpyAsync(at(dev_in[i], in_off[i]), at(host_in[i], in_off[i]), in_len[i],
                                     cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaEventRecord(hp->loaded[c], hp->in));
      MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->loaded[c], 0));
      mm4_attention_plan sub = *p;
      if (bhsd) {
        sub.d.batch = 1;
        sub.d.heads_q = static_cast<int32_t>(np * group);
        sub.d.heads_kv = static_cast<int32_t>(np);
      } else {
        sub.d.batch = static_cast<int32_t>(np);
      }
      mm4_status r = mm4_attention_bwd(
          &sub, at(dev_in[0], qo), at(dev_in[1], ko), at(dev_in[2], ko), at(dev_in[3], qo), at(dev_in[4], qo),
          reinterpret_cast<const float*>(at(dev_in[5], lo)), at(dev_out[0], qo), at(dev_out[1], ko),
          at(dev_out[2], ko), at(workspace, p0 * w_piece), np * w_piece, stream);
      if (r != MM4_OK) return r;
      MM4_CUDA_TRY(cudaEventRecord(hp->done[c], st));
      MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->done[c], 0));
      const size_t out_off[3] = {qo, ko, ko}, out_len[3] = {qn, kn, kn};
      for (int i = 0; i < 3; ++i)
        MM4_CUDA_TRY(cudaMemcpyAsync(at(host_out[i], out_off[i]), at(dev_out[i], out_off[i]), out_len[i],
                                     cudaMemcpyDeviceToHost, hp->out));
    }
    MM4_CUDA_TRY(cudaEventRecord(hp->end, hp->out));
    MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->end, 0));
    return MM4_OK;
  };
  rc = run();
  if (rc != MM4_OK) host_pipe_join(hp, st);
  return rc;
}

}  // extern "C"

namespace {

// Evaluates the forward kernel's two exponentials on a vector: method 0 is
// the hardware ex2.approx.ftz (MUFU), method 1 the FMA-pipe cubic
// ex2_poly2 (packed fp32x2: lane x takes x[i], lane y x[i + 1]).
__global__ void debug_ex2_kernel(const float* x, float* y, long long n, int method) {
  const long long i = 2 * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float a = x[i];
  const float b = i + 1 < n ? x[i + 1] : 0.f;
  float2 r;
  if (method == 1) {
    r = ex2_poly2(make_float2(a, b));
  } else {
    r.x = ex2_approx(a);
    r.y = ex2_approx(b);
  }
  y[i] = r.x;
  if (i + 1 < n) y[i + 1] = r.y;
}

}  // namespace

extern "C" {

mm4_status mm4_debug_ex2(const float* x, float* y, int64_t n, int method, mm4_stream_t stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return fail(MM4_ERR_INVALID, "mm4_debug_ex2: bad vector");
  if (method != 0 && method != 1) return fail(MM4_ERR_INVALID, "mm4_debug_ex2: method must be 0 or 1");
  if (n == 0) return MM4_OK;
  const long long pairs = (n + 1) / 2;
  const int threads = 256;
  const long long blocks = (pairs + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return fail(MM4_ERR_INVALID, "mm4_debug_ex2: vector too long");
  debug_ex2_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, y, static_cast<long long>(n), method);
  MM4_CUDA_TRY(cudaGetLastError());
  return MM4_OK;
}

}  // extern "C"

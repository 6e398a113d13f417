// Attention plans and dispatch: replaces the reference's attention
// createSource + run(...) (Sources/attention/attention.swift:23-382, :398-541).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

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
  if (d->head_dim != ATT_D)
    return fail(MM4_ERR_UNSUPPORTED, "head_dim %d: this build implements head_dim 128 (the reference's D)",
                d->head_dim);
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

mm4_status mm4_attention_fwd(const mm4_attention_plan* p, const void* Q, const void* K, const void* V, void* O,
                             mm4_stream_t stream, int duplicated_count) {
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
  args.scale_log2 = p->scale * 1.4426950408889634f;
  args.O = static_cast<__half*>(O);
  args.status = status;
  args.timeout_ns = wait_timeout_ns();

  rc = ensure_smem_attr(reinterpret_cast<const void*>(attention_fwd_sm100_kernel), ATT_SMEM_BYTES);
  if (rc != MM4_OK) return rc;
  {
    // The kernel moves registers between warpgroups (setmaxnreg); that only
    // completes if the launch allocates at least ATT_REGS_NEEDED per thread.
    static int launch_regs = -1;
    if (launch_regs < 0) {
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(attention_fwd_sm100_kernel));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(attention_fwd_sm100_kernel)");
      launch_regs = fa.numRegs;
    }
    if (launch_regs < ATT_REGS_NEEDED)
      return fail(MM4_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, needs %d", launch_regs,
                  ATT_REGS_NEEDED);
  }
  dim3 grid((d.rows + ATT_CTA_ROWS - 1) / ATT_CTA_ROWS, d.heads_q, d.batch);
  if (grid.y > 65535 || grid.z > 65535) return fail(MM4_ERR_UNSUPPORTED, "too many heads or batches for one launch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < duplicated_count; ++i) {
    attention_fwd_sm100_kernel<<<grid, ATT_THREADS, ATT_SMEM_BYTES, st>>>(tq, tk, tv, args);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "attention_fwd_sm100_kernel launch");
  }
  return MM4_OK;
}

}  // extern "C"

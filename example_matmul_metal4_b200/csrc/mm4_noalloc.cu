// Split-K GEMM entry point that allocates no device memory.
//
// Who needs it: callers that must not call cudaMalloc from the thread that
// issues the GEMM — code running under a custom device allocator that owns
// all of GPU memory (a framework's caching allocator or a memory pool that
// would be bypassed and fragmented), hard real-time or inference-serving
// loops where an allocation can stall or fail mid-request, and plug-in hosts
// that hand the library only the input and output buffers. For them this
// entry point keeps the split-K partial-sum scratch in a file-scope
// `static __device__` array instead of a caller- or library-allocated
// workspace.
//
// The scratch is MM4_NOALLOC_SCRATCH_BYTES (4 MiB) per device: it lives in
// the library image, so every GPU that loads libmm4.so holds it until the
// process exits. A plan whose split-K workspace would not fit is rejected
// with MM4_ERR_WORKSPACE.
//
// Set-up: the first call on a device (with that device current) resolves the
// device addresses of the scratch array and of this file's status word with
// cudaGetSymbolAddress. Make that first call before any stream capture.
//
// Sharing: every call on a device uses the same scratch. Each call first
// clears the part it uses (the fp32 partial sums and the per-tile arrival
// counters must start at zero) with cudaMemsetAsync on the caller's stream,
// so back-to-back calls on one stream are correct; calls that overlap on
// the GPU (different streams without ordering, or concurrent host threads)
// race on the scratch and give wrong results.
//
// Device-side bounded waits still end a stuck kernel; a run-out wait is
// recorded in this file's own static status word (mm4_check() reads the
// library's per-device status word, which this entry point never allocates).
#include <algorithm>
#include <cstring>
#include <mutex>

#include "gemm_launch.cuh"

using namespace mm4;

constexpr size_t MM4_NOALLOC_SCRATCH_BYTES = size_t(4) << 20;

// File-scope device storage. In host code these names are host-side
// stand-ins, not device addresses: only the pointers resolved by
// setup_device() may be handed to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MM4_NOALLOC_SCRATCH_BYTES];
static __device__ int g_noalloc_status;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
int* g_status_ptr[kMaxDevices] = {};

// Resolves the device addresses of the static arrays for the current device
// (the host-side names are only stand-ins and must never reach a kernel).
mm4_status setup_device(int dev, void** scratch, int** status) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* s = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&s, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    void* st = nullptr;
    e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_status)");
    g_scratch_ptr[dev] = s;
    g_status_ptr[dev] = static_cast<int*>(st);
  }
  *scratch = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  return MM4_OK;
}

}  // namespace

extern "C" {

mm4_status mm4_gemm_splitk_run_noalloc(const mm4_gemm_plan* p, const void* A, const void* B, const void* bias,
                                       void* C, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!A || !B || !C) return fail(MM4_ERR_INVALID, "null A/B/C pointer");
  if (p->d.bias && !bias) return fail(MM4_ERR_INVALID, "plan has bias but bias pointer is null");
  if (!p->d.bias) bias = nullptr;
  if (!p->tensor_core || p->splits <= 1)
    return fail(MM4_ERR_INVALID,
                "mm4_gemm_splitk_run_noalloc needs a tensor-core split-K plan (split_k > 1, 16-byte row pitches); "
                "this plan dispatches to %s",
                p->name);
  if (!aligned16(A) || !aligned16(B)) return fail(MM4_ERR_INVALID, "A and B must be 16-byte aligned");
  if (p->ws_bytes > MM4_NOALLOC_SCRATCH_BYTES)
    return fail(MM4_ERR_WORKSPACE,
                "split-K scratch of %zu bytes exceeds the no-alloc limit of %zu bytes (4 MiB); use mm4_gemm_run "
                "with a caller workspace",
                p->ws_bytes, MM4_NOALLOC_SCRATCH_BYTES);

  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  void* scratch = nullptr;
  int* status = nullptr;
  rc = setup_device(info.device, &scratch, &status);
  if (rc != MM4_OK) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The partial sums and arrival counters must start at zero.
  cudaError_t e = cudaMemsetAsync(scratch, 0, p->ws_bytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(no-alloc scratch)");

  CUtensorMap ta, tb;
  rc = gemm_build_maps(p, A, B, &ta, &tb);
  if (rc != MM4_OK) return rc;

  GemmArgs args{};
  gemm_plan_args(p, &args);
  args.bias = static_cast<const __half*>(bias);
  args.C = static_cast<__half*>(C);
  args.C32 = nullptr;
  args.ws = static_cast<float*>(scratch);
  args.counters = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + p->ws_counter_offset);
  args.coop_finalize = 0;  // the last-arriving unit of each tile finalizes it
  args.status = status;
  args.timeout_ns = wait_timeout_ns();
  return gemm_dispatch(p, MODE_SPLITK_F16, ta, tb, args, gemm_grid(p, args.num_units, info.sm_count), st);
}

}  // extern "C"

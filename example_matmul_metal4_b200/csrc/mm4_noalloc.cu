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
// device addresses of the scratch array and of this file's two status words
// with cudaGetSymbolAddress. Make that first call before any stream capture.
// The resolved addresses belong to the device's current context: do not use
// the entry point across a cudaDeviceReset on that device.
//
// Sharing: every call on a device uses the same scratch. Each call first runs
// a small prepare kernel on the caller's stream that clears the part it uses
// (the fp32 partial sums and the per-tile arrival counters must start at
// zero), so back-to-back calls on one stream are correct; calls that overlap
// on the GPU (different streams without ordering, or concurrent host threads)
// race on the scratch and give wrong results.
//
// Errors: device-side bounded waits end a stuck kernel and record
// MM4_ERR_TIMEOUT in this file's status word. The next call's prepare kernel
// moves that code into a second, "pending" word and clears the status word,
// so one run-out wait never makes later calls abort; mm4_check() reads and
// clears both words (and allocates nothing), which is how callers of this
// entry point learn about device-side errors.
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
static __device__ int g_noalloc_status;   // written by the bounded waits of the running call
static __device__ int g_noalloc_pending;  // first error of an earlier call, until mm4_check reads it

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
int* g_status_ptr[kMaxDevices] = {};
int* g_pending_ptr[kMaxDevices] = {};

// Resolves the device addresses of the static arrays for the current device
// (the host-side names are only stand-ins and must never reach a kernel).
mm4_status setup_device(int dev, void** scratch, int** status, int** pending) {
  if (dev < 0 || dev >= kMaxDevices) return fail(MM4_ERR_CUDA, "device id %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* s = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&s, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    void* st = nullptr;
    e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_status)");
    void* pd = nullptr;
    e = cudaGetSymbolAddress(&pd, g_noalloc_pending);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_pending)");
    g_status_ptr[dev] = static_cast<int*>(st);
    g_pending_ptr[dev] = static_cast<int*>(pd);
    g_scratch_ptr[dev] = s;  // set last: a non-null scratch pointer means all three are resolved
  }
  *scratch = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  *pending = g_pending_ptr[dev];
  return MM4_OK;
}

// Clears `words16` 16-byte words of the scratch and moves an error that an
// earlier call left in the status word into the pending word (keeping the
// oldest), so this call's waits start from a clean status.
__global__ void noalloc_prepare_kernel(uint4* scratch, size_t words16, int* status, int* pending) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int s = *status;
    if (s != 0) {
      if (*pending == 0) *pending = s;
      *status = 0;
    }
  }
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < words16; i += stride)
    scratch[i] = make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace

namespace mm4 {

// Called by mm4_check with the stream already synchronised: reads and clears
// the no-alloc status words of device `dev` (nothing to do if no no-alloc
// call ever ran there). Returns the older error first.
mm4_status noalloc_take_status(int dev, int* code) {
  *code = 0;
  int* status = nullptr;
  int* pending = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (dev < 0 || dev >= kMaxDevices || !g_scratch_ptr[dev]) return MM4_OK;
    status = g_status_ptr[dev];
    pending = g_pending_ptr[dev];
  }
  int v[2] = {0, 0};
  MM4_CUDA_TRY(cudaMemcpy(&v[0], pending, sizeof(int), cudaMemcpyDeviceToHost));
  MM4_CUDA_TRY(cudaMemcpy(&v[1], status, sizeof(int), cudaMemcpyDeviceToHost));
  if (v[0] != 0) MM4_CUDA_TRY(cudaMemset(pending, 0, sizeof(int)));
  if (v[1] != 0) MM4_CUDA_TRY(cudaMemset(status, 0, sizeof(int)));
  *code = v[0] != 0 ? v[0] : v[1];
  return MM4_OK;
}

}  // namespace mm4

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
  const size_t words16 = (p->ws_bytes + 15) / 16;
  if (words16 * 16 > MM4_NOALLOC_SCRATCH_BYTES)
    return fail(MM4_ERR_WORKSPACE,
                "split-K scratch of %zu bytes exceeds the no-alloc limit of %zu bytes (4 MiB); use mm4_gemm_run "
                "with a caller workspace",
                p->ws_bytes, MM4_NOALLOC_SCRATCH_BYTES);

  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  void* scratch = nullptr;
  int* status = nullptr;
  int* pending = nullptr;
  rc = setup_device(info.device, &scratch, &status, &pending);
  if (rc != MM4_OK) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The partial sums and arrival counters must start at zero, and the waits
  // of this call must not see an earlier call's error.
  const int prep_blocks = static_cast<int>(std::min<size_t>((words16 + 255) / 256, size_t(2) * info.sm_count));
  noalloc_prepare_kernel<<<std::max(prep_blocks, 1), 256, 0, st>>>(static_cast<uint4*>(scratch), words16, status,
                                                                   pending);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "noalloc_prepare_kernel launch");

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
  args.det_split_floats = p->det_split_floats;
  args.coop_finalize = 0;  // the last-arriving unit of each tile finalizes it
  args.status = status;
  args.timeout_ns = wait_timeout_ns();
  return gemm_dispatch(p, MODE_SPLITK_F16, ta, tb, args, gemm_grid(p, args.num_units, info.sm_count), st);
}

mm4_status mm4_debug_noalloc_wait_timeout(uint64_t timeout_ns, mm4_stream_t stream) {
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  void* scratch = nullptr;
  int* status = nullptr;
  int* pending = nullptr;
  rc = setup_device(info.device, &scratch, &status, &pending);
  if (rc != MM4_OK) return rc;
  return launch_debug_wait(status, timeout_ns, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// Host-side runtime shared by the mm4 translation units: error reporting,
// per-device status words, device properties and TMA descriptor encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "mm4.h"

namespace mm4 {

// Sets the thread-local message returned by mm4_last_error and returns `code`.
mm4_status fail(mm4_status code, const char* fmt, ...);
// Maps a CUDA error to MM4_ERR_CUDA with a message naming `what`.
mm4_status cuda_fail(cudaError_t err, const char* what);

#define MM4_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t mm4_e_ = (expr);                            \
    if (mm4_e_ != cudaSuccess) return ::mm4::cuda_fail(mm4_e_, #expr); \
  } while (0)

// Two library streams and a pool of events per device for the host-buffer
// entry points (copies in on `in`, copies out on `out`, the kernels on the
// caller's stream), created on first use and kept for the process.
constexpr int kHostMaxChunks = 64;
struct HostPipe {
  bool ready = false;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t start, end, loaded[kHostMaxChunks], done[kHostMaxChunks];
};
// The pipe of device `dev`; call with host_pipe_mutex() held for the whole
// enqueue of one call.
mm4_status host_pipe(int dev, HostPipe** out);
std::mutex& host_pipe_mutex();
// After an error part-way through an enqueue: orders `st` after whatever was
// already queued on the pipe's streams (best effort), so that synchronising
// `st` still means no copy of the call touches the caller's buffers any more.
void host_pipe_join(HostPipe* hp, cudaStream_t st);

// Current device id, its SM count and whether it is an sm_100 part.
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t smem_optin = 0;
};
mm4_status current_device(DeviceInfo* info);

// Device status word of the current device (lazily allocated, zeroed).
mm4_status status_word(int** ptr);
uint64_t wait_timeout_ns();

// Launches the one-warp bounded-wait test kernel on `word` (records
// MM4_ERR_TIMEOUT at wait site 99 after `timeout_ns`).
mm4_status launch_debug_wait(int* word, uint64_t timeout_ns, cudaStream_t stream);

// Reads and clears the allocation-free split-K entry point's status words on
// device `dev` (0 when that entry point never ran there); the caller has
// synchronised the stream. Defined in mm4_noalloc.cu.
mm4_status noalloc_take_status(int dev, int* code);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda, so the library loads on machines without a GPU).
mm4_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                        const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle swizzle);

// cuTensorMapEncodeIm2col: `pixels` pixels of `channels` channels per load,
// walking the spatial dims (innermost first, then the outermost dim) over the
// box [lower, dim - 1 + upper] of each spatial dim (corners given in the
// order of dims[1..rank-2]); element strides 1.
mm4_status encode_im2col(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                         const uint64_t* dims, const uint64_t* strides_bytes, const int* lower, const int* upper,
                         uint32_t channels, uint32_t pixels, CUtensorMapSwizzle swizzle);

// Sets cudaFuncAttributeMaxDynamicSharedMemorySize once per (kernel, device).
mm4_status ensure_smem_attr(const void* kernel, int bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mm4

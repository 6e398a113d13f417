// Host runtime of the mm4 C ABI: status codes, thread-local error messages,
// per-device status words read by mm4_check, TMA descriptor encoding, and
// the bounded-wait test hook.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <set>
#include <utility>

#include "mm4_internal.h"
#include "mm4_ptx.cuh"

namespace mm4 {

namespace {

thread_local char g_last_error[1024] = "";
std::atomic<uint64_t> g_timeout_ns{2000000000ull};

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int* g_status_words[kMaxDevices] = {};
DeviceInfo g_info[kMaxDevices];
bool g_info_valid[kMaxDevices] = {};
std::set<std::pair<const void*, int>> g_smem_set;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode_tiled = nullptr;
using EncodeIm2colFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeIm2colFn g_encode_im2col = nullptr;

}  // namespace

mm4_status fail(mm4_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

mm4_status cuda_fail(cudaError_t err, const char* what) {
  return fail(MM4_ERR_CUDA, "CUDA error %d (%s) in %s", static_cast<int>(err), cudaGetErrorString(err), what);
}

mm4_status current_device(DeviceInfo* info) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MM4_ERR_CUDA, "device id %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_info_valid[dev]) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    g_info[dev].device = dev;
    g_info[dev].sm_count = prop.multiProcessorCount;
    g_info[dev].cc_major = prop.major;
    g_info[dev].cc_minor = prop.minor;
    g_info[dev].smem_optin = prop.sharedMemPerBlockOptin;
    g_info_valid[dev] = true;
  }
  *info = g_info[dev];
  if (info->cc_major != 10)
    return fail(MM4_ERR_UNSUPPORTED, "device %d is sm_%d%d; the mm4 kernels are built for sm_100a only", dev,
                info->cc_major, info->cc_minor);
  return MM4_OK;
}

mm4_status status_word(int** ptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MM4_ERR_CUDA, "device id %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_status_words[dev]) {
    int* p = nullptr;
    e = cudaMalloc(&p, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status word)");
    e = cudaMemset(p, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status word)");
    g_status_words[dev] = p;
  }
  *ptr = g_status_words[dev];
  return MM4_OK;
}

uint64_t wait_timeout_ns() { return g_timeout_ns.load(); }

namespace {
constexpr int kHostMaxDevices = 64;
HostPipe g_host_pipe[kHostMaxDevices];
std::mutex g_host_mutex;
}  // namespace

std::mutex& host_pipe_mutex() { return g_host_mutex; }

mm4_status host_pipe(int dev, HostPipe** out) {
  if (dev < 0 || dev >= kHostMaxDevices) return fail(MM4_ERR_CUDA, "device id %d out of range", dev);
  HostPipe& hp = g_host_pipe[dev];
  if (!hp.ready) {
    MM4_CUDA_TRY(cudaStreamCreateWithFlags(&hp.in, cudaStreamNonBlocking));
    MM4_CUDA_TRY(cudaStreamCreateWithFlags(&hp.out, cudaStreamNonBlocking));
    MM4_CUDA_TRY(cudaEventCreateWithFlags(&hp.start, cudaEventDisableTiming));
    MM4_CUDA_TRY(cudaEventCreateWithFlags(&hp.end, cudaEventDisableTiming));
    for (int i = 0; i < kHostMaxChunks; ++i) {
      MM4_CUDA_TRY(cudaEventCreateWithFlags(&hp.loaded[i], cudaEventDisableTiming));
      MM4_CUDA_TRY(cudaEventCreateWithFlags(&hp.done[i], cudaEventDisableTiming));
    }
    hp.ready = true;
  }
  *out = &hp;
  return MM4_OK;
}

void host_pipe_join(HostPipe* hp, cudaStream_t st) {
  if (!hp || !hp->ready) return;
  if (cudaEventRecord(hp->start, hp->in) == cudaSuccess) (void)cudaStreamWaitEvent(st, hp->start, 0);
  if (cudaEventRecord(hp->end, hp->out) == cudaSuccess) (void)cudaStreamWaitEvent(st, hp->end, 0);
}

mm4_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                        const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_encode_tiled) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(MM4_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
      g_encode_tiled = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode_tiled(map, dtype, rank, const_cast<void*>(base), d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MM4_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return MM4_OK;
}

mm4_status encode_im2col(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                         const uint64_t* dims, const uint64_t* strides_bytes, const int* lower, const int* upper,
                         uint32_t channels, uint32_t pixels, CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_encode_im2col) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(MM4_ERR_CUDA, "cuTensorMapEncodeIm2col entry point unavailable");
      g_encode_im2col = reinterpret_cast<EncodeIm2colFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t es[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode_im2col(map, dtype, rank, const_cast<void*>(base), d, s, lower, upper, channels, pixels, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MM4_ERR_CUDA, "cuTensorMapEncodeIm2col failed (CUresult %d)", static_cast<int>(r));
  return MM4_OK;
}

mm4_status ensure_smem_attr(const void* kernel, int bytes) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mutex);
  auto key = std::make_pair(kernel, dev);
  if (g_smem_set.count(key)) return MM4_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  g_smem_set.insert(key);
  return MM4_OK;
}

// One warp waits on an mbarrier that nothing arrives at; the bounded wait
// records MM4_ERR_TIMEOUT (site 99) and the kernel returns normally.
__global__ void debug_wait_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const Watchdog wd{status, limit_ns};
    mbar_wait(&bar, 0, wd, 99);
  }
}

mm4_status launch_debug_wait(int* word, uint64_t timeout_ns, cudaStream_t stream) {
  debug_wait_kernel<<<1, 32, 0, stream>>>(word, timeout_ns);
  MM4_CUDA_TRY(cudaGetLastError());
  return MM4_OK;
}

}  // namespace mm4

using namespace mm4;

extern "C" {

int mm4_version(void) { return 100; }

const char* mm4_status_string(mm4_status s) {
  switch (s) {
    case MM4_OK: return "MM4_OK";
    case MM4_ERR_INVALID: return "MM4_ERR_INVALID";
    case MM4_ERR_UNSUPPORTED: return "MM4_ERR_UNSUPPORTED";
    case MM4_ERR_CUDA: return "MM4_ERR_CUDA";
    case MM4_ERR_NCCL: return "MM4_ERR_NCCL";
    case MM4_ERR_TIMEOUT: return "MM4_ERR_TIMEOUT";
    case MM4_ERR_WORKSPACE: return "MM4_ERR_WORKSPACE";
    default: return "MM4_ERR_UNKNOWN";
  }
}

const char* mm4_last_error(void) { return g_last_error; }

int mm4_device_supported(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  DeviceInfo info;
  return current_device(&info) == MM4_OK ? 1 : 0;
}

void mm4_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns); }
uint64_t mm4_get_wait_timeout_ns(void) { return g_timeout_ns.load(); }

mm4_status mm4_check(mm4_stream_t stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MM4_CUDA_TRY(cudaStreamSynchronize(st));
  MM4_CUDA_TRY(cudaGetLastError());
  int dev = -1;
  MM4_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(MM4_ERR_CUDA, "device id %d out of range", dev);
  // The library's word exists once a kernel that uses it was launched; before that there is nothing
  // to read, and mm4_check allocates nothing (callers of the allocation-free entry point rely on it).
  int* word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    word = g_status_words[dev];
  }
  int v = 0;
  if (word) {
    MM4_CUDA_TRY(cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) MM4_CUDA_TRY(cudaMemset(word, 0, sizeof(int)));
  }
  int nv = 0;
  mm4_status rc = noalloc_take_status(dev, &nv);
  if (rc != MM4_OK) return rc;
  if (v == 0) v = nv;
  if (v != 0) {
    const int code = v & 0xff;
    const int site = v >> 8;
    return fail(code, "device-side error %s recorded at wait site %d", mm4_status_string(code), site);
  }
  return MM4_OK;
}

mm4_status mm4_debug_wait_timeout(uint64_t timeout_ns, mm4_stream_t stream) {
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* word = nullptr;
  rc = status_word(&word);
  if (rc != MM4_OK) return rc;
  return launch_debug_wait(word, timeout_ns, static_cast<cudaStream_t>(stream));
}

mm4_status mm4_workspace_clear(void* workspace, size_t bytes, mm4_stream_t stream) {
  if (bytes == 0) return MM4_OK;
  if (!workspace) return fail(MM4_ERR_INVALID, "mm4_workspace_clear: null workspace");
  MM4_CUDA_TRY(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)));
  return MM4_OK;
}

}  // extern "C"

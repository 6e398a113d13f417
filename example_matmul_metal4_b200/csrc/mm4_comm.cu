// NCCL-bootstrapped communicator for the multi-GPU split-K: the C ABI that a
// caller with an NCCL unique id (MPI / a launcher store) binds, on top of the
// fused peer-memory group (mm4_group.cu). NCCL is only used at set-up time,
// to exchange the CUDA IPC handles of the exchange buffers and the root's C;
// every run is one fused launch per GPU. libnccl is loaded at run time
// (dlopen of libnccl.so.2, which resolves to the copy a host framework such
// as PyTorch already loaded), so libmm4.so has no link-time NCCL dependency.
// No reference counterpart (the reference is single-device); it replaces the
// distributed wrapper a multi-GPU port of matmul.swift:345-511 would add.
#include <dlfcn.h>

#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <vector>

#include "mm4_gemm_plan.h"
#include "mm4_internal.h"

using namespace mm4;

namespace {

// The public NCCL C API entry points used here (nccl.h).
struct NcclUniqueId {
  char internal[128];
};
using ncclComm_t = void*;
using NcclGetUniqueIdFn = int (*)(NcclUniqueId*);
using NcclCommInitRankFn = int (*)(ncclComm_t*, int, NcclUniqueId, int);
using NcclAllGatherFn = int (*)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t);
using NcclBroadcastFn = int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t);
using NcclCommDestroyFn = int (*)(ncclComm_t);
using NcclGetErrorStringFn = const char* (*)(int);
constexpr int kNcclUint8 = 1;

struct Nccl {
  bool loaded = false;
  NcclGetUniqueIdFn get_unique_id = nullptr;
  NcclCommInitRankFn comm_init_rank = nullptr;
  NcclAllGatherFn all_gather = nullptr;
  NcclBroadcastFn broadcast = nullptr;
  NcclCommDestroyFn comm_destroy = nullptr;
  NcclGetErrorStringFn error_string = nullptr;
};
Nccl g_nccl;
std::mutex g_nccl_mutex;

mm4_status load_nccl() {
  std::lock_guard<std::mutex> lock(g_nccl_mutex);
  if (g_nccl.loaded) return MM4_OK;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return fail(MM4_ERR_NCCL, "libnccl.so.2 could not be loaded: %s", dlerror());
  g_nccl.get_unique_id = reinterpret_cast<NcclGetUniqueIdFn>(dlsym(h, "ncclGetUniqueId"));
  g_nccl.comm_init_rank = reinterpret_cast<NcclCommInitRankFn>(dlsym(h, "ncclCommInitRank"));
  g_nccl.all_gather = reinterpret_cast<NcclAllGatherFn>(dlsym(h, "ncclAllGather"));
  g_nccl.broadcast = reinterpret_cast<NcclBroadcastFn>(dlsym(h, "ncclBroadcast"));
  g_nccl.comm_destroy = reinterpret_cast<NcclCommDestroyFn>(dlsym(h, "ncclCommDestroy"));
  g_nccl.error_string = reinterpret_cast<NcclGetErrorStringFn>(dlsym(h, "ncclGetErrorString"));
  if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.all_gather || !g_nccl.broadcast ||
      !g_nccl.comm_destroy)
    return fail(MM4_ERR_NCCL, "libnccl.so.2 lacks a required entry point");
  g_nccl.loaded = true;
  return MM4_OK;
}

mm4_status nccl_fail(int r, const char* what) {
  return fail(MM4_ERR_NCCL, "%s failed: NCCL error %d (%s)", what, r,
              g_nccl.error_string ? g_nccl.error_string(r) : "?");
}

struct GroupState {
  void* exchange = nullptr;          // own exchange buffer (peer memory)
  void* c_root = nullptr;            // root: own C buffer (peer memory)
  std::vector<void*> opened;         // peer mappings to close
  mm4_splitk_group* group = nullptr;
};

}  // namespace

struct mm4_comm {
  ncclComm_t nccl = nullptr;
  int nranks = 0, rank = 0, device = -1;
  void* scratch = nullptr;  // device buffer for handle exchange, nranks x 64 bytes + 64
  std::map<const mm4_gemm_plan*, GroupState> groups;
};

namespace {

// Collective over the communicator: every rank must call it for the same plan.
mm4_status setup_group(mm4_comm* c, const mm4_gemm_plan* plan, cudaStream_t st, GroupState* out) {
  GroupState gs;
  size_t bytes = 0;
  mm4_status rc = mm4_splitk_group_exchange_bytes(plan, c->nranks, &bytes);
  if (rc != MM4_OK) return rc;
  mm4_peer_handle h, hc;
  std::memset(&hc, 0, sizeof(hc));
  rc = mm4_peer_alloc(bytes, &gs.exchange, &h);
  if (rc == MM4_OK && c->rank == 0)
    rc = mm4_peer_alloc(static_cast<size_t>(plan->d.M) * plan->d.N * 2, &gs.c_root, &hc);
  if (rc != MM4_OK) {
    mm4_peer_free(gs.exchange);
    return rc;
  }
  // Gather every rank's exchange handle and broadcast the root's C handle.
  const size_t hb = sizeof(mm4_peer_handle);
  std::vector<mm4_peer_handle> all(c->nranks);
  char* dev = static_cast<char*>(c->scratch);
  cudaError_t e = cudaMemcpyAsync(dev + c->nranks * hb, &h, hb, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && c->rank == 0) e = cudaMemcpyAsync(dev + (c->nranks + 1) * hb, &hc, hb, cudaMemcpyHostToDevice, st);
  int r = 0;
  if (e == cudaSuccess) r = g_nccl.all_gather(dev + c->nranks * hb, dev, hb, kNcclUint8, c->nccl, st);
  if (e == cudaSuccess && r == 0)
    r = g_nccl.broadcast(dev + (c->nranks + 1) * hb, dev + (c->nranks + 1) * hb, hb, kNcclUint8, 0, c->nccl, st);
  if (e == cudaSuccess && r == 0) e = cudaMemcpyAsync(all.data(), dev, c->nranks * hb, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && r == 0) e = cudaMemcpyAsync(&hc, dev + (c->nranks + 1) * hb, hb, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && r == 0) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess || r != 0) {
    mm4_peer_free(gs.exchange);
    mm4_peer_free(gs.c_root);
    return e != cudaSuccess ? cuda_fail(e, "split-K group handle exchange") : nccl_fail(r, "handle exchange");
  }
  std::vector<void*> ptrs(c->nranks, nullptr);
  for (int i = 0; i < c->nranks && rc == MM4_OK; ++i) {
    if (i == c->rank) {
      ptrs[i] = gs.exchange;
    } else {
      rc = mm4_peer_open(&all[i], &ptrs[i]);
      if (rc == MM4_OK) gs.opened.push_back(ptrs[i]);
    }
  }
  void* c_root = gs.c_root;
  if (rc == MM4_OK && c->rank != 0) {
    rc = mm4_peer_open(&hc, &c_root);
    if (rc == MM4_OK) gs.opened.push_back(c_root);
  }
  if (rc == MM4_OK) rc = mm4_splitk_group_create(&gs.group, plan, c->nranks, c->rank, 0, ptrs.data(), c_root);
  if (rc != MM4_OK) {
    for (void* p : gs.opened) mm4_peer_close(p);
    mm4_peer_free(gs.exchange);
    mm4_peer_free(gs.c_root);
    return rc;
  }
  *out = gs;
  return MM4_OK;
}

// A stream-ordered barrier over the communicator (a one-byte all-gather).
mm4_status comm_barrier(mm4_comm* c) {
  char* dev = static_cast<char*>(c->scratch);
  int r = g_nccl.all_gather(dev + c->rank, dev, 1, kNcclUint8, c->nccl, nullptr);  // in place
  if (r != 0) return nccl_fail(r, "barrier");
  MM4_CUDA_TRY(cudaStreamSynchronize(nullptr));
  return MM4_OK;
}

}  // namespace

extern "C" {

mm4_status mm4_comm_unique_id(void* id) {
  if (!id) return fail(MM4_ERR_INVALID, "null id buffer");
  mm4_status rc = load_nccl();
  if (rc != MM4_OK) return rc;
  NcclUniqueId u;
  const int r = g_nccl.get_unique_id(&u);
  if (r != 0) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return MM4_OK;
}

mm4_status mm4_comm_init(mm4_comm** out, int32_t nranks, int32_t rank, const void* nccl_unique_id) {
  if (!out) return fail(MM4_ERR_INVALID, "null comm pointer");
  *out = nullptr;
  if (!nccl_unique_id) return fail(MM4_ERR_INVALID, "null NCCL unique id");
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks)
    return fail(MM4_ERR_INVALID, "rank %d of %d: 1..8 ranks are supported", rank, nranks);
  mm4_status rc = load_nccl();
  if (rc != MM4_OK) return rc;
  mm4_comm* c = new (std::nothrow) mm4_comm();
  if (!c) return fail(MM4_ERR_INVALID, "out of host memory");
  c->nranks = nranks;
  c->rank = rank;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->scratch, (nranks + 2) * sizeof(mm4_peer_handle));
  if (e != cudaSuccess) {
    delete c;
    return cuda_fail(e, "mm4_comm_init");
  }
  NcclUniqueId u;
  std::memcpy(&u, nccl_unique_id, sizeof(u));
  const int r = g_nccl.comm_init_rank(&c->nccl, nranks, u, rank);
  if (r != 0) {
    cudaFree(c->scratch);
    delete c;
    return nccl_fail(r, "ncclCommInitRank");
  }
  *out = c;
  return MM4_OK;
}

void mm4_comm_destroy(mm4_comm* c) {
  if (!c) return;
  if (!c->groups.empty()) {
    cudaDeviceSynchronize();
    comm_barrier(c);  // no rank still runs a kernel that maps our buffers
    for (auto& kv : c->groups) {
      mm4_splitk_group_destroy(kv.second.group);
      for (void* p : kv.second.opened) mm4_peer_close(p);
    }
    comm_barrier(c);  // every rank has unmapped before the owners free
    for (auto& kv : c->groups) {
      mm4_peer_free(kv.second.exchange);
      mm4_peer_free(kv.second.c_root);
    }
  }
  if (c->nccl) g_nccl.comm_destroy(c->nccl);
  cudaFree(c->scratch);
  delete c;
}

mm4_status mm4_gemm_splitk_run_distributed(const mm4_gemm_plan* plan, mm4_comm* c, const void* A, const void* B,
                                           const void* bias, void* C, mm4_stream_t stream, int duplicated_count) {
  if (!plan || !c) return fail(MM4_ERR_INVALID, "null plan or communicator");
  if (duplicated_count < 1) return fail(MM4_ERR_INVALID, "duplicated_count must be >= 1");
  if (c->rank == 0 && !C) return fail(MM4_ERR_INVALID, "the root needs an output C");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto it = c->groups.find(plan);
  if (it == c->groups.end()) {
    GroupState gs;
    mm4_status rc = setup_group(c, plan, st, &gs);
    if (rc != MM4_OK) return rc;
    it = c->groups.emplace(plan, gs).first;
  }
  for (int i = 0; i < duplicated_count; ++i) {
    mm4_status rc = mm4_gemm_splitk_group_run(plan, it->second.group, A, B, bias, stream);
    if (rc != MM4_OK) return rc;
  }
  if (c->rank == 0 && C != it->second.c_root) {
    MM4_CUDA_TRY(cudaMemcpyAsync(C, it->second.c_root, static_cast<size_t>(plan->d.M) * plan->d.N * 2,
                                 cudaMemcpyDeviceToDevice, st));
  }
  return MM4_OK;
}

}  // extern "C"

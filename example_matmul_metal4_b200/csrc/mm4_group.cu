// Multi-GPU split-K group: peer memory (CUDA IPC) and the fused
// compute + cross-GPU reduction entry point. One process per GPU; every rank
// runs the same plan on its own K shard and the fp32 partials meet inside the
// kernels' epilogues over peer memory (see SplitKGroupArgs), so a run is one
// launch per GPU with no separate collective. The reference is single-device;
// this replaces the NCCL reduce of the K-shard partials a multi-GPU port would
// place after the per-split partial of matmul.swift:127-185.
#include <cstdlib>
#include <cstring>
#include <new>

#include "gemm_sm100.cuh"
#include "mm4_gemm_plan.h"
#include "mm4_internal.h"

using namespace mm4;

static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(mm4_peer_handle), "IPC handle does not fit mm4_peer_handle");

struct mm4_splitk_group {
  int world, rank, root, owner_mode;
  int num_slices;
  size_t half_bytes;  // one staging half (world slots)
  size_t slot_bytes;  // one rank's slot of a half
  unsigned long long epoch;
  char* exchange[MM4_MAX_GROUP];
  unsigned long long* ready[MM4_MAX_GROUP];
  unsigned long long* consumed[MM4_MAX_GROUP];
  unsigned long long* done;
  __half* c_root;
  void* scratch;      // rank-local split-K scratch (the plan's workspace), owned by the group
  int device;
  // plan geometry the group was sized for
  int M, N, splits, num_tiles, halves;
  size_t ws_bytes;
};

namespace {

// Exchange buffer of one rank: staging half 0 | half 1 (each [world slots]
// [stage_rows][ws_ld] fp32, slots and halves 256-aligned) | ready
// [num_slices][world] u64 | consumed [num_slices] u64 | done [num_slices] u64
// (used on the root). Rank r pushes the slices an owner finishes into slot r
// of the owner's half.
struct ExchangeLayout {
  size_t slot_bytes, half_bytes, ready_offset, consumed_offset, done_offset, total;
};

ExchangeLayout exchange_layout(const mm4_gemm_plan* p, int world) {
  ExchangeLayout L;
  const int halves = p->pair ? 2 : 1;
  const size_t num_slices = static_cast<size_t>(p->num_tiles) * halves * p->splits;
  const size_t stage_rows = static_cast<size_t>(p->num_m_tiles) * (p->pair ? 256 : 128);
  const size_t ws_ld = static_cast<size_t>(p->num_n_tiles) * p->bn;
  L.slot_bytes = (stage_rows * ws_ld * sizeof(float) + 255) & ~static_cast<size_t>(255);
  L.half_bytes = L.slot_bytes * static_cast<size_t>(world);
  L.ready_offset = 2 * L.half_bytes;
  L.consumed_offset = L.ready_offset + num_slices * world * sizeof(unsigned long long);
  L.done_offset = L.consumed_offset + num_slices * sizeof(unsigned long long);
  L.total = L.done_offset + num_slices * sizeof(unsigned long long);
  return L;
}

mm4_status check_group_plan(const mm4_gemm_plan* p, int world) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (world < 1 || world > MM4_MAX_GROUP)
    return fail(MM4_ERR_UNSUPPORTED, "group size %d: 1..%d ranks are supported", world, MM4_MAX_GROUP);
  if (!p->tensor_core || p->splits < 2)
    return fail(MM4_ERR_UNSUPPORTED, "a split-K group needs a tensor-core split-K plan (got %s)", p->name);
  return MM4_OK;
}

// Which ranks finish the slices. The root alone (default): one hop, the
// other ranks push (world-1) partials into the root over NVLink. Spread
// (MM4_SPLITK_GROUP_OWNERS=spread): rank slice % world finishes the slice,
// receiving (world-1)/world of the partials, then writes the root's C and
// raises a done flag there, a second hop. Measured on B200 with the earlier
// pull design (512x512, K 65536 per rank, split 32): root 56.5 / 63.7 us per
// step at 2 / 4 ranks, spread 67.2 / 73.9 us.
int choose_owner_mode(int /*world*/) {
  const char* v = std::getenv("MM4_SPLITK_GROUP_OWNERS");
  if (v && std::strcmp(v, "spread") == 0) return 1;
  return 0;
}

}  // namespace

extern "C" {

mm4_status mm4_peer_alloc(size_t bytes, void** ptr, mm4_peer_handle* handle) {
  if (!ptr || !handle) return fail(MM4_ERR_INVALID, "null output pointer");
  *ptr = nullptr;
  if (bytes == 0) return fail(MM4_ERR_INVALID, "zero-byte peer allocation");
  void* p = nullptr;
  MM4_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "mm4_peer_alloc");
  }
  std::memset(handle, 0, sizeof(*handle));
  std::memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return MM4_OK;
}

mm4_status mm4_peer_free(void* ptr) {
  if (!ptr) return MM4_OK;
  MM4_CUDA_TRY(cudaFree(ptr));
  return MM4_OK;
}

mm4_status mm4_peer_open(const mm4_peer_handle* handle, void** ptr) {
  if (!ptr || !handle) return fail(MM4_ERR_INVALID, "null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  MM4_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MM4_OK;
}

mm4_status mm4_peer_close(void* ptr) {
  if (!ptr) return MM4_OK;
  MM4_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return MM4_OK;
}

mm4_status mm4_splitk_group_exchange_bytes(const mm4_gemm_plan* plan, int32_t world, size_t* bytes) {
  if (!bytes) return fail(MM4_ERR_INVALID, "null output pointer");
  *bytes = 0;
  mm4_status rc = check_group_plan(plan, world);
  if (rc != MM4_OK) return rc;
  *bytes = exchange_layout(plan, world).total;
  return MM4_OK;
}

mm4_status mm4_splitk_group_create(mm4_splitk_group** out, const mm4_gemm_plan* plan, int32_t world, int32_t rank,
                                   int32_t root, void* const* exchange, void* c_root) {
  if (!out) return fail(MM4_ERR_INVALID, "null group pointer");
  *out = nullptr;
  mm4_status rc = check_group_plan(plan, world);
  if (rc != MM4_OK) return rc;
  if (rank < 0 || rank >= world || root < 0 || root >= world)
    return fail(MM4_ERR_INVALID, "rank %d / root %d outside a group of %d", rank, root, world);
  if (!exchange || !c_root) return fail(MM4_ERR_INVALID, "null exchange buffers or root output");
  if ((reinterpret_cast<uintptr_t>(c_root) & 7u) != 0) return fail(MM4_ERR_INVALID, "root C must be 8-byte aligned");
  for (int r = 0; r < world; ++r)
    if (!exchange[r] || (reinterpret_cast<uintptr_t>(exchange[r]) & 255u) != 0)
      return fail(MM4_ERR_INVALID, "exchange[%d] null or not 256-byte aligned", r);
  mm4_splitk_group* g = new (std::nothrow) mm4_splitk_group();
  if (!g) return fail(MM4_ERR_INVALID, "out of host memory");
  // Rank-local split-K scratch: plain device memory (the partial sums are
  // reduced into it with L2 atomics; only finished slices are shared).
  cudaError_t e = cudaGetDevice(&g->device);
  if (e == cudaSuccess) e = cudaMalloc(&g->scratch, plan->ws_bytes);
  if (e == cudaSuccess) e = cudaMemset(g->scratch, 0, plan->ws_bytes);
  if (e != cudaSuccess) {
    if (g->scratch) cudaFree(g->scratch);
    delete g;
    return cuda_fail(e, "split-K group scratch");
  }
  const ExchangeLayout L = exchange_layout(plan, world);
  g->world = world;
  g->rank = rank;
  g->root = root;
  g->owner_mode = choose_owner_mode(world);
  g->halves = plan->pair ? 2 : 1;
  g->num_slices = plan->num_tiles * g->halves * plan->splits;
  g->half_bytes = L.half_bytes;
  g->slot_bytes = L.slot_bytes;
  g->epoch = 0;
  for (int r = 0; r < world; ++r) {
    char* base = static_cast<char*>(exchange[r]);
    g->exchange[r] = base;
    g->ready[r] = reinterpret_cast<unsigned long long*>(base + L.ready_offset);
    g->consumed[r] = reinterpret_cast<unsigned long long*>(base + L.consumed_offset);
  }
  g->done = reinterpret_cast<unsigned long long*>(static_cast<char*>(exchange[root]) + L.done_offset);
  g->c_root = static_cast<__half*>(c_root);
  g->M = plan->d.M;
  g->N = plan->d.N;
  g->splits = plan->splits;
  g->num_tiles = plan->num_tiles;
  g->ws_bytes = plan->ws_bytes;
  *out = g;
  return MM4_OK;
}

void mm4_splitk_group_destroy(mm4_splitk_group* g) {
  if (!g) return;
  if (g->scratch) {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != g->device) cudaSetDevice(g->device);
    cudaFree(g->scratch);
    if (cur != g->device && cur >= 0) cudaSetDevice(cur);
  }
  delete g;
}

mm4_status mm4_gemm_splitk_group_run(const mm4_gemm_plan* plan, mm4_splitk_group* g, const void* A, const void* B,
                                     const void* bias, mm4_stream_t stream) {
  if (!plan || !g) return fail(MM4_ERR_INVALID, "null plan or group");
  if (!A || !B) return fail(MM4_ERR_INVALID, "null A/B pointer");
  if (plan->d.M != g->M || plan->d.N != g->N || plan->splits != g->splits || plan->num_tiles != g->num_tiles ||
      (plan->pair ? 2 : 1) != g->halves || plan->ws_bytes != g->ws_bytes)
    return fail(MM4_ERR_INVALID, "plan does not match the plan the group was created for");
  if (!aligned16(A) || !aligned16(B)) return fail(MM4_ERR_INVALID, "A and B must be 16-byte aligned");
  SplitKGroupArgs ga{};
  ga.world = g->world;
  ga.rank = g->rank;
  ga.root = g->root;
  ga.owner_mode = g->owner_mode;
  ga.num_slices = g->num_slices;
  ga.epoch = g->epoch;
  ga.slot_floats = static_cast<long long>(g->slot_bytes / sizeof(float));
  const size_t half = static_cast<size_t>(g->epoch & 1ull) * g->half_bytes;
  for (int r = 0; r < g->world; ++r) {
    ga.stage[r] = reinterpret_cast<float*>(g->exchange[r] + half);
    ga.ready[r] = g->ready[r];
    ga.consumed[r] = g->consumed[r];
  }
  ga.done = g->done;
  ga.c_root = g->c_root;
  mm4_status rc = gemm_run_tc(plan, A, B, bias, g->c_root, nullptr, g->scratch, g->ws_bytes,
                              static_cast<cudaStream_t>(stream), &ga);
  if (rc == MM4_OK) ++g->epoch;
  return rc;
}

}  // extern "C"

/*
 * mm4 — B200 (sm_100a) tensor-op contraction library, C ABI.
 *
 * This is the drop-in boundary for the tensor-op contraction path of
 * liuliu/example_matmul_metal4: the generated matmul2d GEMM (bias, split-K,
 * dynamic K), the flash-attention forward, and conv2d / conv3d (with and
 * without padding). The reference exposes that path as Swift descriptor
 * structs + MSL source generators + Metal "sessions"; the entries below take
 * the same descriptors and run hand-written CUDA kernels instead.
 *
 * Conventions
 *  - Every call returns an mm4_status; nothing throws and nothing aborts.
 *    mm4_last_error() gives a thread-local message for the last failure.
 *  - The caller owns every device buffer (inputs, outputs, workspace). Plans
 *    own only kernel choice and shape-derived constants; they are immutable
 *    after create and may be used concurrently on different streams.
 *  - Launches are stream-ordered and do not block. `duplicated_count`
 *    repeats the launch, like the reference's duplicatedCount.
 *  - Kernels never hang: every device-side wait is bounded. A wait that runs
 *    out records MM4_ERR_TIMEOUT in a per-device status word, read (and
 *    cleared) by mm4_check().
 *  - There is no CPU fallback: without a usable sm_100 device every compute
 *    entry returns MM4_ERR_CUDA / MM4_ERR_UNSUPPORTED.
 *  - All tensors are fp16 (IEEE binary16) unless stated; accumulation is fp32.
 */
#ifndef MM4_H
#define MM4_H

#include <stddef.h>
#include <stdint.h>

#include "mm4_status_codes.h"

#if defined(__GNUC__)
#define MM4_API __attribute__((visibility("default")))
#else
#define MM4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int mm4_status; /* one of the MM4_OK / MM4_ERR_* codes */
typedef void* mm4_stream_t; /* a cudaStream_t; NULL is the legacy default stream */

/* Library version (major*10000 + minor*100 + patch). */
MM4_API int mm4_version(void);
/* Human-readable name of a status code. */
MM4_API const char* mm4_status_string(mm4_status status);
/* Thread-local message describing the most recent failure on this thread. */
MM4_API const char* mm4_last_error(void);
/* 1 when the current CUDA device is an sm_100 part the kernels can run on. */
MM4_API int mm4_device_supported(void);

/* Synchronises `stream`, then reads and clears the current device's status
 * words: the library's own, and the two of mm4_gemm_splitk_run_noalloc.
 * Returns MM4_ERR_TIMEOUT when a kernel recorded a run-out wait (the
 * message names the wait site), MM4_ERR_CUDA on a CUDA error, else MM4_OK.
 * It allocates no device memory. */
MM4_API mm4_status mm4_check(mm4_stream_t stream);

/* Upper bound, in nanoseconds, for any single device-side wait (default
 * 2e9 = 2 s). Applies to launches made after the call. */
MM4_API void mm4_set_wait_timeout_ns(uint64_t ns);
MM4_API uint64_t mm4_get_wait_timeout_ns(void);

/* Test hook for the failure path: launches a one-warp kernel that waits on an
 * mbarrier nothing ever arrives at, bounded by `timeout_ns`. The kernel
 * records MM4_ERR_TIMEOUT and returns, so a following mm4_check() reports it
 * and the context stays usable. No reference counterpart (the reference
 * calls fatalError on a failed command buffer, ConvolutionShared.swift:955-958). */
MM4_API mm4_status mm4_debug_wait_timeout(uint64_t timeout_ns, mm4_stream_t stream);

/* Test hook for the attention forward's softmax exponentials: y[i] = 2^x[i]
 * for i < n (fp32 device vectors) by the hardware ex2.approx (method 0) or
 * by the kernel's FMA-pipe cubic (method 1; inputs clamped at -125). No
 * reference counterpart (the reference's softmax uses the Metal exp2,
 * attention.swift:24). */
MM4_API mm4_status mm4_debug_ex2(const float* x, float* y, int64_t n, int method, mm4_stream_t stream);

/* Stream-ordered memset to zero (e.g. first-time split-K workspace init). */
MM4_API mm4_status mm4_workspace_clear(void* workspace, size_t bytes, mm4_stream_t stream);

/* ======================================================================== */
/* GEMM: C[M,N] = A * B (+ bias[N])                                         */
/* ======================================================================== */

/* Replaces GEMMDimensions + BuildOptions + createSource(matrixDimensions:
 * blockDimensions:transpose:bias:buildOptions:) and run(M:N:K:...)
 * (Sources/matmul/matmul.swift:5-16, :18-329, :345-511).
 *  transpose_left  = 0: A stored [M][K] (K contiguous)   — reference default
 *                  = 1: A stored [K][M]
 *  transpose_right = 1: B stored [N][K]                  — reference default
 *                  = 0: B stored [K][N] (row-major NN, the BASELINE layout)
 *  C is stored [M][N] row-major, fp16. bias (if set) is fp16 [N].
 *  split_k > 1 splits the K loop over split_k CTAs; fp32 partials are reduced
 *  in-kernel (needs the workspace), then bias-added and stored as fp16.
 *  block_m/n/k, cooperative/preemptive simdgroups and swap_mn are the
 *  reference's tuning knobs: accepted, validated (>= 0), and used only as
 *  hints — the sm_100 tile is chosen by the dispatcher. */
typedef struct mm4_gemm_desc {
  int32_t M, N, K;
  int32_t transpose_left;
  int32_t transpose_right;
  int32_t bias;
  int32_t split_k;
  int32_t block_m, block_n, block_k;
  int32_t cooperative_simdgroups;
  int32_t preemptive_simdgroups;
  int32_t swap_mn;
} mm4_gemm_desc;

typedef struct mm4_gemm_plan mm4_gemm_plan;

MM4_API mm4_status mm4_gemm_plan_create(mm4_gemm_plan** plan, const mm4_gemm_desc* desc);
MM4_API void mm4_gemm_plan_destroy(mm4_gemm_plan* plan);

/* C = A * B (+ bias) from and to host memory (page-locked for the copies to
 * overlap), through the caller's device buffers dA, dB, dbias, dC of the
 * plan's full sizes and the plan's workspace. B and bias are copied in
 * first; then, for `chunks` blocks of 256-row multiples of A and C (<= 0: 16;
 * one when A is stored [K][M]), the copy of A's rows, the GEMM on them and the
 * copy of C's rows out run as a pipeline on `stream` and two library streams.
 * Each block runs as a GEMM of its own height, so a split-K plan's blocks may
 * differ from one whole-problem run in the last fp32 bit; direct plans give
 * mm4_gemm_run's bits. Ordering and errors as for mm4_attention_fwd_host. */
MM4_API mm4_status mm4_gemm_run_host(const mm4_gemm_plan* plan, const void* hA, const void* hB, const void* hbias,
                                     void* hC, void* dA, void* dB, void* dbias, void* dC, void* workspace,
                                     size_t workspace_bytes, int32_t chunks, mm4_stream_t stream);

/* Bytes of device workspace mm4_gemm_run needs (0 when split_k <= 1). The
 * workspace must be zero-filled before its first use (mm4_workspace_clear);
 * every run leaves it zero-filled again. Runs sharing a workspace must not
 * overlap on the GPU. */
MM4_API size_t mm4_gemm_workspace_size(const mm4_gemm_plan* plan);

/* Describes the kernel the plan dispatches to (static string). */
MM4_API const char* mm4_gemm_plan_kernel_name(const mm4_gemm_plan* plan);

/* C = A*B (+bias). Replaces matmul.swift run(...) dispatch + reduce_sum_2
 * (matmul.swift:438-474). */
MM4_API mm4_status mm4_gemm_run(const mm4_gemm_plan* plan, const void* A, const void* B, const void* bias, void* C,
                        void* workspace, size_t workspace_bytes, mm4_stream_t stream, int duplicated_count);

/* K-shard partial: C32[M][N] (fp32) = A*B over this call's K only, no bias,
 * no rounding. Used by the multi-GPU split-K path, where each rank owns a K
 * shard and the fp32 partials are summed across ranks before
 * mm4_splitk_finalize. No reference counterpart (the reference is
 * single-device); its role is the per-split partial of matmul.swift:127-185. */
MM4_API mm4_status mm4_gemm_partial_run(const mm4_gemm_plan* plan, const void* A, const void* B, float* C32,
                                void* workspace, size_t workspace_bytes, mm4_stream_t stream);

/* C[M][N] (fp16) = C32 + bias[N] (bias may be NULL). The bias/cast step the
 * reference folds into split 0 (matmul.swift:21-38). */
MM4_API mm4_status mm4_splitk_finalize(int32_t M, int32_t N, const float* C32, const void* bias, void* C,
                               mm4_stream_t stream);

/* Split-K GEMM that allocates no device memory: C = A*B (+bias) like
 * mm4_gemm_run, for callers that cannot call cudaMalloc where they issue the
 * GEMM (a framework allocator that owns all GPU memory, real-time or serving
 * loops where an allocation may stall or fail, plug-in hosts that only pass
 * in their input/output buffers). No reference counterpart: the reference
 * allocates its split-K output buffer per run (matmul.swift:395-400).
 * The fp32 partial-sum scratch is a static 4 MiB device array inside the
 * library (held on every device that loads it until exit); plans whose
 * mm4_gemm_workspace_size() exceeds 4 MiB, or that are not tensor-core
 * split-K plans, are rejected. The first call on a device resolves the
 * array's device address (make it before any stream capture; do not use the
 * entry point across a cudaDeviceReset of that device). Each call clears the
 * scratch it uses on `stream`; calls that overlap on the GPU share the
 * scratch and race. A device-side wait that runs out in one call is kept for
 * mm4_check() (which reports and clears it) and does not affect later calls. */
MM4_API mm4_status mm4_gemm_splitk_run_noalloc(const mm4_gemm_plan* plan, const void* A, const void* B,
                                               const void* bias, void* C, mm4_stream_t stream);
/* Test hook for the entry point above: one warp waits, bounded by
 * `timeout_ns`, on an mbarrier nothing arrives at and records MM4_ERR_TIMEOUT
 * in the no-alloc status word, as a run-out wait of a no-alloc call would.
 * No reference counterpart. */
MM4_API mm4_status mm4_debug_noalloc_wait_timeout(uint64_t timeout_ns, mm4_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU split-K: one process per GPU, fused compute + cross-GPU reduce  */
/* ------------------------------------------------------------------------ */

/* Device memory another process on this node can map (CUDA IPC), zero-filled.
 * The handle is plain bytes to pass between processes (e.g. through
 * torch.distributed.all_gather_object). No reference counterpart (the
 * reference is single-device). */
typedef struct mm4_peer_handle {
  unsigned char bytes[64];
} mm4_peer_handle;
MM4_API mm4_status mm4_peer_alloc(size_t bytes, void** ptr, mm4_peer_handle* handle);
MM4_API mm4_status mm4_peer_free(void* ptr);
MM4_API mm4_status mm4_peer_open(const mm4_peer_handle* handle, void** ptr);
MM4_API mm4_status mm4_peer_close(void* ptr);

/* A group of `world` ranks (<= 8) running one split-K plan, each on its own K
 * shard (same M, N, shard K, split_k on every rank), whose fp32 partials are
 * summed inside the kernels over peer memory. Each rank publishes its
 * finished fp32 slices of C into its exchange buffer; the owner of each slice
 * (the root; slice % world with MM4_SPLITK_GROUP_OWNERS=spread) reads the
 * ranks' rows of the slice from there, sums them in rank order, adds bias,
 * rounds to fp16 and writes the rows into the root's C. One launch per
 * GPU and no separate collective; the root's launch completes when all of C
 * is written. Replaces the NCCL reduce a multi-GPU port would put after the
 * per-split partials of matmul.swift:127-185 + the bias/cast of :21-38.
 *
 * Every rank allocates an exchange buffer of mm4_splitk_group_exchange_bytes()
 * with mm4_peer_alloc; the root also allocates C [M][N] fp16 with
 * mm4_peer_alloc. exchange[r] is rank r's buffer as mapped in this process
 * (mm4_peer_open; this rank's own pointer at [rank]); c_root likewise. Every
 * rank must make the same sequence of mm4_gemm_splitk_group_run calls. The
 * plan must give one CTA (pair) per (split, M-tile) on the device (split_k x
 * M-tiles <= the SM count, or half of it for 256-row tiles). */
typedef struct mm4_splitk_group mm4_splitk_group;
MM4_API mm4_status mm4_splitk_group_exchange_bytes(const mm4_gemm_plan* plan, int32_t world, size_t* bytes);
MM4_API mm4_status mm4_splitk_group_create(mm4_splitk_group** group, const mm4_gemm_plan* plan, int32_t world,
                                           int32_t rank, int32_t root, void* const* exchange, void* c_root);
MM4_API void mm4_splitk_group_destroy(mm4_splitk_group* group);
MM4_API mm4_status mm4_gemm_splitk_group_run(const mm4_gemm_plan* plan, mm4_splitk_group* group, const void* A,
                                             const void* B, const void* bias, mm4_stream_t stream);

/* Communicator form of the same fused multi-GPU split-K, bootstrapped from an
 * NCCL unique id (rank 0 calls mm4_comm_unique_id and hands the 128 bytes to
 * every rank, e.g. over MPI or a launcher store). mm4_comm_init creates the
 * NCCL communicator (libnccl.so.2 is loaded at run time); the first
 * mm4_gemm_splitk_run_distributed call for a plan is collective and sets up
 * the plan's split-K group over it (exchange buffers, IPC handle exchange);
 * later calls are one fused launch per GPU. Every rank passes its own K shard
 * (A [M][K_r], B [K_r][N]) and the same bias; rank 0 receives C [M][N] fp16
 * (other ranks may pass C = NULL). mm4_comm_destroy is collective. */
typedef struct mm4_comm mm4_comm;
MM4_API mm4_status mm4_comm_unique_id(void* nccl_unique_id /* 128 bytes */);
MM4_API mm4_status mm4_comm_init(mm4_comm** comm, int32_t nranks, int32_t rank, const void* nccl_unique_id);
MM4_API void mm4_comm_destroy(mm4_comm* comm);
MM4_API mm4_status mm4_gemm_splitk_run_distributed(const mm4_gemm_plan* plan, mm4_comm* comm, const void* A,
                                                   const void* B, const void* bias, void* C, mm4_stream_t stream,
                                                   int duplicated_count);

/* ======================================================================== */
/* Flash-attention forward and backward                                     */
/* ======================================================================== */

/* Replaces AttentionDimensions / BlockDimenions / BuildOptions + the
 * `attention` kernel generator and run(...) (Sources/attention/
 * attention.swift:4-21, :23-382, :398-541). Non-causal softmax(Q K^T *
 * scale) V with an fp32 online softmax; O is fp16.
 *  rows = R (query length), columns = C (key/value length), head_dim = D:
 *  128 (the reference's) or 64 (run(...) takes it as a parameter,
 *  attention.swift:398); other values return MM4_ERR_UNSUPPORTED.
 *  layout MM4_ATTN_BHSD: tensors [batch][heads][seq][D] (BASELINE);
 *         MM4_ATTN_BSHD: tensors [batch][seq][heads][D] (the reference's
 *         [S][H][D] packing, attention.swift:463-471, with batch outermost).
 *  heads_kv must divide heads_q (grouped-query attention when smaller).
 *  scale <= 0 selects 1/sqrt(D) (Network.swift:153). */
enum { MM4_ATTN_BHSD = 0, MM4_ATTN_BSHD = 1 };

typedef struct mm4_attention_desc {
  int32_t batch;
  int32_t heads_q, heads_kv;
  int32_t rows, columns;
  int32_t head_dim;
  float scale;
  int32_t layout;
} mm4_attention_desc;

typedef struct mm4_attention_plan mm4_attention_plan;

MM4_API mm4_status mm4_attention_plan_create(mm4_attention_plan** plan, const mm4_attention_desc* desc);
MM4_API void mm4_attention_plan_destroy(mm4_attention_plan* plan);
MM4_API const char* mm4_attention_plan_kernel_name(const mm4_attention_plan* plan);
MM4_API mm4_status mm4_attention_fwd(const mm4_attention_plan* plan, const void* Q, const void* K, const void* V, void* O,
                             mm4_stream_t stream, int duplicated_count);

/* Forward that also writes each query row's log-sum-exp, lse[b][h][row] =
 * log(sum_c exp(scale * S[row][c])) (natural log; Network.swift createLTerm,
 * :181-203), fp32 [batch][heads_q][rows], for the backward below. */
MM4_API mm4_status mm4_attention_fwd_lse(const mm4_attention_plan* plan, const void* Q, const void* K, const void* V,
                                         void* O, float* lse, mm4_stream_t stream);

/* Forward from and to host memory: Q, K, V are read from hQ, hK, hV and O
 * is written to hO (host buffers; page-locked for the copies to overlap),
 * through the caller's device buffers dQ, dK, dV, dO of the plan's full
 * sizes. The (batch, head) units are cut into `chunks` pieces (<= 0: 16; at
 * most 64; whole key/value heads with their query heads in [B][H][S][D],
 * whole batch elements in [B][S][H][D]) and run as a pipeline on `stream`
 * and two library streams: copies in, the kernel, copies out, so the
 * transfers in both directions overlap each other and the kernels. The
 * reference's buffers are host-visible (Apple unified memory); this is the
 * call for callers whose tensors live on the host. Ordered on `stream`:
 * work queued on it before the call precedes the copies, and later work
 * follows the last copy out. Results equal mm4_attention_fwd's bit for
 * bit. A call that fails part-way still orders `stream` after every copy it
 * queued, so synchronising `stream` before freeing the buffers stays safe. */
MM4_API mm4_status mm4_attention_fwd_host(const mm4_attention_plan* plan, const void* hQ, const void* hK,
                                          const void* hV, void* hO, void* dQ, void* dK, void* dV, void* dO,
                                          int32_t chunks, mm4_stream_t stream);

/* Attention backward. The reference has it only as CPU code
 * (Network.swift:205-401: derivativeQ / derivativeK / derivativeV of the
 * loss sum(dO * O)); this is its GPU form. Inputs: Q, K, V, the forward's O
 * and lse (mm4_attention_fwd_lse), and dO, all in the plan's layout; outputs
 * dQ, dK, dV (fp16, same layouts as Q, K, V; with heads_kv < heads_q, dK and
 * dV sum over the query heads sharing a key/value head). workspace: at least
 * mm4_attention_bwd_workspace_size(plan) bytes, 16-byte aligned, any
 * contents. Three stream-ordered launches. */
MM4_API size_t mm4_attention_bwd_workspace_size(const mm4_attention_plan* plan);
MM4_API mm4_status mm4_attention_bwd(const mm4_attention_plan* plan, const void* Q, const void* K, const void* V,
                                     const void* O, const void* dO, const float* lse, void* dQ, void* dK, void* dV,
                                     void* workspace, size_t workspace_bytes, mm4_stream_t stream);

/* Backward from and to host memory, as mm4_attention_fwd_host for the
 * forward: host_in = {Q, K, V, O, dO, lse} and host_out = {dQ, dK, dV} are
 * host buffers (page-locked for overlap); dev_in / dev_out the caller's
 * device buffers of the same full sizes; workspace as for mm4_attention_bwd.
 * Chunks of whole key/value heads (with their query heads, [B][H][S][D]) or
 * batch elements ([B][S][H][D]) are copied in, differentiated and copied out
 * as a pipeline. Results equal mm4_attention_bwd's bit for bit. */
MM4_API mm4_status mm4_attention_bwd_host(const mm4_attention_plan* plan, const void* const* host_in,
                                          void* const* host_out, void* const* dev_in, void* const* dev_out,
                                          void* workspace, size_t workspace_bytes, int32_t chunks,
                                          mm4_stream_t stream);

/* ======================================================================== */
/* Convolution (implicit GEMM)                                              */
/* ======================================================================== */

/* Weight layouts. The reference consumes HWIO / DHWIO (ConvolutionShared.swift
 * weightIndex, :4848-4860, :4920-4930) and permutes from OIDHW
 * (:4593-4629); the BASELINE configs store weights [Cout][k...][Cin]. */
enum {
  MM4_WEIGHTS_HWIO = 0,  /* 2-D: [KH][KW][Cin][Cout] */
  MM4_WEIGHTS_OHWI = 1,  /* 2-D: [Cout][KH][KW][Cin] */
  MM4_WEIGHTS_OIHW = 2,  /* 2-D: [Cout][Cin][KH][KW] (permute source only) */
  MM4_WEIGHTS_DHWIO = 3, /* 3-D: [KD][KH][KW][Cin][Cout] */
  MM4_WEIGHTS_ODHWI = 4, /* 3-D: [Cout][KD][KH][KW][Cin] */
  MM4_WEIGHTS_OIDHW = 5  /* 3-D: [Cout][Cin][KD][KH][KW] (permute source only) */
};

/* Conv2DDimensions (ConvolutionShared.swift:5-70), NHWC activations, NHWC
 * output [N][OH][OW][Cout]; output size follows :56-62. */
typedef struct mm4_conv2d_desc {
  int32_t batch_size;
  int32_t input_height, input_width;
  int32_t input_channels, output_channels;
  int32_t kernel_height, kernel_width;
  int32_t stride_y, stride_x;
  int32_t dilation_y, dilation_x;
  int32_t padding_top, padding_bottom, padding_left, padding_right;
  int32_t weight_layout; /* MM4_WEIGHTS_HWIO or MM4_WEIGHTS_OHWI */
  int32_t bias;          /* add bias[Cout] */
} mm4_conv2d_desc;

/* Conv3DDimensions (ConvolutionShared.swift:72-153), NDHWC activations and
 * output. padding_front/back (depth padding) is an extension: the reference
 * has none (:135-137), and 0 reproduces it exactly. */
typedef struct mm4_conv3d_desc {
  int32_t batch_size;
  int32_t input_depth, input_height, input_width;
  int32_t input_channels, output_channels;
  int32_t kernel_depth, kernel_height, kernel_width;
  int32_t stride_z, stride_y, stride_x;
  int32_t dilation_z, dilation_y, dilation_x;
  int32_t padding_top, padding_bottom, padding_left, padding_right;
  int32_t padding_front, padding_back;
  int32_t weight_layout; /* MM4_WEIGHTS_DHWIO or MM4_WEIGHTS_ODHWI */
  int32_t bias;
} mm4_conv3d_desc;

typedef struct mm4_conv_plan mm4_conv_plan;

/* Replaces TensorOpSession / the padded conv2d probe session
 * (ConvolutionShared.swift:844-988; convolution2d_padding.swift:235-290). */
MM4_API mm4_status mm4_conv2d_plan_create(mm4_conv_plan** plan, const mm4_conv2d_desc* desc);
/* Replaces TensorOpSession3D / TensorOpBiasSession3D /
 * TensorOpHorizontalPaddingSession3D (ConvolutionShared.swift:990-1575) —
 * one launch instead of N*OD*KD host-orchestrated slices. */
MM4_API mm4_status mm4_conv3d_plan_create(mm4_conv_plan** plan, const mm4_conv3d_desc* desc);
MM4_API void mm4_conv_plan_destroy(mm4_conv_plan* plan);
MM4_API const char* mm4_conv_plan_kernel_name(const mm4_conv_plan* plan);
/* Output tiles the plan launches over (assuming 16-byte-aligned operands):
 * grid[0] along output pixels (tiles of 128, or 256 for CTA pairs; virtual
 * rows OW + KW - 1 wide when the kw taps share one activation box), grid[1]
 * along output channels, grid[2] = 1. The analogue of the reference's
 * threadgroup dispatch grid (tensorOpDispatchThreadgroups,
 * ConvolutionShared.swift:938); host-only. */
MM4_API mm4_status mm4_conv_plan_tile_grid(const mm4_conv_plan* plan, int32_t grid[3]);
/* Output element count of the plan (N*OD*OH*OW*Cout). */
MM4_API int64_t mm4_conv_output_elements(const mm4_conv_plan* plan);
/* y = conv(x, w) (+ bias) from and to host memory (page-locked for the
 * copies to overlap), through the caller's device buffers of the plan's
 * full sizes: the weights and bias are copied in first, then `chunks` groups
 * of whole batch elements (<= 0: 16) are copied in, convolved and copied out
 * as a pipeline on `stream` and two library streams. Each output pixel is
 * computed as in mm4_conv_run. Ordering and errors as for
 * mm4_attention_fwd_host. */
MM4_API mm4_status mm4_conv_run_host(const mm4_conv_plan* plan, const void* hx, const void* hw, const void* hbias,
                                     void* hy, void* dx, void* dw, void* dbias, void* dy, int32_t chunks,
                                     mm4_stream_t stream);
/* y = conv(x, w) (+ bias). */
MM4_API mm4_status mm4_conv_run(const mm4_conv_plan* plan, const void* x, const void* w, const void* bias, void* y,
                        mm4_stream_t stream, int duplicated_count);

/* Weight layout transform (K10): permute_oidhw_to_dhwio and its 2-D
 * analogues (ConvolutionShared.swift:4593-4629, :1577-1675).
 * dims = {Cout, Cin, KD, KH, KW}; KD = 1 for 2-D layouts. Supported pairs:
 * any of the 2-D layouts to any other 2-D layout, any 3-D to any 3-D. */
MM4_API mm4_status mm4_permute_weights(int from_layout, int to_layout, const int32_t dims[5], const void* src, void* dst,
                               mm4_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MM4_H */

// Convolution plans and dispatch (conv2d / conv3d as one implicit-GEMM
// launch) and the weight-layout permutation.
//
// Replaces TensorOpSession / TensorOpSession3D / TensorOpBiasSession3D /
// TensorOpHorizontalPaddingSession3D / WeightPermutationSession3D
// (ConvolutionShared.swift:844-1675) and the padded conv2d probe session
// (convolution2d_padding.swift:235-290).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "conv_sm100.cuh"
#include "conv_sm100_pair.cuh"
#include "mm4_internal.h"

using namespace mm4;

struct mm4_conv_plan {
  ConvGeom g;  // pointers filled per run
  int bias;
  int bn;
  long long m_total;
  int num_m_tiles, num_n_tiles;
  bool w_tma_shape;  // weight pitch allows TMA (pointer alignment checked per run)
  bool w_mn;         // HWIO / DHWIO: Cout contiguous
  bool x_tma_shape;  // stride 1 and 16-byte channel pitch: activations by TMA
  int a_mode;        // CONV_A_IM2COL or CONV_A_RECT on the TMA path
  bool pair;         // im2col path on 2-CTA clusters (256-pixel tiles)
  bool taprow;       // pair path reading all kw taps from one box per (kd, kh, slab)
  int vw;            // taprow: virtual row width OW + KW - 1
  long long m_virtual;  // taprow: N * OD * OH * vw tile rows
  int tw, th;        // output rectangle per tile on the rectangle path (tw * th = 128)
  int tiles_w, tiles_h;
  int dims;            // 2 or 3: the descriptor the plan was created from
  mm4_conv2d_desc d2;  // (for plans of a batch chunk, mm4_conv_run_host)
  mm4_conv3d_desc d3;
  char name[96];
};

namespace {

int out_size(int in, int plo, int phi, int k, int s, int d) { return (in + plo + phi - ((k - 1) * d + 1)) / s + 1; }

mm4_status finish_plan(mm4_conv_plan* p) {
  ConvGeom& g = p->g;
  if (g.OD <= 0 || g.OH <= 0 || g.OW <= 0)
    return fail(MM4_ERR_INVALID, "convolution output is empty (OD=%d OH=%d OW=%d)", g.OD, g.OH, g.OW);
  g.ncb = (g.C + 63) / 64;
  g.taps = g.KD * g.KH * g.KW;
  p->m_total = static_cast<long long>(g.N) * g.OD * g.OH * g.OW;
  if (p->m_total > (1ll << 31) - 256) return fail(MM4_ERR_UNSUPPORTED, "too many output pixels");
  p->bn = g.O <= 128 ? 128 : 256;
  p->num_m_tiles = static_cast<int>((p->m_total + GEMM_BM - 1) / GEMM_BM);
  p->num_n_tiles = (g.O + p->bn - 1) / p->bn;
  p->w_mn = (g.w_layout == MM4_WEIGHTS_HWIO || g.w_layout == MM4_WEIGHTS_DHWIO);
  p->w_tma_shape = p->w_mn ? (g.O % 8 == 0) : (g.C % 8 == 0);
  p->x_tma_shape = p->w_tma_shape && g.C % 8 == 0 && g.SX == 1 && g.SY == 1 && g.SZ == 1;
  p->tw = g.OW > 32 ? 64 : g.OW > 16 ? 32 : g.OW > 8 ? 16 : 8;
  p->th = GEMM_BM / p->tw;
  p->tiles_w = (g.OW + p->tw - 1) / p->tw;
  p->tiles_h = (g.OH + p->th - 1) / p->th;
  // im2col tiles are 128 consecutive output pixels: no lanes lost to a
  // rectangle that overhangs the output width, and the fewest tiles (the
  // last wave is the fullest). Its 5-D window box corners must fit in 5 bits
  // signed and the tap offsets in 5 bits; the rectangle path covers the rest
  // (MM4_CONV_ACTIVATIONS=rect forces it).
  const int lo[3] = {-g.PL, -g.PT, -g.PF};
  const int hi[3] = {g.OW - g.PL - g.W, g.OH - g.PT - g.H, g.OD - g.PF - g.D};
  const int span[3] = {(g.KW - 1) * g.DX, (g.KH - 1) * g.DY, (g.KD - 1) * g.DZ};
  bool im2col_ok = true;
  for (int i = 0; i < 3; ++i)
    im2col_ok = im2col_ok && lo[i] >= -16 && lo[i] <= 15 && hi[i] >= -16 && hi[i] <= 15 && span[i] <= 31;
  const char* force = std::getenv("MM4_CONV_ACTIVATIONS");
  if (force && std::strcmp(force, "rect") == 0) im2col_ok = false;
  p->a_mode = im2col_ok ? CONV_A_IM2COL : CONV_A_RECT;
  // CTA pairs on the im2col path (MM4_CONV_PAIR=0 keeps one-CTA tiles).
  const char* pair_env = std::getenv("MM4_CONV_PAIR");
  p->pair = p->x_tma_shape && p->a_mode == CONV_A_IM2COL && !(pair_env && pair_env[0] == '0');
  // Tap rows on the pair path (MM4_CONV_TAPREUSE=0 keeps one box per tap):
  // dilation-1 filters 2 or 3 taps wide, with the widened window box's
  // upper W corner still in 5 bits signed.
  p->vw = g.OW + g.KW - 1;
  p->m_virtual = static_cast<long long>(g.N) * g.OD * g.OH * p->vw;
  const int vw_upper = p->vw - g.PL - g.W;
  const char* tap_env = std::getenv("MM4_CONV_TAPREUSE");
  p->taprow = p->pair && g.DX == 1 && g.KW >= 2 && g.KW <= CONV_ROW_MAX_KW && vw_upper >= -16 && vw_upper <= 15 &&
              p->m_virtual <= (1ll << 31) - 512 && !(tap_env && tap_env[0] == '0');
  snprintf(p->name, sizeof(p->name), "conv_sm100%s<BN=%d,%s,%s>", p->pair ? "_pair" : "", p->bn,
           p->w_tma_shape ? (p->w_mn ? "W:tma-MN" : "W:tma-K") : "W:gather",
           p->x_tma_shape ? (p->a_mode == CONV_A_IM2COL ? (p->taprow ? "X:tma-im2col-taprow" : "X:tma-im2col")
                                                       : "X:tma-rect")
                          : (g.C % 8 == 0) ? "X:cp.async16" : "X:gather16");
  return MM4_OK;
}

template <int BN, bool B_TMA, bool B_MN, int A_MODE>
mm4_status launch(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& args, const ConvGeom& g, int grid,
                  cudaStream_t st) {
  auto kern = conv_sm100_kernel<BN, B_TMA, B_MN, A_MODE>;
  constexpr int smem = GemmCfg<BN>::SMEM_BYTES;
  mm4_status rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (rc != MM4_OK) return rc;
  kern<<<grid, CONV_THREADS, smem, st>>>(tw, tx, args, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "conv_sm100_kernel launch");
  return MM4_OK;
}

template <int BN, bool B_MN, bool TAPROW>
mm4_status launch_pair(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& args, const ConvGeom& g,
                       int grid, cudaStream_t st) {
  auto kern = conv_sm100_pair_kernel<BN, B_MN, TAPROW>;
  constexpr int smem = ConvPairCfg<BN, TAPROW>::SMEM_BYTES;
  mm4_status rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (rc != MM4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, args, g);
  if (e != cudaSuccess) return cuda_fail(e, "conv_sm100_pair_kernel launch");
  return MM4_OK;
}

template <int BN>
mm4_status launch_bn(bool wtma, bool mn, int amode, const CUtensorMap& tw, const CUtensorMap& tx,
                     const GemmArgs& args, const ConvGeom& g, int grid, cudaStream_t st) {
  if (!wtma) return launch<BN, false, false, CONV_A_GATHER>(tw, tx, args, g, grid, st);
  if (amode == CONV_A_IM2COL) {
    if (mn) return launch<BN, true, true, CONV_A_IM2COL>(tw, tx, args, g, grid, st);
    return launch<BN, true, false, CONV_A_IM2COL>(tw, tx, args, g, grid, st);
  }
  if (amode == CONV_A_RECT) {
    if (mn) return launch<BN, true, true, CONV_A_RECT>(tw, tx, args, g, grid, st);
    return launch<BN, true, false, CONV_A_RECT>(tw, tx, args, g, grid, st);
  }
  if (mn) return launch<BN, true, true, CONV_A_GATHER>(tw, tx, args, g, grid, st);
  return launch<BN, true, false, CONV_A_GATHER>(tw, tx, args, g, grid, st);
}

mm4_status check_layout_2d(int layout) {
  if (layout != MM4_WEIGHTS_HWIO && layout != MM4_WEIGHTS_OHWI)
    return fail(MM4_ERR_INVALID, "conv2d weight_layout must be MM4_WEIGHTS_HWIO or MM4_WEIGHTS_OHWI (got %d)", layout);
  return MM4_OK;
}

mm4_status check_layout_3d(int layout) {
  if (layout != MM4_WEIGHTS_DHWIO && layout != MM4_WEIGHTS_ODHWI)
    return fail(MM4_ERR_INVALID, "conv3d weight_layout must be MM4_WEIGHTS_DHWIO or MM4_WEIGHTS_ODHWI (got %d)",
                layout);
  return MM4_OK;
}

}  // namespace

extern "C" {

mm4_status mm4_conv2d_plan_create(mm4_conv_plan** out, const mm4_conv2d_desc* d) {
  if (!out) return fail(MM4_ERR_INVALID, "null plan pointer");
  *out = nullptr;
  if (!d) return fail(MM4_ERR_INVALID, "null conv2d descriptor");
  if (d->batch_size <= 0 || d->input_height <= 0 || d->input_width <= 0 || d->input_channels <= 0 ||
      d->output_channels <= 0 || d->kernel_height <= 0 || d->kernel_width <= 0 || d->stride_y <= 0 ||
      d->stride_x <= 0 || d->dilation_y <= 0 || d->dilation_x <= 0 || d->padding_top < 0 || d->padding_bottom < 0 ||
      d->padding_left < 0 || d->padding_right < 0)
    return fail(MM4_ERR_INVALID, "conv2d dimensions must be positive and paddings non-negative");
  mm4_status rc = check_layout_2d(d->weight_layout);
  if (rc != MM4_OK) return rc;
  mm4_conv_plan* p = new (std::nothrow) mm4_conv_plan();
  if (!p) return fail(MM4_ERR_INVALID, "out of host memory");
  ConvGeom& g = p->g;
  g.N = d->batch_size;
  g.D = 1;
  g.H = d->input_height;
  g.W = d->input_width;
  g.C = d->input_channels;
  g.O = d->output_channels;
  g.KD = 1;
  g.KH = d->kernel_height;
  g.KW = d->kernel_width;
  g.SZ = 1;
  g.SY = d->stride_y;
  g.SX = d->stride_x;
  g.DZ = 1;
  g.DY = d->dilation_y;
  g.DX = d->dilation_x;
  g.PF = 0;
  g.PT = d->padding_top;
  g.PL = d->padding_left;
  g.OD = 1;
  g.OH = out_size(g.H, d->padding_top, d->padding_bottom, g.KH, g.SY, g.DY);
  g.OW = out_size(g.W, d->padding_left, d->padding_right, g.KW, g.SX, g.DX);
  g.w_layout = d->weight_layout;
  p->bias = d->bias ? 1 : 0;
  p->dims = 2;
  p->d2 = *d;
  rc = finish_plan(p);
  if (rc != MM4_OK) {
    delete p;
    return rc;
  }
  *out = p;
  return MM4_OK;
}

mm4_status mm4_conv3d_plan_create(mm4_conv_plan** out, const mm4_conv3d_desc* d) {
  if (!out) return fail(MM4_ERR_INVALID, "null plan pointer");
  *out = nullptr;
  if (!d) return fail(MM4_ERR_INVALID, "null conv3d descriptor");
  if (d->batch_size <= 0 || d->input_depth <= 0 || d->input_height <= 0 || d->input_width <= 0 ||
      d->input_channels <= 0 || d->output_channels <= 0 || d->kernel_depth <= 0 || d->kernel_height <= 0 ||
      d->kernel_width <= 0 || d->stride_z <= 0 || d->stride_y <= 0 || d->stride_x <= 0 || d->dilation_z <= 0 ||
      d->dilation_y <= 0 || d->dilation_x <= 0 || d->padding_top < 0 || d->padding_bottom < 0 ||
      d->padding_left < 0 || d->padding_right < 0 || d->padding_front < 0 || d->padding_back < 0)
    return fail(MM4_ERR_INVALID, "conv3d dimensions must be positive and paddings non-negative");
  mm4_status rc = check_layout_3d(d->weight_layout);
  if (rc != MM4_OK) return rc;
  mm4_conv_plan* p = new (std::nothrow) mm4_conv_plan();
  if (!p) return fail(MM4_ERR_INVALID, "out of host memory");
  ConvGeom& g = p->g;
  g.N = d->batch_size;
  g.D = d->input_depth;
  g.H = d->input_height;
  g.W = d->input_width;
  g.C = d->input_channels;
  g.O = d->output_channels;
  g.KD = d->kernel_depth;
  g.KH = d->kernel_height;
  g.KW = d->kernel_width;
  g.SZ = d->stride_z;
  g.SY = d->stride_y;
  g.SX = d->stride_x;
  g.DZ = d->dilation_z;
  g.DY = d->dilation_y;
  g.DX = d->dilation_x;
  g.PF = d->padding_front;
  g.PT = d->padding_top;
  g.PL = d->padding_left;
  g.OD = out_size(g.D, d->padding_front, d->padding_back, g.KD, g.SZ, g.DZ);
  g.OH = out_size(g.H, d->padding_top, d->padding_bottom, g.KH, g.SY, g.DY);
  g.OW = out_size(g.W, d->padding_left, d->padding_right, g.KW, g.SX, g.DX);
  g.w_layout = d->weight_layout;
  p->bias = d->bias ? 1 : 0;
  p->dims = 3;
  p->d3 = *d;
  rc = finish_plan(p);
  if (rc != MM4_OK) {
    delete p;
    return rc;
  }
  *out = p;
  return MM4_OK;
}

void mm4_conv_plan_destroy(mm4_conv_plan* plan) { delete plan; }

const char* mm4_conv_plan_kernel_name(const mm4_conv_plan* plan) { return plan ? plan->name : ""; }

mm4_status mm4_conv_plan_tile_grid(const mm4_conv_plan* p, int32_t grid[3]) {
  if (!p || !grid) return fail(MM4_ERR_INVALID, "null plan or grid");
  const long long rows = p->taprow ? p->m_virtual : p->m_total;
  const int tile_m = p->pair ? 2 * GEMM_BM : GEMM_BM;
  grid[0] = p->a_mode == CONV_A_RECT && p->x_tma_shape && !p->pair
                ? p->g.N * p->g.OD * p->tiles_h * p->tiles_w
                : static_cast<int32_t>((rows + tile_m - 1) / tile_m);
  grid[1] = p->num_n_tiles;
  grid[2] = 1;
  return MM4_OK;
}

int64_t mm4_conv_output_elements(const mm4_conv_plan* plan) {
  return plan ? plan->m_total * plan->g.O : 0;
}

mm4_status mm4_conv_run_host(const mm4_conv_plan* p, const void* hx, const void* hw, const void* hbias, void* hy,
                             void* dx, void* dw, void* dbias, void* dy, int32_t chunks, mm4_stream_t stream) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!hx || !hw || !hy || !dx || !dw || !dy) return fail(MM4_ERR_INVALID, "null buffer pointer");
  if (p->bias && (!hbias || !dbias)) return fail(MM4_ERR_INVALID, "plan has bias but a bias pointer is null");
  const ConvGeom& g = p->g;
  const size_t x_img = static_cast<size_t>(g.D) * g.H * g.W * g.C * 2;
  const size_t y_img = static_cast<size_t>(g.OD) * g.OH * g.OW * g.O * 2;
  const size_t w_bytes = static_cast<size_t>(g.taps) * g.C * g.O * 2, b_bytes = static_cast<size_t>(g.O) * 2;
  int n = chunks > 0 ? chunks : 16;
  n = std::max(1, std::min(std::min(n, kHostMaxChunks), g.N));
  const int per = (g.N + n - 1) / n;
  n = (g.N + per - 1) / per;
  const int last = g.N - (n - 1) * per;
  // Plans of the chunk batch sizes (all but the last share one).
  mm4_conv_plan* sub[2] = {nullptr, nullptr};
  auto cleanup = [&]() {
    for (auto*& q : sub)
      if (q) {
        mm4_conv_plan_destroy(q);
        q = nullptr;
      }
  };
  for (int i = 0; i < 2; ++i) {
    const int nb = i == 0 ? std::min(per, g.N) : last;
    mm4_status rc;
    if (p->dims == 2) {
      mm4_conv2d_desc d = p->d2;
      d.batch_size = nb;
      rc = mm4_conv2d_plan_create(&sub[i], &d);
    } else {
      mm4_conv3d_desc d = p->d3;
      d.batch_size = nb;
      rc = mm4_conv3d_plan_create(&sub[i], &d);
    }
    if (rc != MM4_OK) {
      cleanup();
      return rc;
    }
  }
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
    // Weights and bias first: every chunk needs them whole.
    MM4_CUDA_TRY(cudaMemcpyAsync(dw, hw, w_bytes, cudaMemcpyHostToDevice, hp->in));
    if (p->bias) MM4_CUDA_TRY(cudaMemcpyAsync(dbias, hbias, b_bytes, cudaMemcpyHostToDevice, hp->in));
    for (int c = 0; c < n; ++c) {
      const int nb = c == n - 1 ? last : per;
      const size_t xo = static_cast<size_t>(c) * per * x_img, yo = static_cast<size_t>(c) * per * y_img;
      MM4_CUDA_TRY(cudaMemcpyAsync(at(dx, xo), at(hx, xo), nb * x_img, cudaMemcpyHostToDevice, hp->in));
      MM4_CUDA_TRY(cudaEventRecord(hp->loaded[c], hp->in));
      MM4_CUDA_TRY(cudaStreamWaitEvent(st, hp->loaded[c], 0));
      mm4_status r = mm4_conv_run(c == n - 1 ? sub[1] : sub[0], at(dx, xo), dw, p->bias ? dbias : nullptr,
                                  at(dy, yo), stream, 1);
      if (r != MM4_OK) return r;
      MM4_CUDA_TRY(cudaEventRecord(hp->done[c], st));
      MM4_CUDA_TRY(cudaStreamWaitEvent(hp->out, hp->done[c], 0));
      MM4_CUDA_TRY(cudaMemcpyAsync(at(hy, yo), at(dy, yo), nb * y_img, cudaMemcpyDeviceToHost, hp->out));
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

mm4_status mm4_conv_run(const mm4_conv_plan* p, const void* x, const void* w, const void* bias, void* y,
                        mm4_stream_t stream, int duplicated_count) {
  if (!p) return fail(MM4_ERR_INVALID, "null plan");
  if (!x || !w || !y) return fail(MM4_ERR_INVALID, "null x/w/y pointer");
  if (p->bias && !bias) return fail(MM4_ERR_INVALID, "plan has bias but bias pointer is null");
  if (duplicated_count < 1) return fail(MM4_ERR_INVALID, "duplicated_count must be >= 1");
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  int* status = nullptr;
  rc = status_word(&status);
  if (rc != MM4_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  ConvGeom g = p->g;
  g.x = static_cast<const __half*>(x);
  g.w = static_cast<const __half*>(w);
  g.x_vec = (g.C % 8 == 0) && aligned16(x);
  const bool tma = p->w_tma_shape && aligned16(w);

  CUtensorMap tm;
  memset(&tm, 0, sizeof(tm));
  if (tma) {
    if (!p->w_mn) {  // [Cout][taps][Cin]
      const uint64_t dims[3] = {static_cast<uint64_t>(g.C), static_cast<uint64_t>(g.taps),
                                static_cast<uint64_t>(g.O)};
      const uint64_t strides[2] = {static_cast<uint64_t>(g.C) * 2, static_cast<uint64_t>(g.taps) * g.C * 2};
      const uint32_t box[3] = {64, 1, static_cast<uint32_t>(p->pair ? p->bn / 2 : p->bn)};
      rc = encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {  // [taps][Cin][Cout]
      const uint64_t dims[3] = {static_cast<uint64_t>(g.O), static_cast<uint64_t>(g.C),
                                static_cast<uint64_t>(g.taps)};
      const uint64_t strides[2] = {static_cast<uint64_t>(g.O) * 2, static_cast<uint64_t>(g.C) * g.O * 2};
      const uint32_t box[3] = {64, 64, 1};
      rc = encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc != MM4_OK) return rc;
  }
  const bool xtma = tma && p->x_tma_shape && aligned16(x);
  const int amode = xtma ? p->a_mode : CONV_A_GATHER;
  const bool pair = xtma && p->pair;
  const bool taprow = pair && p->taprow;
  CUtensorMap tx;
  memset(&tx, 0, sizeof(tx));
  if (xtma) {  // NDHWC activations
    const uint64_t dims[5] = {static_cast<uint64_t>(g.C), static_cast<uint64_t>(g.W), static_cast<uint64_t>(g.H),
                              static_cast<uint64_t>(g.D), static_cast<uint64_t>(g.N)};
    const uint64_t strides[4] = {static_cast<uint64_t>(g.C) * 2, static_cast<uint64_t>(g.W) * g.C * 2,
                                 static_cast<uint64_t>(g.H) * g.W * g.C * 2,
                                 static_cast<uint64_t>(g.D) * g.H * g.W * g.C * 2};
    if (amode == CONV_A_IM2COL) {
      // Window box of output pixel (ox, oy, oz): input origin (ox - PL, ...);
      // the box walks origins [-PL, W - 1 + (OW - PL - W)] = OW positions
      // per row (tap rows: vw = OW + KW - 1 positions, and KW - 1 more pixels
      // per box).
      const int row_w = taprow ? p->vw : g.OW;
      const int lower[3] = {-g.PL, -g.PT, -g.PF};
      const int upper[3] = {row_w - g.PL - g.W, g.OH - g.PT - g.H, g.OD - g.PF - g.D};
      const int pixels = taprow ? GEMM_BM + g.KW - 1 : GEMM_BM;
      rc = encode_im2col(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, x, dims, strides, lower, upper, 64, pixels,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    } else {  // box {64 ch, TW, TH, 1, 1}
      const uint32_t box[5] = {64, static_cast<uint32_t>(p->tw), static_cast<uint32_t>(p->th), 1, 1};
      rc = encode_tiled(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc != MM4_OK) return rc;
  }

  GemmArgs args{};
  args.M = static_cast<int>(p->m_total);
  args.N = g.O;
  args.K = g.taps * g.C;
  args.num_m_tiles = p->num_m_tiles;
  if (amode == CONV_A_RECT) {
    args.rowmap = 1;
    args.rm_tw = p->tw;
    args.rm_th = p->th;
    args.rm_tiles_w = p->tiles_w;
    args.rm_tiles_h = p->tiles_h;
    args.rm_od = g.OD;
    args.rm_oh = g.OH;
    args.rm_ow = g.OW;
    args.num_m_tiles = g.N * g.OD * p->tiles_h * p->tiles_w;
  }
  if (pair) args.num_m_tiles = static_cast<int>((p->m_total + 2 * GEMM_BM - 1) / (2 * GEMM_BM));
  args.kb_total = g.taps * g.ncb;
  if (taprow) {
    args.M = static_cast<int>(p->m_virtual);
    args.rowmap = 2;
    args.rm_vw = p->vw;
    args.rm_vrows = g.N * g.OD * g.OH;
    args.rm_ow = g.OW;
    args.num_m_tiles = static_cast<int>((p->m_virtual + 2 * GEMM_BM - 1) / (2 * GEMM_BM));
    args.kb_total = g.KD * g.KH * g.ncb;  // one k-block per (kd, kh, slab), KW taps each
  }
  args.num_n_tiles = p->num_n_tiles;
  args.num_tiles = args.num_m_tiles * p->num_n_tiles;
  args.splits = 1;
  args.num_units = args.num_tiles;
  args.group_m = 16;
  args.bias = p->bias ? static_cast<const __half*>(bias) : nullptr;
  args.C = static_cast<__half*>(y);
  args.status = status;
  args.timeout_ns = wait_timeout_ns();
  const int grid = pair ? 2 * std::min(args.num_units, info.sm_count / 2) : std::min(args.num_units, info.sm_count);
  for (int i = 0; i < duplicated_count; ++i) {
    if (taprow) {
      if (p->bn == 256)
        rc = p->w_mn ? launch_pair<256, true, true>(tm, tx, args, g, grid, st)
                     : launch_pair<256, false, true>(tm, tx, args, g, grid, st);
      else
        rc = p->w_mn ? launch_pair<128, true, true>(tm, tx, args, g, grid, st)
                     : launch_pair<128, false, true>(tm, tx, args, g, grid, st);
    } else if (pair) {
      if (p->bn == 256)
        rc = p->w_mn ? launch_pair<256, true, false>(tm, tx, args, g, grid, st)
                     : launch_pair<256, false, false>(tm, tx, args, g, grid, st);
      else
        rc = p->w_mn ? launch_pair<128, true, false>(tm, tx, args, g, grid, st)
                     : launch_pair<128, false, false>(tm, tx, args, g, grid, st);
    } else {
      rc = (p->bn == 256) ? launch_bn<256>(tma, p->w_mn, amode, tm, tx, args, g, grid, st)
                          : launch_bn<128>(tma, p->w_mn, amode, tm, tx, args, g, grid, st);
    }
    if (rc != MM4_OK) return rc;
  }
  return MM4_OK;
}

mm4_status mm4_permute_weights(int from, int to, const int32_t dims[5], const void* src, void* dst,
                               mm4_stream_t stream) {
  if (!dims || !src || !dst) return fail(MM4_ERR_INVALID, "null argument");
  const bool from2 = from >= 0 && from <= 2, to2 = to >= 0 && to <= 2;
  const bool from3 = from >= 3 && from <= 5, to3 = to >= 3 && to <= 5;
  if (!((from2 && to2) || (from3 && to3)))
    return fail(MM4_ERR_INVALID, "permute needs two 2-D or two 3-D weight layouts (got %d -> %d)", from, to);
  const int O = dims[0], C = dims[1], KD = dims[2], KH = dims[3], KW = dims[4];
  if (O <= 0 || C <= 0 || KD <= 0 || KH <= 0 || KW <= 0) return fail(MM4_ERR_INVALID, "dims must be positive");
  if (from2 && KD != 1) return fail(MM4_ERR_INVALID, "2-D layouts need KD == 1");
  if (src == dst) return fail(MM4_ERR_INVALID, "permute cannot run in place");
  DeviceInfo info;
  mm4_status rc = current_device(&info);
  if (rc != MM4_OK) return rc;
  const long long total = static_cast<long long>(O) * C * KD * KH * KW;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(info.sm_count) * 16));
  permute_weights_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      from, to, O, C, KD, KH, KW, static_cast<const unsigned short*>(src), static_cast<unsigned short*>(dst));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "permute_weights_kernel launch");
  return MM4_OK;
}

}  // extern "C"

// Reduced-alignment GEMM used only where the tensor-core kernel cannot be fed
// by TMA: a K-major operand whose row pitch is not a multiple of 16 bytes
// (K % 8 != 0, e.g. the reference's K = 1/31/33 sweep points,
// matmul.swift:338-343) or an operand pointer that is not 16-byte aligned.
// TMA requires 16-byte-aligned global strides and base addresses; rather than
// copying such inputs into padded buffers this kernel reads them directly.
//
// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread, fp32
// accumulation in ascending k (the order of the reference's CPU loop,
// matmul.swift:499-510). Split-K is a scheduling knob and is not applied here.
#pragma once

#include <cuda_fp16.h>

namespace mm4 {

template <bool OUT_F32>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* __restrict__ A, long long a_sm, long long a_sk,
                                                        const __half* __restrict__ B, long long b_sk, long long b_sn,
                                                        const __half* __restrict__ bias, void* __restrict__ Cv, int M,
                                                        int N, int K) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tx = threadIdx.x & 15;
  const int ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64;
  const int n0 = blockIdx.x * 64;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i >> 6, mm = i & 63;
      const int gk = k0 + kk;
      const int gm = m0 + mm, gn = n0 + mm;
      As[kk][mm] = (gm < M && gk < K) ? __half2float(A[gm * a_sm + gk * a_sk]) : 0.f;
      Bs[kk][mm] = (gn < N && gk < K) ? __half2float(B[gk * b_sk + gn * b_sn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      if constexpr (OUT_F32) {
        static_cast<float*>(Cv)[static_cast<size_t>(gm) * N + gn] = acc[i][j];
      } else {
        float v = acc[i][j];
        if (bias) v += __half2float(bias[gn]);
        static_cast<__half*>(Cv)[static_cast<size_t>(gm) * N + gn] = __float2half_rn(v);
      }
    }
  }
}

// C[M][N] = fp16(C32 + bias): the bias/cast step after a cross-rank sum of
// fp32 K-shard partials.
__global__ void splitk_finalize_kernel(int M, int N, const float* __restrict__ C32, const __half* __restrict__ bias,
                                       __half* __restrict__ C) {
  const size_t total = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float v = C32[i];
    if (bias) v += __half2float(bias[i % N]);
    C[i] = __float2half_rn(v);
  }
}

}  // namespace mm4

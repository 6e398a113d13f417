/*
 * mm4 CPU oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's own CPU validation loops for the
 * tensor-op contraction path of liuliu/example_matmul_metal4. It is the
 * checker the parity tests compare the CUDA kernels against, and the timed
 * CPU baseline of bench.py. Nothing in the mm4 library links, loads or calls
 * it.
 *
 * Every routine follows the loop order of the Swift code it cites: fp16
 * inputs widened to fp32, one fp32 accumulator, ascending reduction index.
 * An optional thread count parallelises the OUTER output loop only (OpenMP),
 * so the per-element arithmetic is identical in every mode.
 *
 * Parity pinning: the reference cannot run here (Swift + Metal, Apple GPU
 * only), so these routines are pinned against the reference's
 * formula-generated known-answer cases (tests/test_oracle.py): the 1-channel
 * centre-tap identity conv (ConvolutionShared.swift:4876-4893), the
 * set_offsets ramp probe (convolution.swift:204-216, :372-392), the recorded
 * device outcomes (AGENTS.md:120-124) and an independent float64 restatement.
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 */

/* IEEE 754 binary16 -> binary32, exact. */
float mm4o_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        mant <<= 1;
        ++e;
      } while ((mant & 0x400u) == 0);
      mant &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* binary32 -> binary16 with round-to-nearest-even (IEEE 754 default). */
uint16_t mm4o_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
  if (ax < 0x38800000u) {                                   /* result subnormal or zero */
    if (ax < 0x33000000u) return sign;                      /* < 2^-25: rounds to 0 */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e; /* 14 + (113 - e) */
    uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t r = ((ax - 0x38000000u) >> 13); /* rebias exponent, drop 13 bits */
  const uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return (uint16_t)(sign | r);
}

void mm4o_half_to_float_array(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = mm4o_half_to_float(src[i]);
}

void mm4o_float_to_half_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = mm4o_float_to_half(src[i]);
}

static void set_threads(int threads) {
#ifdef _OPENMP
  omp_set_num_threads(threads > 0 ? threads : 1);
#else
  (void)threads;
#endif
}

int mm4o_max_threads(void) {
#ifdef _OPENMP
  return omp_get_num_procs();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------- GEMM */

/*
 * out[m][n] = bias[n] + sum_k A(m,k) * B(k,n), fp32, k ascending, bias first
 * (matmul.swift:499-510: `expected = bias[n]; expected += A[i + m*K] *
 * B[i + n*K]`). transA/transB take the reference's `transpose` meanings
 * (matmul.swift:80-117): transA = 0 -> A[M][K]; 1 -> A[K][M];
 * transB = 1 -> B[N][K] (reference default); 0 -> B[K][N] (NN).
 * Rows [row_begin, row_end) only, so a bounded sample can be timed.
 */
void mm4o_gemm(int M, int N, int K, const uint16_t* A, const uint16_t* B, const uint16_t* bias, int transA,
               int transB, float* out, int row_begin, int row_end, int threads) {
  (void)M;
  set_threads(threads);
  const int64_t a_sm = transA ? 1 : K, a_sk = transA ? M : 1;
  const int64_t b_sn = transB ? K : 1, b_sk = transB ? 1 : N;
  /* Widen B once to [N][K] fp32 (exact), so the inner loop is the
   * reference's dot product over contiguous k. */
  float* Bt = (float*)malloc((size_t)N * (size_t)K * sizeof(float));
  if (!Bt) return;
  for (int n = 0; n < N; ++n)
    for (int i = 0; i < K; ++i) Bt[(int64_t)n * K + i] = mm4o_half_to_float(B[i * b_sk + n * b_sn]);
#pragma omp parallel if (threads > 1)
  {
    float* arow = (float*)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(dynamic, 1)
    for (int m = row_begin; m < row_end; ++m) {
      if (!arow) continue;
      for (int i = 0; i < K; ++i) arow[i] = mm4o_half_to_float(A[m * a_sm + i * a_sk]);
      for (int n = 0; n < N; ++n) {
        const float* brow = Bt + (int64_t)n * K;
        float expected = bias ? mm4o_half_to_float(bias[n]) : 0.0f;
        for (int i = 0; i < K; ++i) expected += arow[i] * brow[i];
        out[(int64_t)(m - row_begin) * N + n] = expected;
      }
    }
    free(arow);
  }
  free(Bt);
}

/* ----------------------------------------------------------- attention */

/*
 * One (batch, head): O[row][d] for rows [row_begin, row_end), following
 * Network.createMatrixSRow / createMatrixPRow / inferenceAttention
 * (Network.swift:134-179, :286-311):
 *   S = q.k (d ascending); value = scale*S; max; sum exp(value - max);
 *   lse = max + log(sum); P = exp(value - lse); O[d] = sum_c P[c] * V[c][d].
 * q/k/v/o are per-head base pointers with element strides between rows
 * (the head-dim elements are contiguous).
 */
void mm4o_attention_head(int R, int C, int D, float scale, const uint16_t* q, int64_t q_rs, const uint16_t* k,
                         int64_t k_rs, const uint16_t* v, int64_t v_rs, float* o, int64_t o_rs, int row_begin,
                         int row_end, float* scratch /* C floats */) {
  (void)R;
  for (int row = row_begin; row < row_end; ++row) {
    float* srow = scratch;
    for (int c = 0; c < C; ++c) {
      float dot = 0.0f;
      for (int d = 0; d < D; ++d)
        dot += mm4o_half_to_float(q[row * q_rs + d]) * mm4o_half_to_float(k[c * k_rs + d]);
      srow[c] = dot;
    }
    float maximum = -3.40282347e+38f;
    for (int c = 0; c < C; ++c) {
      const float value = scale * srow[c];
      maximum = value > maximum ? value : maximum;
    }
    float sum = 0.0f;
    for (int c = 0; c < C; ++c) sum += expf(scale * srow[c] - maximum);
    const float lse = maximum + logf(sum);
    for (int c = 0; c < C; ++c) srow[c] = expf(scale * srow[c] - lse);
    for (int d = 0; d < D; ++d) {
      float dot = 0.0f;
      for (int c = 0; c < C; ++c) dot += srow[c] * mm4o_half_to_float(v[c * v_rs + d]);
      o[(int64_t)(row - row_begin) * o_rs + d] = dot;
    }
  }
}

/*
 * Batched attention over [batch][heads] with the mm4 layouts:
 * layout 0 = [B][H][S][D], layout 1 = [B][S][H][D]. Heads of K/V are
 * shared by heads_q/heads_kv query heads. Output rows [row_begin,row_end)
 * of every (b, h) into out[b][h][row - row_begin][d].
 */
void mm4o_attention(int batch, int heads_q, int heads_kv, int R, int C, int D, float scale, int layout,
                    const uint16_t* Q, const uint16_t* K, const uint16_t* V, float* out, int row_begin, int row_end,
                    int threads, float* scratch /* threads*C floats */) {
  set_threads(threads);
  const int rows = row_end - row_begin;
  const int group = heads_q / heads_kv;
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
  for (int bh = 0; bh < batch * heads_q; ++bh) {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    const int b = bh / heads_q, h = bh % heads_q, hk = h / group;
    const uint16_t *q, *k, *v;
    int64_t q_rs, kv_rs;
    if (layout == 0) {
      q = Q + ((int64_t)b * heads_q + h) * R * D;
      k = K + ((int64_t)b * heads_kv + hk) * C * D;
      v = V + ((int64_t)b * heads_kv + hk) * C * D;
      q_rs = D;
      kv_rs = D;
    } else {
      q = Q + (int64_t)b * R * heads_q * D + (int64_t)h * D;
      k = K + (int64_t)b * C * heads_kv * D + (int64_t)hk * D;
      v = V + (int64_t)b * C * heads_kv * D + (int64_t)hk * D;
      q_rs = (int64_t)heads_q * D;
      kv_rs = (int64_t)heads_kv * D;
    }
    float* o = out + (int64_t)bh * rows * D;
    mm4o_attention_head(R, C, D, scale, q, q_rs, k, kv_rs, v, kv_rs, o, D, row_begin, row_end,
                        scratch + (int64_t)tid * C);
  }
}

/*
 * Attention gradients of the loss sum(dO * O) (Network.swift:313-326) for
 * every (batch, key/value head), following Network.swift:
 *   createLTerm (:181-203): lse = max + log(sum exp(value - max)), value = scale * S;
 *   createMatrixPRow (:151-179): P = exp(value - lse);
 *   createDTerm (:258-282): O = P V (columns ascending), D = O . dO;
 *   createDerivativePRow (:205-218): dP = dO V^T (d ascending);
 *   createDerivativeSRow (:220-256): dS = P (dP - D) * scale;
 *   derivativeQ (:375-401): dQ row = dS K (columns ascending);
 *   derivativeK (:351-373): dK[c] += dS[c] * q (rows ascending);
 *   derivativeV (:328-350): dV[c] += P[c] * dO row (rows ascending).
 * Grouped-query heads: the query heads sharing a key/value head are taken in
 * ascending order, so dK / dV sum over them. dQ, dK, dV are written with the
 * element offsets of Q, K, V (same layout, fp32); lse is [batch][heads_q][R].
 * scratch: threads * (2 * C + D) floats.
 */
void mm4o_attention_bwd(int batch, int heads_q, int heads_kv, int R, int C, int D, float scale, int layout,
                        const uint16_t* Q, const uint16_t* K, const uint16_t* V, const uint16_t* dO, float* dQ,
                        float* dK, float* dV, float* lse_out, int threads, float* scratch) {
  set_threads(threads);
  const int group = heads_q / heads_kv;
  const int64_t q_rs = layout == 0 ? D : (int64_t)heads_q * D;
  const int64_t kv_rs = layout == 0 ? D : (int64_t)heads_kv * D;
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
  for (int bk = 0; bk < batch * heads_kv; ++bk) {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    float* prow = scratch + (int64_t)tid * (2 * C + D);
    float* dprow = prow + C;
    float* orow = dprow + C;
    const int b = bk / heads_kv, hk = bk % heads_kv;
    const int64_t kv_base = layout == 0 ? ((int64_t)b * heads_kv + hk) * C * D
                                        : (int64_t)b * C * heads_kv * D + (int64_t)hk * D;
    const uint16_t* k = K + kv_base;
    const uint16_t* v = V + kv_base;
    float* dk = dK + kv_base;
    float* dv = dV + kv_base;
    for (int c = 0; c < C; ++c)
      for (int d = 0; d < D; ++d) {
        dk[c * kv_rs + d] = 0.0f;
        dv[c * kv_rs + d] = 0.0f;
      }
    for (int g = 0; g < group; ++g) {
      const int h = hk * group + g;
      const int64_t q_base = layout == 0 ? ((int64_t)b * heads_q + h) * R * D
                                         : (int64_t)b * R * heads_q * D + (int64_t)h * D;
      const uint16_t* q = Q + q_base;
      const uint16_t* go = dO + q_base;
      float* dq = dQ + q_base;
      for (int row = 0; row < R; ++row) {
        for (int c = 0; c < C; ++c) {
          float dot = 0.0f;
          for (int d = 0; d < D; ++d)
            dot += mm4o_half_to_float(q[row * q_rs + d]) * mm4o_half_to_float(k[c * kv_rs + d]);
          prow[c] = dot;
        }
        float maximum = -3.40282347e+38f;
        for (int c = 0; c < C; ++c) {
          const float value = scale * prow[c];
          maximum = value > maximum ? value : maximum;
        }
        float sum = 0.0f;
        for (int c = 0; c < C; ++c) sum += expf(scale * prow[c] - maximum);
        const float lse = maximum + logf(sum);
        lse_out[((int64_t)b * heads_q + h) * R + row] = lse;
        for (int c = 0; c < C; ++c) prow[c] = expf(scale * prow[c] - lse);
        for (int d = 0; d < D; ++d) {
          float dot = 0.0f;
          for (int c = 0; c < C; ++c) dot += prow[c] * mm4o_half_to_float(v[c * kv_rs + d]);
          orow[d] = dot;
        }
        float term_d = 0.0f;
        for (int d = 0; d < D; ++d) term_d += orow[d] * mm4o_half_to_float(go[row * q_rs + d]);
        for (int c = 0; c < C; ++c) {
          float dot = 0.0f;
          for (int d = 0; d < D; ++d)
            dot += mm4o_half_to_float(go[row * q_rs + d]) * mm4o_half_to_float(v[c * kv_rs + d]);
          dprow[c] = dot;
        }
        for (int c = 0; c < C; ++c) {
          float value = prow[c] * (dprow[c] - term_d);
          value *= scale;
          dprow[c] = value; /* dS */
        }
        for (int d = 0; d < D; ++d) {
          float dot = 0.0f;
          for (int c = 0; c < C; ++c) dot += dprow[c] * mm4o_half_to_float(k[c * kv_rs + d]);
          dq[row * q_rs + d] = dot;
        }
        for (int c = 0; c < C; ++c)
          for (int d = 0; d < D; ++d) {
            dk[c * kv_rs + d] += dprow[c] * mm4o_half_to_float(q[row * q_rs + d]);
            dv[c * kv_rs + d] += prow[c] * mm4o_half_to_float(go[row * q_rs + d]);
          }
      }
    }
  }
}

/* ---------------------------------------------------------------- conv */

/* Weight element offset for (oc, kd, kh, kw, ic) in the given layout
 * (ConvolutionShared.swift weightIndex :4848-4860, :4920-4930). */
static int64_t weight_offset(int layout, int O, int C, int KD, int KH, int KW, int oc, int kd, int kh, int kw,
                             int ic) {
  switch (layout) {
    case 0: /* HWIO */ return (((int64_t)kh * KW + kw) * C + ic) * O + oc;
    case 1: /* OHWI */ return (((int64_t)oc * KH + kh) * KW + kw) * C + ic;
    case 2: /* OIHW */ return (((int64_t)oc * C + ic) * KH + kh) * KW + kw;
    case 3: /* DHWIO */ return ((((int64_t)kd * KH + kh) * KW + kw) * C + ic) * O + oc;
    case 4: /* ODHWI */ return ((((int64_t)oc * KD + kd) * KH + kh) * KW + kw) * C + ic;
    case 5: /* OIDHW */ return ((((int64_t)oc * C + ic) * KD + kd) * KH + kh) * KW + kw;
    default: return 0;
  }
}

/*
 * conv3d NDHWC (conv2d is D = KD = 1), following referenceConvolution 2D/3D
 * and referenceConvolutionWithBias (ConvolutionShared.swift:4994-5096,
 * convolution2d_padding.swift:79-107): for each output element, sum over
 * (kd, kh, kw, ic) in that order with zero padding by bounds check, then add
 * bias. Depth padding (pad_front) is an extension of the reference, which has
 * none (:5045 `iz = oz*strideZ + kd*dilationZ`); pad_front = 0 reproduces it.
 * Output rows = flattened (n, oz, oh) indices [row_begin, row_end).
 */
void mm4o_conv3d(int N, int D, int H, int W, int C, int O, int KD, int KH, int KW, int SZ, int SY, int SX, int DZ,
                 int DY, int DX, int pad_front, int pad_top, int pad_left, int OD, int OH, int OW, int layout,
                 const uint16_t* x, const uint16_t* w, const uint16_t* bias, float* out, int64_t row_begin,
                 int64_t row_end, int threads) {
  (void)N;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) if (threads > 1)
  for (int64_t r = row_begin; r < row_end; ++r) {
    const int oh = (int)(r % OH);
    const int oz = (int)((r / OH) % OD);
    const int n = (int)(r / ((int64_t)OH * OD));
    for (int ow = 0; ow < OW; ++ow) {
      for (int oc = 0; oc < O; ++oc) {
        float sum = 0.0f;
        for (int kd = 0; kd < KD; ++kd) {
          const int iz = oz * SZ + kd * DZ - pad_front;
          for (int kh = 0; kh < KH; ++kh) {
            const int ih = oh * SY + kh * DY - pad_top;
            for (int kw = 0; kw < KW; ++kw) {
              const int iw = ow * SX + kw * DX - pad_left;
              for (int ic = 0; ic < C; ++ic) {
                if (iz >= 0 && iz < D && ih >= 0 && ih < H && iw >= 0 && iw < W) {
                  const float a = mm4o_half_to_float(x[((((int64_t)n * D + iz) * H + ih) * W + iw) * C + ic]);
                  const float b = mm4o_half_to_float(w[weight_offset(layout, O, C, KD, KH, KW, oc, kd, kh, kw, ic)]);
                  sum += a * b;
                }
              }
            }
          }
        }
        if (bias) sum += mm4o_half_to_float(bias[oc]);
        out[((r - row_begin) * OW + ow) * O + oc] = sum;
      }
    }
  }
}

/* Weight layout permutation (permute_oidhw_to_dhwio, ConvolutionShared.swift
 * :4593-4629): dst[to(oc,kd,kh,kw,ic)] = src[from(oc,kd,kh,kw,ic)]. */
void mm4o_permute_weights(int from_layout, int to_layout, int O, int C, int KD, int KH, int KW, const uint16_t* src,
                          uint16_t* dst) {
  for (int oc = 0; oc < O; ++oc)
    for (int kd = 0; kd < KD; ++kd)
      for (int kh = 0; kh < KH; ++kh)
        for (int kw = 0; kw < KW; ++kw)
          for (int ic = 0; ic < C; ++ic)
            dst[weight_offset(to_layout, O, C, KD, KH, KW, oc, kd, kh, kw, ic)] =
                src[weight_offset(from_layout, O, C, KD, KH, KW, oc, kd, kh, kw, ic)];
}

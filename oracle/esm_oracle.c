/* CPU restatement of the reference esm.cpp hot path -- TEST INFRASTRUCTURE.
 *
 * Plain C, scalar, compiled with the reference's release flags (-O3
 * -march=x86-64-v3, GCC's default FP contraction; oracle/Makefile) so every
 * float step rounds where the reference's build rounds, including the
 * multiply-adds GCC fuses into FMAs.  Each function
 * names the reference function (path:line in ayan-goel/esm-cpp) whose
 * arithmetic it restates.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg load this library; the product never does.
 *
 * Pinned by tests/test_oracle_pins.py against oracle/_ref (the reference
 * compiled from its own sources) and the reference's unit-test known answers.
 */
#include "esm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static int clamp127(float v) {
  if (v > 127.0f) v = 127.0f;
  if (v < -127.0f) v = -127.0f;
  return (int)v;
}

/* pack.cpp:149-177 -- per-output-channel symmetric weights.  An all-zero row
 * keeps scale 0 and q 0. */
void orc_quantize_weights(const float* W, int N, int K, int8_t* q, float* scales) {
  for (int n = 0; n < N; ++n) {
    const float* row = W + (size_t)n * K;
    float row_max = 0.0f;
    for (int k = 0; k < K; ++k) {
      float a = fabsf(row[k]);
      if (a > row_max) row_max = a;
    }
    int8_t* qr = q + (size_t)n * K;
    if (row_max == 0.0f) {
      scales[n] = 0.0f;
      memset(qr, 0, (size_t)K);
      continue;
    }
    const float scale = row_max / 127.0f;
    scales[n] = scale;
    const float inv = 1.0f / scale;
    for (int k = 0; k < K; ++k) qr[k] = (int8_t)clamp127(nearbyintf(row[k] * inv));
  }
}

/* gemm_int8.cpp:394-408 / 440-472: max |A| over the whole operand. */
float orc_absmax(const float* x, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = fabsf(x[i]);
    if (a > m) m = a;
  }
  return m;
}

/* gemm_int8.cpp:434 / 479: act_scale = amax>0 ? amax/127 : 1. */
float orc_act_scale(float amax) { return (amax > 0.0f) ? (amax / 127.0f) : 1.0f; }

/* gemm_int8.cpp:409-426 / 484-498 vector path: q = clamp(cvt_rne(x*inv)).
 * The reference stores q+128 as u8 for VPDPBUSD and removes the 128 again with
 * col_sum (gemm_int8.cpp:115-117); the s8 value kept here is that same q. */
void orc_quantize_act(const float* x, size_t n, float scale, int8_t* q) {
  const float inv = 1.0f / scale;
  for (size_t i = 0; i < n; ++i) q[i] = (int8_t)clamp127(nearbyintf(x[i] * inv));
}

/* Per-token mode: QuantizeActivationSymmetricRef (pack.cpp:134-147) applied
 * to one row at a time with that row's own absmax scale. */
void orc_quantize_act_per_token(const float* x, int M, int K, int8_t* q,
                                float* row_scales) {
  for (int m = 0; m < M; ++m) {
    const float* r = x + (size_t)m * K;
    const float s = orc_act_scale(orc_absmax(r, (size_t)K));
    row_scales[m] = s;
    orc_quantize_act(r, (size_t)K, s, q + (size_t)m * K);
  }
}

/* The integer core of Kernel6x32 / Kernel32x32 after the zero-point
 * correction (gemm_int8.cpp:115-117): sum_k q[m,k]*w[n,k], exact in int32
 * because K*127*127 < 2^31 for every ESM-2 width. */
void orc_gemm_i8_s32(const int8_t* q, const int8_t* w, int32_t* acc, int M, int N,
                     int K) {
  for (int m = 0; m < M; ++m) {
    const int8_t* a = q + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const int8_t* b = w + (size_t)n * K;
      int32_t s = 0;
      for (int k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
      acc[(size_t)m * N + n] = s;
    }
  }
}

/* gemm_int8.cpp:109-126 FinalizeStore16: fma(float(acc), ws[n]*as, bias[n]),
 * with the ws*as product rounded before the fma. */
void orc_dequant(const int32_t* acc, const float* ws, float act_scale,
                 const float* row_scales, const float* bias, float* C, int M, int N) {
  for (int m = 0; m < M; ++m) {
    const float as = row_scales ? row_scales[m] : act_scale;
    for (int n = 0; n < N; ++n) {
      const float combined = ws[n] * as;
      const float b = bias ? bias[n] : 0.0f;
      C[(size_t)m * N + n] = fmaf((float)acc[(size_t)m * N + n], combined, b);
    }
  }
}

/* gemm_fp32.cpp:33-46 LinearRef. */
void orc_linear_f32(const float* A, const float* W, const float* bias, float* C,
                    int M, int N, int K) {
  for (int m = 0; m < M; ++m) {
    const float* a = A + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      const float* w = W + (size_t)n * K;
      float acc = bias ? bias[n] : 0.0f;
      for (int k = 0; k < K; ++k) acc += a[k] * w[k];
      C[(size_t)m * N + n] = acc;
    }
  }
}

/* layernorm.cpp:23-43 LayerNormRef. */
void orc_layernorm(const float* x, const float* g, const float* b, float eps,
                   float* out, int rows, int d) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * d;
    float* yr = out + (size_t)r * d;
    double mean = 0.0;
    for (int i = 0; i < d; ++i) mean += xr[i];
    mean /= d;
    double var = 0.0;
    for (int i = 0; i < d; ++i) {
      double diff = xr[i] - mean;
      var += diff * diff;
    }
    var /= d;
    const float inv_std = 1.0f / sqrtf((float)var + eps);
    const float meanf = (float)mean;
    for (int i = 0; i < d; ++i) {
      float normed = (xr[i] - meanf) * inv_std;
      yr[i] = normed * g[i] + b[i];
    }
  }
}

/* gelu.cpp:30-35 GeluRef. */
void orc_gelu(const float* x, float* out, size_t n) {
  const float kInvSqrt2 = 0.70710678118654752440f;
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * 0.5f * (1.0f + erff(x[i] * kInvSqrt2));
}

/* residual.cpp:23-29. */
void orc_residual_add(float* y, const float* x, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] += x[i];
}
void orc_scale(float* x, size_t n, float s) {
  for (size_t i = 0; i < n; ++i) x[i] *= s;
}

/* rope_tables.cpp:14-29: inv_freq = 10000^(-2i/dh), duplicated half/half. */
void orc_rope_build_tables(int L, int dh, float* cos_t, float* sin_t) {
  const int half = dh / 2;
  for (int i = 0; i < half; ++i) {
    const float exponent = (float)(2 * i) / (float)dh;
    const float inv_freq = powf(10000.0f, -exponent);
    for (int t = 0; t < L; ++t) {
      const float angle = (float)t * inv_freq;
      const float c = cosf(angle), s = sinf(angle);
      cos_t[t * dh + i] = c;
      cos_t[t * dh + i + half] = c;
      sin_t[t * dh + i] = s;
      sin_t[t * dh + i + half] = s;
    }
  }
}

/* rope.cpp:47-70 (Ref) and rope.cpp:98-121 (AVX-512, fused). Positions
 * restart at every cu_seqlens boundary. */
void orc_rope_apply_varlen(float* x, const float* cos_t, const float* sin_t,
                           const int* cu, int B, int H, int dh, int fused) {
  const int half = dh / 2;
  for (int b = 0; b < B; ++b) {
    for (int p = 0; p < cu[b + 1] - cu[b]; ++p) {
      const int t = cu[b] + p;
      const float* c = cos_t + (size_t)p * dh;
      const float* s = sin_t + (size_t)p * dh;
      for (int h = 0; h < H; ++h) {
        float* xr = x + ((size_t)t * H + h) * dh;
        for (int i = 0; i < half; ++i) {
          const float lo = xr[i], hi = xr[i + half];
          if (fused) {
            xr[i] = fmaf(-hi, s[i], lo * c[i]);
            xr[i + half] = fmaf(hi, c[i], lo * s[i]);
          } else {
            xr[i] = lo * c[i] + (-hi) * s[i];
            xr[i + half] = hi * c[i + half] + lo * s[i + half];
          }
        }
      }
    }
  }
}

/* attention.cpp:99-144 AttentionVarlenRef: per (sequence, head, query): FP32
 * dot products, max-subtracted expf, softmax sum in double, inv_sum rounded
 * to float, out = sum_j (e_j*inv_sum) * v_j accumulated in j order. */
void orc_attention_varlen(const float* q, const float* k, const float* v,
                          const int* cu, int B, int H, int dh, float* out) {
  int maxL = 0;
  for (int b = 0; b < B; ++b)
    if (cu[b + 1] - cu[b] > maxL) maxL = cu[b + 1] - cu[b];
  float* scores = (float*)malloc(sizeof(float) * (size_t)(maxL > 0 ? maxL : 1));
  for (int b = 0; b < B; ++b) {
    const int s0 = cu[b], L = cu[b + 1] - cu[b];
    if (L <= 0) continue;
    for (int h = 0; h < H; ++h) {
      for (int i = 0; i < L; ++i) {
        const float* qi = q + ((size_t)(s0 + i) * H + h) * dh;
        float mx = -INFINITY;
        for (int j = 0; j < L; ++j) {
          const float* kj = k + ((size_t)(s0 + j) * H + h) * dh;
          float dot = 0.0f;
          for (int d = 0; d < dh; ++d) dot += qi[d] * kj[d];
          scores[j] = dot;
          if (dot > mx) mx = dot;
        }
        double sum = 0.0;
        for (int j = 0; j < L; ++j) {
          float e = expf(scores[j] - mx);
          scores[j] = e;
          sum += e;
        }
        const float inv_sum = sum > 0.0 ? (float)(1.0 / sum) : 0.0f;
        float* o = out + ((size_t)(s0 + i) * H + h) * dh;
        for (int d = 0; d < dh; ++d) o[d] = 0.0f;
        for (int j = 0; j < L; ++j) {
          const float w = scores[j] * inv_sum;
          if (w == 0.0f) continue;
          const float* vj = v + ((size_t)(s0 + j) * H + h) * dh;
          for (int d = 0; d < dh; ++d) o[d] += w * vj[d];
        }
      }
    }
  }
  free(scores);
}

/* model.cpp:737-778 Embed. kTokenDropoutMaskRatioTrain = 0.15f*0.8f
 * (model.cpp:32); scale = (1-0.12)/max(1-observed_mask_ratio, 1e-12). Mask
 * tokens and pad rows are zero. */
void orc_embed(const float* embed_w, int d, const int* ids, const int* masks,
               const int* cu, int B, int mask_id, float* out) {
  const float ratio_train = 0.15f * 0.8f;
  for (int b = 0; b < B; ++b) {
    int src_len = 0, observed = 0;
    for (int t = cu[b]; t < cu[b + 1]; ++t) {
      if (!masks || masks[t] != 0) ++src_len;
      if (ids[t] == mask_id) ++observed;
    }
    const float obs = src_len > 0 ? (float)observed / (float)src_len : 0.0f;
    float denom = 1.0f - obs;
    if (denom < 1e-12f) denom = 1e-12f;
    const float scale = (1.0f - ratio_train) / denom;
    for (int t = cu[b]; t < cu[b + 1]; ++t) {
      float* o = out + (size_t)t * d;
      const int zero = (ids[t] == mask_id) || (masks && masks[t] == 0);
      const float* row = embed_w + (size_t)ids[t] * d;
      for (int i = 0; i < d; ++i) o[i] = zero ? 0.0f : row[i] * scale;
    }
  }
}

/* orc_plan_batches lives in esm_oracle_plan.cpp: the reference splits chunks
 * with std::sort (scheduler.cpp:31-36), whose tie order only the same C++
 * library call reproduces. */

/* CPU restatement of the reference's default x86 kernels (the AVX-512 forms
 * its dispatch picks on this hardware) -- TEST INFRASTRUCTURE ONLY, the
 * checker of the GPU's reference-rounding mode (esmcu_math_mode
 * ESMCU_MATH_AVX512).
 *
 * Compiled with -ffp-contract=off: every multiply-add that the reference's
 * release build fuses (g++ -O3, contraction on) is an explicit fmaf here,
 * and every other step rounds on its own, so the C below states the exact
 * rounding sequence.  tests/test_oracle_pins.py checks each function bit for
 * bit against the reference compiled from its own sources (oracle/_ref).
 *
 *   orc_layernorm_avx   LayerNormAvx512        layernorm.cpp:59-149
 *   orc_gelu_avx        GeluAvx512             gelu.cpp:48-148
 *   orc_attention_avx   AttentionVarlenAvx512  attention.cpp:230-437, 770-811
 *   orc_expf_libc       the C library's expf, which that attention calls for
 *                       the keys past the last whole 16-key block
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "esm_oracle.h"

static float as_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t as_u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static double as_d(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static uint64_t as_u64(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

/* _mm512_reduce_add_ps as GCC defines it: fold lanes j and j+8, then j and
 * j+4, then j and j+2, then 0 and 1. */
static float reduce16(const float v[16]) {
  float t3[8], t6[4];
  for (int j = 0; j < 8; ++j) t3[j] = v[8 + j] + v[j];
  for (int j = 0; j < 4; ++j) t6[j] = t3[4 + j] + t3[j];
  return (t6[0] + t6[2]) + (t6[1] + t6[3]);
}

/* layernorm.cpp:59-149, d % 16 == 0 (every ESM-2 width).  Four 16-lane
 * accumulators over 64-column steps (16-column steps go to the first), the
 * lanes combined as (s0 + s1) + (s2 + s3), then the horizontal sum; the
 * variance the same with one FMA per element; the build fuses
 * `var = sum * inv_d; var + eps` into fmaf(sum, inv_d, eps). */
void orc_layernorm_avx(const float* x, const float* g, const float* b, float eps, float* out,
                       int rows, int d) {
  const float inv_d = 1.0f / (float)d;
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (long)r * d;
    float* yr = out + (long)r * d;
    float s[4][16] = {{0}}, sv[16];
    int i = 0;
    for (; i + 64 <= d; i += 64)
      for (int k = 0; k < 4; ++k)
        for (int l = 0; l < 16; ++l) s[k][l] = s[k][l] + xr[i + 16 * k + l];
    for (; i + 16 <= d; i += 16)
      for (int l = 0; l < 16; ++l) s[0][l] = s[0][l] + xr[i + l];
    for (int l = 0; l < 16; ++l) sv[l] = (s[0][l] + s[1][l]) + (s[2][l] + s[3][l]);
    const float mean = (reduce16(sv) + 0.0f) * inv_d;
    float v[4][16] = {{0}}, vv[16];
    i = 0;
    for (; i + 64 <= d; i += 64)
      for (int k = 0; k < 4; ++k)
        for (int l = 0; l < 16; ++l) {
          const float dd = xr[i + 16 * k + l] - mean;
          v[k][l] = fmaf(dd, dd, v[k][l]);
        }
    for (; i + 16 <= d; i += 16)
      for (int l = 0; l < 16; ++l) {
        const float dd = xr[i + l] - mean;
        v[0][l] = fmaf(dd, dd, v[0][l]);
      }
    for (int l = 0; l < 16; ++l) vv[l] = (v[0][l] + v[1][l]) + (v[2][l] + v[3][l]);
    const float inv_std = 1.0f / sqrtf(fmaf(reduce16(vv) + 0.0f, inv_d, eps));
    for (int c = 0; c < d; ++c) yr[c] = fmaf((xr[c] - mean) * inv_std, g[c], b[c]);
  }
}

/* ExpAvx512 (gelu.cpp:48-68) and ExpAvx512Attn (attention.cpp:156-176):
 * n = rint(x log2 e); r = (x - n ln2_hi) - n ln2_lo with both subtractions
 * fused by the build; 5-term Horner; 2^n from the exponent bits without a
 * range guard (cvtps2dq gives 0x80000000 out of range). */
static float exp_avx(float x) {
  const float nf = rintf(x * 1.44269504088896340736f);
  float r = fmaf(-nf, 6.93145752e-1f, x);
  r = fmaf(-nf, 1.42860677e-6f, r);
  float p = 1.0f / 120.0f;
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t ni = fabsf(nf) < 2147483648.0f ? (uint32_t)(int32_t)nf : 0x80000000u;
  return p * as_f((ni + 127u) << 23);
}

/* gelu.cpp:76-94 (ErfAvx512, A&S 7.1.26) and 98-148. */
void orc_gelu_avx(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float v = x[i];
    const float z = v * 0.70710678118654752440f;
    const uint32_t sign = as_u(z) & 0x80000000u;
    const float t = 1.0f / fmaf(0.3275911f, fabsf(z), 1.0f);
    float poly = 1.061405429f;
    poly = fmaf(poly, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    poly = poly * t;
    const float e = exp_avx(0.0f - z * z);
    const float erf = as_f(as_u(fmaf(-poly, e, 1.0f)) | sign);
    out[i] = (v * 0.5f) * (1.0f + erf);
  }
}

/* The C library's expf (the exp2-table method of glibc 2.28 and later):
 * k = round(x * 32/ln2) by the 1.5 * 2^52 shift, r = x * 32/ln2 - k,
 * 2^(k/32) = table[k % 32] with k/32 added to its exponent, a degree-3
 * polynomial in r, all in double; one rounding to float.  The table holds
 * 2^(i/32) rounded to double minus i << 47 (oracle/gen_exp2_table.py). */
static const uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

float orc_expf_libc(float x) {
  const uint32_t abstop = (as_u(x) >> 20) & 0x7ff;
  if (abstop >= ((as_u(88.0f) >> 20) & 0x7ff)) {
    if (as_u(x) == as_u(-INFINITY)) return 0.0f;
    if (abstop >= ((as_u(INFINITY) >> 20) & 0x7ff)) return x + x;
    if (x > 0x1.62e42ep6f) return INFINITY;
    if (x < -0x1.9fe368p6f) return 0.0f;
  }
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32;
  const double shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
  const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
  const double z = inv_ln2_n * (double)x;
  double kd = z + shift;
  const uint64_t ki = as_u64(kd);
  kd -= shift;
  const double r = z - kd;
  const double s = as_d(kExp2Tab[ki % 32] + (ki << 47));
  const double zz = fma(c0, r, c1);
  double y = fma(c2, r, 1.0);
  y = fma(zz, r * r, y);
  return (float)(y * s);
}

/* attention.cpp:230-437: per (sequence, head, query): scores by 16 FMA
 * lanes over the head dim and the horizontal sum; softmax with exp_avx on
 * whole 16-key blocks (per-lane running sum, then the horizontal sum) and
 * the C library's expf on the remaining keys, added one by one; O[d] =
 * fma(e_j * (1/sum), V[j][d], O[d]) over j in order, zero weights skipped.
 * head_dim % 16 == 0; scratch holds max_len floats. */
void orc_attention_avx(const float* q, const float* k, const float* v, const int* cu, int B,
                       int H, int dh, float* out, float* scratch) {
  float o[128];
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h) {
      const int s0 = cu[b], L = cu[b + 1] - cu[b];
      for (int i = 0; i < L; ++i) {
        const float* qi = q + ((long)(s0 + i) * H + h) * dh;
        float mx = -INFINITY;
        for (int j = 0; j < L; ++j) {
          const float* kj = k + ((long)(s0 + j) * H + h) * dh;
          float acc[16] = {0};
          for (int c = 0; c + 16 <= dh; c += 16)
            for (int l = 0; l < 16; ++l) acc[l] = fmaf(qi[c + l], kj[c + l], acc[l]);
          scratch[j] = reduce16(acc);
          if (scratch[j] > mx) mx = scratch[j];
        }
        float vs[16] = {0};
        int j = 0;
        for (; j + 16 <= L; j += 16)
          for (int l = 0; l < 16; ++l) {
            const float e = exp_avx(scratch[j + l] - mx);
            scratch[j + l] = e;
            vs[l] = vs[l] + e;
          }
        float sum = reduce16(vs);
        for (; j < L; ++j) {
          const float e = orc_expf_libc(scratch[j] - mx);
          scratch[j] = e;
          sum += e;
        }
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int c = 0; c < dh; ++c) o[c] = 0.0f;
        for (int jj = 0; jj < L; ++jj) {
          const float w = scratch[jj] * inv;
          if (w == 0.0f) continue;
          const float* vj = v + ((long)(s0 + jj) * H + h) * dh;
          for (int c = 0; c < dh; ++c) o[c] = fmaf(w, vj[c], o[c]);
        }
        float* orow = out + ((long)(s0 + i) * H + h) * dh;
        for (int c = 0; c < dh; ++c) orow[c] = o[c];
      }
    }
}

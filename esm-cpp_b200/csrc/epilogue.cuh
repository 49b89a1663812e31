// Row-run epilogue shared by the INT8 and FP32 GEMMs: takes NV finished fp32
// values of one output row and applies store / residual add / GELU, with an
// optional running absmax of what was stored.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {

// gelu.cpp:30-35: x * 0.5 * (1 + erf(x / sqrt(2))), each step rounded.
// erf(z) = sign(z) (1 - erfc|z|) with erfc(a) = 2^(a R(a)): R is a degree-9
// least-squares polynomial fit of log2(erfc(a)) / a on (0, 4] (fitted in
// double precision against erfc, coefficients rounded to float, evaluated by
// Horner FMAs); past |z| = 4 the exponent is driven down so erfc = 0 there
// (erf = +-1, as erf rounds in float).  One ex2 and eleven FMAs in place of
// a general erf: erfc is within about 4e-6 relative (log2 error < 5e-6,
// < 8e-7 for |z| < 1.5), which keeps the GELU within 5% of the 1e-6
// (1 + |gelu|) op tolerance.
__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kR[10] = {-0x1.a0bf78p+0f,  -0x1.d629d6p-1f,  -0x1.30f734p-3f, 0x1.d920dep-6f,
                            -0x1.2cd446p-10f, -0x1.8d0dbcp-10f, 0x1.3426e2p-11f, -0x1.d6149ap-14f,
                            0x1.81f4eap-17f,  -0x1.0f5acep-21f};
  const float kInvSqrt2 = 0.70710678118654752440f;
  const float z = __fmul_rn(x, kInvSqrt2);
  const float az = fabsf(z);
  const float a = fminf(az, 4.0f);
  float r = kR[9];
#pragma unroll
  for (int i = 8; i >= 0; --i) r = __fmaf_rn(r, a, kR[i]);
  const float q = __fmaf_rn(fmaxf(__fsub_rn(az, 4.0f), 0.0f), -1.0e4f, __fmul_rn(r, a));
  const float erf_z = copysignf(__fsub_rn(1.0f, ex2_ftz(q)), z);
  return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, erf_z));
}

// gelu_erf on two values with the packed f32x2 instructions: the same
// operations in the same order, each rounded as in gelu_erf (bit-identical
// results), half the FMA-pipe instructions.
__device__ __forceinline__ void gelu_erf2(float& x0, float& x1) {
  constexpr float kR[10] = {-0x1.a0bf78p+0f,  -0x1.d629d6p-1f,  -0x1.30f734p-3f, 0x1.d920dep-6f,
                            -0x1.2cd446p-10f, -0x1.8d0dbcp-10f, 0x1.3426e2p-11f, -0x1.d6149ap-14f,
                            0x1.81f4eap-17f,  -0x1.0f5acep-21f};
  auto dup = [](float v) { return f2_pack(v, v); };
  const unsigned long long x = f2_pack(x0, x1);
  const unsigned long long z = f2_mul(x, dup(0.70710678118654752440f));
  float z0, z1;
  f2_unpack(z, z0, z1);
  const float az0 = fabsf(z0), az1 = fabsf(z1);
  const unsigned long long a = f2_pack(fminf(az0, 4.0f), fminf(az1, 4.0f));
  unsigned long long r = dup(kR[9]);
#pragma unroll
  for (int i = 8; i >= 0; --i) r = f2_fma(r, a, dup(kR[i]));
  const unsigned long long pen =
      f2_pack(fmaxf(__fsub_rn(az0, 4.0f), 0.0f), fmaxf(__fsub_rn(az1, 4.0f), 0.0f));
  const unsigned long long q = f2_fma(pen, dup(-1.0e4f), f2_mul(r, a));
  float q0, q1;
  f2_unpack(q, q0, q1);
  const unsigned long long om = f2_sub(dup(1.0f), f2_pack(ex2_ftz(q0), ex2_ftz(q1)));
  float o0, o1;
  f2_unpack(om, o0, o1);
  const unsigned long long t = f2_add(dup(1.0f), f2_pack(copysignf(o0, z0), copysignf(o1, z1)));
  f2_unpack(f2_mul(f2_mul(x, dup(0.5f)), t), x0, x1);
}

// Applies kEpiStore / kEpiResidual / kEpiGelu to y[0..NV) = columns
// [c0, c0+NV) of row m (columns >= N are skipped).  Returns max|stored|.
template <int NV>
__device__ __forceinline__ float epi_row_run(const EpiParams& e, long m, int c0, int N,
                                             float (&y)[NV]) {
  float mx = 0.0f;
  float* row = e.C + m * e.ldc + c0;
  const bool vec = (c0 + NV <= N) && ((e.ldc & 3) == 0) && ((c0 & 3) == 0) &&
                   ((reinterpret_cast<uintptr_t>(e.C) & 15) == 0);
  if (vec) {
#pragma unroll
    for (int j = 0; j < NV; j += 4) {
      float4 o = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
      if (e.kind == kEpiResidual) {
        const float4 h = *reinterpret_cast<const float4*>(row + j);
        o.x = __fadd_rn(h.x, o.x);
        o.y = __fadd_rn(h.y, o.y);
        o.z = __fadd_rn(h.z, o.z);
        o.w = __fadd_rn(h.w, o.w);
      } else if (e.kind == kEpiGelu) {
        o.x = gelu_erf(o.x);
        o.y = gelu_erf(o.y);
        o.z = gelu_erf(o.z);
        o.w = gelu_erf(o.w);
      }
      *reinterpret_cast<float4*>(row + j) = o;
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
    }
  } else {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (c0 + j < N) {
        float o = y[j];
        if (e.kind == kEpiResidual) o = __fadd_rn(row[j], o);
        else if (e.kind == kEpiGelu) o = gelu_erf(o);
        row[j] = o;
        mx = fmaxf(mx, fabsf(o));
      }
    }
  }
  return mx;
}

// The q-scale and RoPE of epi_qkv_rope_head on the values only (the caller
// stores them); which = 0 (q), 1 (k), 2 (v).  The row's cos / sin table
// entries 0..31 are in shared memory at cs_row (cos) and cs_row + 128 (sin),
// 16-byte chunk i4 at position i4 ^ swz.
__device__ __forceinline__ void epi_qkv_rope_values(const EpiParams& e, uint32_t cs_row,
                                                    int swz, int which, float (&y)[64]) {
  // Two columns per packed f32x2 instruction, the scalar rounding per column.
  if (which == 0) {
    const unsigned long long qs = f2_pack(e.q_scale, e.q_scale);
#pragma unroll
    for (int j = 0; j < 64; j += 2) f2_unpack(f2_mul(f2_pack(y[j], y[j + 1]), qs), y[j], y[j + 1]);
  }
  if (which <= 1) {
#pragma unroll
    for (int i4 = 0; i4 < 8; ++i4) {
      const uint32_t o = static_cast<uint32_t>((i4 ^ swz) << 4);
      const float4 cv = lds128(cs_row + o), sv = lds128(cs_row + 128u + o);
      const unsigned long long c2[2] = {f2_pack(cv.x, cv.y), f2_pack(cv.z, cv.w)};
      const unsigned long long s2[2] = {f2_pack(sv.x, sv.y), f2_pack(sv.z, sv.w)};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int i = 4 * i4 + 2 * k;
        const unsigned long long lo = f2_pack(y[i], y[i + 1]), hi = f2_pack(y[i + 32], y[i + 33]);
        const unsigned long long nhi = f2_pack(-y[i + 32], -y[i + 33]);
        // lo' = fma(-hi, s, lo * c), hi' = fma(hi, c, lo * s)
        f2_unpack(f2_fma(nhi, s2[k], f2_mul(lo, c2[k])), y[i], y[i + 1]);
        f2_unpack(f2_fma(hi, c2[k], f2_mul(lo, s2[k])), y[i + 32], y[i + 33]);
      }
    }
    if (e.qk_bf16) {
#pragma unroll
      for (int j = 0; j < 64; ++j) y[j] = __bfloat162float(__float2bfloat16_rn(y[j]));
    }
  }
}

// kEpiQkvRope for one 64-wide head chunk of row m starting at output column
// n_base (a multiple of 64): q|k|v split by n_base / d, Q scaled before RoPE
// (model.cpp:976-988), rotate-half RoPE in the AVX-512 form of rope.cpp:109-113
// (lo' = fma(-hi, s, lo*c), hi' = fma(hi, c, lo*s)).
__device__ __forceinline__ void epi_qkv_rope_head(const EpiParams& e, long m, int n_base,
                                                  float (&y)[64]) {
  const int which = n_base / e.d;
  const int col = n_base - which * e.d;
  float* dst = (which == 0 ? e.q : (which == 1 ? e.k : e.v)) + m * e.d + col;
  if (which == 0) {
#pragma unroll
    for (int j = 0; j < 64; ++j) y[j] = __fmul_rn(y[j], e.q_scale);
  }
  if (which <= 1) {
    const int p = e.pos[m];
    const float* c = e.cos_t + static_cast<long>(p) * 64;
    const float* s = e.sin_t + static_cast<long>(p) * 64;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float lo = y[i], hi = y[i + 32];
      const float ci = __ldg(c + i), si = __ldg(s + i);
      y[i] = __fmaf_rn(-hi, si, __fmul_rn(lo, ci));
      y[i + 32] = __fmaf_rn(hi, ci, __fmul_rn(lo, si));
    }
    if (e.qk_bf16) {
#pragma unroll
      for (int j = 0; j < 64; ++j) y[j] = __bfloat162float(__float2bfloat16_rn(y[j]));
    }
  }
#pragma unroll
  for (int j = 0; j < 64; j += 4)
    *reinterpret_cast<float4*>(dst + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
}

}  // namespace esmb200

// Row LayerNorm with the reference's rounding (layernorm.cpp:23-43,
// LayerNormRef): mean and variance accumulated in double, then
// inv_std = 1/sqrtf(float(var) + eps), normed = (x - float(mean)) * inv_std,
// y = fma(normed, g, b) -- the reference's release build contracts that last
// multiply-add into an FMA (its AVX-512 twin, layernorm.cpp:127, uses an
// explicit fmadd there too).  One 128-thread block per row (grid-stride),
// the row held in registers as float4s for d <= 4096 and d % 4 == 0; other
// widths use a one-warp-per-row kernel reading the row from memory.
//
// Fused outputs for the W8A8 path: the absmax of y (per-tensor activation
// scale of the next GEMM) and/or the per-token int8 quantisation of y.
#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int kLnThreads = 128;

// Block-wide sum of a double (all threads call it; result in every thread).
__device__ __forceinline__ double block_sum_d(double v, double* red) {
  v = warp_sum_d(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();  // red[] is reused across calls
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int i = 0; i < kLnThreads / 32; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max_f(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < kLnThreads / 32; ++i) t = fmaxf(t, red[i]);
  return t;
}

// One 128-thread block per row (grid-stride over rows); each thread holds
// NV4 float4 of the row (columns 4*tid + 512*i), d % 4 == 0.
template <int NV4>
__global__ void __launch_bounds__(kLnThreads)
    layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                     const float* __restrict__ b, float eps, float* __restrict__ out, int rows,
                     int d, uint32_t* amax, int8_t* __restrict__ q, long ldq,
                     float* __restrict__ row_scales) {
  __shared__ double red_d[kLnThreads / 32];
  __shared__ float red_f[kLnThreads / 32];
  float tmax = 0.0f;
  for (long r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * d;
    float4 v[NV4];
    double sum = 0.0;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int c = 4 * threadIdx.x + 512 * i;
      v[i] = (c < d) ? __ldg(reinterpret_cast<const float4*>(xr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
      sum += static_cast<double>(v[i].x) + static_cast<double>(v[i].y) +
             (static_cast<double>(v[i].z) + static_cast<double>(v[i].w));
    }
    const double mean = block_sum_d(sum, red_d) / d;
    double var = 0.0;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int c = 4 * threadIdx.x + 512 * i;
      if (c < d) {
        const double a = static_cast<double>(v[i].x) - mean, bb = static_cast<double>(v[i].y) - mean;
        const double cc = static_cast<double>(v[i].z) - mean, dd = static_cast<double>(v[i].w) - mean;
        var += a * a + bb * bb + (cc * cc + dd * dd);
      }
    }
    var = block_sum_d(var, red_d) / d;
    const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(var), eps)));
    const float meanf = static_cast<float>(mean);
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < NV4; ++i) {
      const int c = 4 * threadIdx.x + 512 * i;
      if (c < d) {
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + c));
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b + c));
        v[i].x = __fmaf_rn(__fmul_rn(__fsub_rn(v[i].x, meanf), inv_std), gg.x, bv.x);
        v[i].y = __fmaf_rn(__fmul_rn(__fsub_rn(v[i].y, meanf), inv_std), gg.y, bv.y);
        v[i].z = __fmaf_rn(__fmul_rn(__fsub_rn(v[i].z, meanf), inv_std), gg.z, bv.z);
        v[i].w = __fmaf_rn(__fmul_rn(__fsub_rn(v[i].w, meanf), inv_std), gg.w, bv.w);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        if (out) *reinterpret_cast<float4*>(out + r * d + c) = v[i];
      }
    }
    tmax = fmaxf(tmax, mx);
    if (q != nullptr) {  // per-token int8 of this row
      const float rm = block_max_f(mx, red_f);
      const float s = rm > 0.0f ? __fdiv_rn(rm, 127.0f) : 1.0f;
      const float inv = __fdiv_rn(1.0f, s);
      if (threadIdx.x == 0) row_scales[r] = s;
      int8_t* qr = q + r * ldq;
#pragma unroll
      for (int i = 0; i < NV4; ++i) {
        const int c = 4 * threadIdx.x + 512 * i;
        if (c < d) {
          const int a0 = max(-127, min(127, __float2int_rn(__fmul_rn(v[i].x, inv))));
          const int a1 = max(-127, min(127, __float2int_rn(__fmul_rn(v[i].y, inv))));
          const int a2 = max(-127, min(127, __float2int_rn(__fmul_rn(v[i].z, inv))));
          const int a3 = max(-127, min(127, __float2int_rn(__fmul_rn(v[i].w, inv))));
          *reinterpret_cast<uint32_t*>(qr + c) = (static_cast<uint32_t>(a0) & 0xffu) |
                                                 ((static_cast<uint32_t>(a1) & 0xffu) << 8) |
                                                 ((static_cast<uint32_t>(a2) & 0xffu) << 16) |
                                                 ((static_cast<uint32_t>(a3) & 0xffu) << 24);
        }
      }
      for (int c = d + threadIdx.x; c < ldq; c += kLnThreads) qr[c] = 0;
    }
  }
  if (amax != nullptr) amax_publish(amax, tmax);
}

// Other widths: the same arithmetic, one warp per row, reading the row from
// global memory.
__global__ void layernorm_wide_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                      const float* __restrict__ b, float eps,
                                      float* __restrict__ out, int rows, int d, uint32_t* amax) {
  const int lane = threadIdx.x & 31;
  const long r0 = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const bool live = r0 < rows;
  const long r = live ? r0 : rows - 1;
  const float* xr = x + r * d;
  double sum = 0.0;
  for (int c = lane; c < d; c += 32) sum += static_cast<double>(xr[c]);
  const double mean = warp_sum_d(sum) / d;
  double var = 0.0;
  for (int c = lane; c < d; c += 32) {
    const double diff = static_cast<double>(xr[c]) - mean;
    var += diff * diff;
  }
  var = warp_sum_d(var) / d;
  const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(var), eps)));
  const float meanf = static_cast<float>(mean);
  float mx = 0.0f;
  for (int c = lane; c < d; c += 32) {
    const float y = __fmaf_rn(__fmul_rn(__fsub_rn(xr[c], meanf), inv_std), g[c], b[c]);
    if (live) out[r * d + c] = y;
    mx = fmaxf(mx, fabsf(y));
  }
  if (amax != nullptr) amax_publish(amax, mx);
}

}  // namespace

cudaError_t launch_layernorm(const float* x, const float* g, const float* b, float eps,
                             float* out, int rows, int d, uint32_t* amax, int8_t* q, long ldq,
                             float* row_scales, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const int nv4 = (d + 511) / 512;
  const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   (out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(g) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(b) & 15) == 0) && (q == nullptr || (ldq % 4) == 0);
  const int grid = rows < 148 * 16 ? rows : 148 * 16;
  if (vec && nv4 <= 8) {
    switch (nv4) {
      case 1: layernorm_kernel<1><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
      case 2: layernorm_kernel<2><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
      case 3: layernorm_kernel<3><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
      case 4: layernorm_kernel<4><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
      case 5: layernorm_kernel<5><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
      default: layernorm_kernel<8><<<grid, kLnThreads, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales); break;
    }
    return cudaGetLastError();
  }
  if (q != nullptr || out == nullptr) return cudaErrorInvalidValue;
  const long threads = static_cast<long>(rows) * 32;
  layernorm_wide_kernel<<<static_cast<int>((threads + 255) / 256), 256, 0, s>>>(x, g, b, eps, out, rows, d, amax);
  return cudaGetLastError();
}

}  // namespace esmb200

// Row LayerNorm with the reference's rounding (layernorm.cpp:23-43,
// LayerNormRef): mean and variance accumulated in double, then
// inv_std = 1/sqrtf(float(var) + eps), normed = (x - float(mean)) * inv_std,
// y = fma(normed, g, b) -- the reference's release build contracts that last
// multiply-add into an FMA (its AVX-512 twin, layernorm.cpp:127, uses an
// explicit fmadd there too).  One warp per row; the row stays
// in registers for d <= 2560 (all ESM-2 widths up to 3B).
//
// Fused outputs for the W8A8 path: the absmax of y (per-tensor activation
// scale of the next GEMM) and/or the per-token int8 quantisation of y.
#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

template <int NPL>  // values per lane (d <= 32*NPL)
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                 const float* __restrict__ b, float eps, float* __restrict__ out,
                                 int rows, int d, uint32_t* amax, int8_t* __restrict__ q,
                                 long ldq, float* __restrict__ row_scales) {
  const int lane = threadIdx.x & 31;
  const long r0 = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const bool live = r0 < rows;
  const long r = live ? r0 : rows - 1;  // idle warps recompute the last row, store nothing
  const float* xr = x + r * d;
  float v[NPL];
  double sum = 0.0;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int c = lane + 32 * i;
    v[i] = (c < d) ? xr[c] : 0.0f;
    sum += static_cast<double>(v[i]);
  }
  sum = warp_sum_d(sum);
  const double mean = sum / d;
  double var = 0.0;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int c = lane + 32 * i;
    if (c < d) {
      const double diff = static_cast<double>(v[i]) - mean;
      var += diff * diff;
    }
  }
  var = warp_sum_d(var) / d;
  const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(var), eps)));
  const float meanf = static_cast<float>(mean);
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int c = lane + 32 * i;
    if (c < d) {
      const float normed = __fmul_rn(__fsub_rn(v[i], meanf), inv_std);
      v[i] = __fmaf_rn(normed, __ldg(g + c), __ldg(b + c));
      mx = fmaxf(mx, fabsf(v[i]));
      if (out && live) out[r * d + c] = v[i];
    }
  }
  if (amax != nullptr) amax_publish(amax, mx);  // block-wide: every warp gets here
  if (!live) return;
  if (q != nullptr) {
    mx = warp_max(mx);
    const float s = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, s);
    if (lane == 0) row_scales[r] = s;
    int8_t* qr = q + r * ldq;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int c = lane + 32 * i;
      if (c < d) {
        const int qi = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], inv))));
        qr[c] = static_cast<int8_t>(qi);
      }
    }
    for (int c = d + lane; c < ldq; c += 32) qr[c] = 0;
  }
}

// d > 2560: the same arithmetic reading the row from global memory.
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
  const long threads = static_cast<long>(rows) * 32;
  const int grid = static_cast<int>((threads + 255) / 256);
  const int npl = (d + 31) / 32;
  if (npl <= 4) layernorm_kernel<4><<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
  else if (npl <= 10) layernorm_kernel<10><<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
  else if (npl <= 20) layernorm_kernel<20><<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
  else if (npl <= 40) layernorm_kernel<40><<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
  else if (npl <= 80) layernorm_kernel<80><<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
  else {
    if (q != nullptr || out == nullptr) return cudaErrorInvalidValue;
    layernorm_wide_kernel<<<grid, 256, 0, s>>>(x, g, b, eps, out, rows, d, amax);
  }
  return cudaGetLastError();
}

}  // namespace esmb200

// On-device weight preparation: the SmoothQuant migration of
// smoothquant.cpp:100-185 applied to a model's FP32 weights in HBM.
//
// The migration's per-element steps are single IEEE operations -- a column
// max of |W| (order-free), w * s[k] for the Linear that follows the
// activation, w / s[n] and b / s[n] for the V rows, gamma / s[k] and
// beta / s[k] for the LayerNorm -- so the kernels here give the reference's
// bits.  The scales s themselves (smoothquant.cpp:49-74, one powf pair per
// channel) are computed on the host by the same C library call the
// reference makes; only d values per site cross PCIe.
#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int kColThreads = 256;
constexpr int kRowsPerBlock = 64;

// out[k] = max_n |W[n, k]| folded in as float bits (out zeroed first).
__global__ void __launch_bounds__(kColThreads)
    col_absmax_kernel(const float* __restrict__ W, int N, int K, uint32_t* __restrict__ out) {
  const int k = blockIdx.x * kColThreads + threadIdx.x;
  if (k >= K) return;
  const int n0 = blockIdx.y * kRowsPerBlock;
  const int n1 = min(N, n0 + kRowsPerBlock);
  float m = 0.0f;
  for (int n = n0; n < n1; ++n) m = fmaxf(m, fabsf(__ldg(W + static_cast<long>(n) * K + k)));
  atomicMax(out + k, __float_as_uint(m));
}

// W[n, k] *= s[k] over [N, K].
__global__ void mul_cols_kernel(float* __restrict__ W, long N, int K, const float* __restrict__ s) {
  const long total = N * K;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    W[i] = __fmul_rn(W[i], __ldg(s + i % K));
}

// W[n, k] /= s[n] over [N, K]; b[n] /= s[n] (b nullable).
__global__ void div_rows_kernel(float* __restrict__ W, long N, int K, float* __restrict__ b,
                                const float* __restrict__ s) {
  const long total = N * K;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long n = i / K;
    W[i] = __fdiv_rn(W[i], __ldg(s + n));
    if (b != nullptr && i % K == 0) b[n] = __fdiv_rn(b[n], __ldg(s + n));
  }
}

// x[i] /= s[i] and y[i] /= s[i] (a LayerNorm's gamma and beta).
__global__ void div_vec2_kernel(float* __restrict__ x, float* __restrict__ y, int n,
                                const float* __restrict__ s) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    x[i] = __fdiv_rn(x[i], __ldg(s + i));
    y[i] = __fdiv_rn(y[i], __ldg(s + i));
  }
}

int elem_grid(long n) {
  long g = (n + 255) / 256;
  return static_cast<int>(g < 1 ? 1 : (g > 148L * 32 ? 148L * 32 : g));
}

}  // namespace

cudaError_t launch_col_absmax(const float* W, int N, int K, uint32_t* out, cudaStream_t s) {
  if (K <= 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(K) * 4, s);
  if (e != cudaSuccess || N <= 0) return e;
  dim3 grid((K + kColThreads - 1) / kColThreads, (N + kRowsPerBlock - 1) / kRowsPerBlock);
  col_absmax_kernel<<<grid, kColThreads, 0, s>>>(W, N, K, out);
  return cudaGetLastError();
}

cudaError_t launch_mul_cols(float* W, long N, int K, const float* scales, cudaStream_t s) {
  if (N <= 0 || K <= 0) return cudaSuccess;
  mul_cols_kernel<<<elem_grid(N * K), 256, 0, s>>>(W, N, K, scales);
  return cudaGetLastError();
}

cudaError_t launch_div_rows(float* W, long N, int K, float* bias, const float* scales,
                            cudaStream_t s) {
  if (N <= 0 || K <= 0) return cudaSuccess;
  div_rows_kernel<<<elem_grid(N * K), 256, 0, s>>>(W, N, K, bias, scales);
  return cudaGetLastError();
}

cudaError_t launch_div_vec2(float* x, float* y, int n, const float* scales, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  div_vec2_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, y, n, scales);
  return cudaGetLastError();
}

}  // namespace esmb200

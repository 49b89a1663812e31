// Activation quantisation for the W8A8 GEMMs.
//
// Per-tensor (the reference's semantics, gemm_int8.cpp:391-508): the scale
// is max|A|/127 over the whole [M,K] operand (1 when the tensor is all
// zero) and q = clamp(round_half_even(x * (1/scale)), -127, 127).  The
// absmax is folded into *amax_bits by the kernel that produced A (LayerNorm,
// attention, the fc1 GELU epilogue); this kernel only applies it.
//
// Per-token: the same formula with one scale per row (the reference's
// QuantizeActivationSymmetricRef, pack.cpp:134-147, applied row by row).
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

__device__ __forceinline__ float act_scale_from_amax(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

__device__ __forceinline__ int quant1(float x, float inv) { return quant_int(x, inv); }

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}

// Each thread writes 16 output bytes (one uint4) of one row.
__global__ void quantize_per_tensor_kernel(const float* __restrict__ x, long ldx, int M, int K,
                                           const uint32_t* __restrict__ amax_bits,
                                           int8_t* __restrict__ q, long ldq,
                                           float* __restrict__ scale_out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_amax;
  if (threadIdx.x < 32) {
    const uint32_t m = max(__ldg(amax_bits + threadIdx.x), __ldg(amax_bits + 32 + threadIdx.x));
    const float v = warp_max(__uint_as_float(m));
    if (threadIdx.x == 0) s_amax = v;
  }
  __syncthreads();
  const float s = act_scale_from_amax(s_amax);
  const float inv = __fdiv_rn(1.0f, s);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  // 16-byte groups: the launcher keeps M * ldq / 16 below 2^30, so the
  // row / column split is a 32-bit division.
  const int groups_per_row = static_cast<int>(ldq / 16);
  const int total = M * groups_per_row;
  const bool vec = ((ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < total; g += gridDim.x * blockDim.x) {
    const int m = g / groups_per_row;
    const int c0 = (g - m * groups_per_row) * 16;
    const float* xr = x + static_cast<long>(m) * ldx;
    uint32_t w[4];
    if (vec && c0 + 16 <= K) {
      float4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __ldg(reinterpret_cast<const float4*>(xr + c0 + 4 * i));
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = quant_pack4(v[i], inv);
    } else {
      int qq[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) qq[i] = (c0 + i < K) ? quant1(xr[c0 + i], inv) : 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = pack4(qq[4 * i], qq[4 * i + 1], qq[4 * i + 2], qq[4 * i + 3]);
    }
    *reinterpret_cast<uint4*>(q + static_cast<long>(m) * ldq + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// One warp per row: absmax, scale, quantise.
__global__ void quantize_per_token_kernel(const float* __restrict__ x, long ldx, int M, int K,
                                          int8_t* __restrict__ q, long ldq,
                                          float* __restrict__ row_scales) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long m = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  if (m >= M) return;
  const float* xr = x + m * ldx;
  float mx = 0.0f;
  for (int c = lane; c < K; c += 32) mx = fmaxf(mx, fabsf(xr[c]));
  mx = warp_max(mx);
  const float s = act_scale_from_amax(mx);
  const float inv = __fdiv_rn(1.0f, s);
  if (lane == 0) row_scales[m] = s;
  int8_t* qr = q + m * ldq;
  for (int c = lane; c < ldq; c += 32) qr[c] = static_cast<int8_t>(c < K ? quant1(xr[c], inv) : 0);
}

__global__ void absmax_kernel(const float* __restrict__ x, long n, uint32_t* amax_bits) {
  float mx = 0.0f;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    mx = fmaxf(mx, fabsf(x[i]));
  amax_publish(amax_bits, mx);
}

// x = float(half(x)), round to nearest even (the layer-0 fc1 input escape,
// model.cpp:912-930, 1031-1033); with amax_bits, also the absmax of the
// rounded values.
__global__ void round_fp16_kernel(float* __restrict__ x, long n, uint32_t* amax_bits) {
  float mx = 0.0f;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float r = __half2float(__float2half_rn(x[i]));
    x[i] = r;
    mx = fmaxf(mx, fabsf(r));
  }
  if (amax_bits != nullptr) amax_publish(amax_bits, mx);
}

// quant::Quantize (pack.cpp:149-177): per output channel (row) n,
// scale = max|W[n,:]| / 127 (IEEE divide), inv = 1 / scale, q = clamp(
// rne(w * inv), +-127); an all-zero row gets scale 0 and zero codes.  One warp
// per row; the max is order-free, so the codes and scales are bit-identical
// to the reference's.
__global__ void quantize_weight_rows_kernel(const float* __restrict__ W, int N, int K,
                                            int8_t* __restrict__ q, long ldq,
                                            float* __restrict__ scale) {
  const int warps = static_cast<int>(blockDim.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  for (long n = static_cast<long>(blockIdx.x) * warps + (threadIdx.x >> 5); n < N;
       n += static_cast<long>(gridDim.x) * warps) {
    const float* row = W + n * K;
    int8_t* qr = q + n * ldq;
    float mx = 0.0f;
    for (int k = lane; k < K; k += 32) mx = fmaxf(mx, fabsf(row[k]));
    mx = warp_max(mx);
    if (mx == 0.0f) {
      if (lane == 0) scale[n] = 0.0f;
      for (int k = lane; k < K; k += 32) qr[k] = 0;
      continue;
    }
    const float sc = __fdiv_rn(mx, 127.0f);
    const float inv = __fdiv_rn(1.0f, sc);
    if (lane == 0) scale[n] = sc;
    for (int k = lane; k < K; k += 32) {
      const float v = fminf(fmaxf(rintf(__fmul_rn(row[k], inv)), -127.0f), 127.0f);
      qr[k] = static_cast<int8_t>(static_cast<int>(v));
    }
  }
}

int grid_for(long work, int block) {
  long g = (work + block - 1) / block;
  if (g > 148L * 16) g = 148L * 16;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t launch_quantize_per_tensor(const float* x, long ldx, int M, int K,
                                       const uint32_t* amax_bits, int8_t* q, long ldq,
                                       float* scale_out, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if ((ldq & 15) || ldq < K || (reinterpret_cast<uintptr_t>(q) & 15)) return cudaErrorInvalidValue;
  const long work = static_cast<long>(M) * (ldq / 16);
  if (work >= (1l << 30)) return cudaErrorInvalidValue;
  return launch_pdl(quantize_per_tensor_kernel, dim3(grid_for(work, 256)), dim3(256), 0, s, x, ldx,
                    M, K, amax_bits, q, ldq, scale_out);
}

cudaError_t launch_quantize_per_token(const float* x, long ldx, int M, int K, int8_t* q,
                                      long ldq, float* row_scales, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if (ldq < K) return cudaErrorInvalidValue;
  const long threads = static_cast<long>(M) * 32;
  return launch_pdl(quantize_per_token_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)),
                    dim3(256), 0, s, x, ldx, M, K, q, ldq, row_scales);
}

cudaError_t launch_quantize_weights(const float* W, int N, int K, int8_t* q, long ldq,
                                    float* scale, cudaStream_t s) {
  if (N <= 0 || K <= 0) return cudaSuccess;
  if (ldq < K) return cudaErrorInvalidValue;
  quantize_weight_rows_kernel<<<grid_for(static_cast<long>(N) * 32, 256), 256, 0, s>>>(W, N, K, q,
                                                                                     ldq, scale);
  return cudaGetLastError();
}

cudaError_t launch_round_fp16(float* x, long n, uint32_t* amax_bits, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  round_fp16_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, amax_bits);
  return cudaGetLastError();
}

cudaError_t launch_absmax(const float* x, long n, uint32_t* amax_bits, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  absmax_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, amax_bits);
  return cudaGetLastError();
}

}  // namespace esmb200

// FP32 GEMM C = A[M,K] . W[N,K]^T + bias (the reference's Linear /
// LinearAvx512, gemm_fp32.cpp:272-292, W in PyTorch [out, in] layout).
// Used by the LM head (dense d x d and the tied decoder V x d) and by every
// Linear of an unquantised model.  FP32 SIMT: 128x128 CTA tile, K step 8,
// 256 threads with an 8x8 register tile, double-buffered shared memory.
// Parity with the reference is at FP32 rounding (1e-4 relative class): the
// summation order differs from the reference's, the arithmetic does not.
#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int TM = 128, TN = 128, TK = 8;

template <bool VEC>
__global__ void __launch_bounds__(256)
    gemm_f32_kernel(const float* __restrict__ A, long lda, const float* __restrict__ W, long ldw,
                    int M, int N, int K, const float* __restrict__ bias, EpiParams e) {
  __shared__ __align__(16) float As[2][TK][TM + 4];
  __shared__ __align__(16) float Ws[2][TK][TN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const long m0 = static_cast<long>(blockIdx.y) * TM;
  const int n0 = blockIdx.x * TN;
  // Loader mapping: thread -> (row lr, k quad lk) of a 128 x 8 tile.
  const int lr = tid >> 1, lk = (tid & 1) * 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  auto load = [&](int k0, float (&ra)[4], float (&rw)[4]) {
    const long am = m0 + lr;
    const int wn = n0 + lr;
    if (VEC) {
      const bool ka = k0 + lk + 3 < K;
      float4 a = make_float4(0, 0, 0, 0), w = make_float4(0, 0, 0, 0);
      if (am < M && ka) a = __ldg(reinterpret_cast<const float4*>(A + am * lda + k0 + lk));
      if (wn < N && ka) w = __ldg(reinterpret_cast<const float4*>(W + static_cast<long>(wn) * ldw + k0 + lk));
      ra[0] = a.x; ra[1] = a.y; ra[2] = a.z; ra[3] = a.w;
      rw[0] = w.x; rw[1] = w.y; rw[2] = w.z; rw[3] = w.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kk = k0 + lk + i;
        ra[i] = (am < M && kk < K) ? A[am * lda + kk] : 0.0f;
        rw[i] = (wn < N && kk < K) ? W[static_cast<long>(wn) * ldw + kk] : 0.0f;
      }
    }
  };
  auto store = [&](int buf, const float (&ra)[4], const float (&rw)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      As[buf][lk + i][lr] = ra[i];
      Ws[buf][lk + i][lr] = rw[i];
    }
  };

  float ra[4], rw[4];
  load(0, ra, rw);
  store(0, ra, rw);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += TK) {
    const bool more = k0 + TK < K;
    if (more) load(k0 + TK, ra, rw);
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[8], w[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 w0 = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
      const float4 w1 = *reinterpret_cast<const float4*>(&Ws[buf][kk][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w;
      w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], w[j], acc[i][j]);
    }
    if (more) {
      store(buf ^ 1, ra, rw);
      __syncthreads();
      buf ^= 1;
    }
  }

  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int c0 = n0 + half * 64 + tx * 4;
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = min(c0 + j, N - 1);
        y[j] = __fadd_rn(acc[i][half * 4 + j], bias ? __ldg(bias + n) : 0.0f);
      }
      mx = fmaxf(mx, epi_row_run<4>(e, m, c0, N, y));
    }
  }
  if (e.amax != nullptr) amax_publish(e.amax, mx);
}

}  // namespace

cudaError_t launch_gemm_f32(const GemmF32Args& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  if (a.epi.kind == kEpiQkvRope) return cudaErrorInvalidValue;
  dim3 grid((a.N + TN - 1) / TN, (a.M + TM - 1) / TM);
  const bool vec = (a.K % 4 == 0) && (a.lda % 4 == 0) && (a.ldw % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(a.A) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(a.W) & 15) == 0);
  if (vec) gemm_f32_kernel<true><<<grid, 256, 0, s>>>(a.A, a.lda, a.W, a.ldw, a.M, a.N, a.K, a.bias, a.epi);
  else gemm_f32_kernel<false><<<grid, 256, 0, s>>>(a.A, a.lda, a.W, a.ldw, a.M, a.N, a.K, a.bias, a.epi);
  return cudaGetLastError();
}

}  // namespace esmb200

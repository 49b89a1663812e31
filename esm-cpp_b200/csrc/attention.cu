// Packed-varlen bidirectional attention (replaces the reference's
// AttentionVarlenAvx512 / AttentionVarlenRef, attention.cpp:99-144, 240-430,
// 770-811).  Q arrives pre-scaled by 1/sqrt(dh) and RoPE'd; each query of
// sequence b attends to the keys of sequence b only (cu_seqlens isolation).
//
// This FP32 SIMT kernel serves head dims other than 64 and sequences longer
// than 256 tokens; attention_tma.cu covers the rest on the tensor cores.
// One CTA per (sequence, head); each thread owns one query
// row (q and the output accumulator live in registers) and streams the
// sequence's keys/values through shared memory in 32-row tiles with an
// online (running-max) softmax, so any length up to the tokenizer's 1024
// runs in constant shared memory.  Scores, exponentials and the output are
// FP32; the result matches the reference within FP32 rounding (the
// reference's Ref twin sums the softmax denominator in double, its AVX-512
// path in float).
#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int KT = 32;        // keys per shared-memory tile
constexpr int QT = 128;       // queries (threads) per CTA pass

template <int DH>
__global__ void __launch_bounds__(QT)
    attention_varlen_kernel(const float* __restrict__ q, const float* __restrict__ k,
                            const float* __restrict__ v, const int* __restrict__ cu, int H,
                            int dh, float* __restrict__ out, uint32_t* amax, int min_len) {
  __shared__ __align__(16) float sK[KT][DH];
  __shared__ __align__(16) float sV[KT][DH];
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int s0 = __ldg(cu + b);
  const int L = __ldg(cu + b + 1) - s0;
  if (L <= 0 || L <= min_len) return;  // shorter sequences run on the tensor-core kernel
  const long row_stride = static_cast<long>(H) * dh;
  float mx_out = 0.0f;

  for (int q0 = 0; q0 < L; q0 += QT) {
    const int i = q0 + threadIdx.x;
    const bool active = i < L;
    float qr[DH], o[DH];
    const float* qp = q + (s0 + (active ? i : 0)) * row_stride + static_cast<long>(h) * dh;
#pragma unroll
    for (int d = 0; d < DH; ++d) {
      qr[d] = (d < dh) ? qp[d] : 0.0f;
      o[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;

    for (int j0 = 0; j0 < L; j0 += KT) {
      const int nk = min(KT, L - j0);
      __syncthreads();
      for (int e = threadIdx.x; e < KT * DH; e += QT) {
        const int jj = e / DH, d = e % DH;
        float kv = 0.0f, vv = 0.0f;
        if (jj < nk && d < dh) {
          const long off = (s0 + j0 + jj) * row_stride + static_cast<long>(h) * dh + d;
          kv = __ldg(k + off);
          vv = __ldg(v + off);
        }
        sK[jj][d] = kv;
        sV[jj][d] = vv;
      }
      __syncthreads();

      float s[KT];
      float tmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < KT; ++jj) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(&sK[jj][d]);
          a0 = __fmaf_rn(qr[d], kk.x, a0);
          a1 = __fmaf_rn(qr[d + 1], kk.y, a1);
          a2 = __fmaf_rn(qr[d + 2], kk.z, a2);
          a3 = __fmaf_rn(qr[d + 3], kk.w, a3);
        }
        s[jj] = (jj < nk) ? __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)) : -INFINITY;
        tmax = fmaxf(tmax, s[jj]);
      }
      const float m_new = fmaxf(m, tmax);
      const float corr = expf(__fsub_rn(m, m_new));  // 0 on the first tile
      l = __fmul_rn(l, corr);
#pragma unroll
      for (int d = 0; d < DH; ++d) o[d] = __fmul_rn(o[d], corr);
#pragma unroll
      for (int jj = 0; jj < KT; ++jj) {
        const float p = (jj < nk) ? expf(__fsub_rn(s[jj], m_new)) : 0.0f;
        l = __fadd_rn(l, p);
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
          const float4 vv = *reinterpret_cast<const float4*>(&sV[jj][d]);
          o[d] = __fmaf_rn(p, vv.x, o[d]);
          o[d + 1] = __fmaf_rn(p, vv.y, o[d + 1]);
          o[d + 2] = __fmaf_rn(p, vv.z, o[d + 2]);
          o[d + 3] = __fmaf_rn(p, vv.w, o[d + 3]);
        }
      }
      m = m_new;
    }

    if (active) {
      const float inv = l > 0.0f ? __fdiv_rn(1.0f, l) : 0.0f;
      float* op = out + (s0 + i) * row_stride + static_cast<long>(h) * dh;
      if (dh == DH) {
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
          const float4 r = make_float4(__fmul_rn(o[d], inv), __fmul_rn(o[d + 1], inv),
                                       __fmul_rn(o[d + 2], inv), __fmul_rn(o[d + 3], inv));
          *reinterpret_cast<float4*>(op + d) = r;
          mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(r.x), fabsf(r.y)), fmaxf(fabsf(r.z), fabsf(r.w))));
        }
      } else {
        for (int d = 0; d < dh; ++d) {
          const float r = __fmul_rn(o[d], inv);
          op[d] = r;
          mx_out = fmaxf(mx_out, fabsf(r));
        }
      }
    }
  }
  if (amax != nullptr) amax_publish(amax, mx_out);
}

}  // namespace

cudaError_t launch_attention_tma(const float* q, const float* k, const float* v, const int* cu,
                                 int B, int H, long T, float* out, uint32_t* amax,
                                 uint32_t* status, int num_sms, bool qk_bf16, cudaStream_t s);
cudaError_t launch_attention_tma_pair(const float* q, const float* k, const float* v,
                                      const int* cu, int B, int H, long T, float* out,
                                      uint32_t* amax, uint32_t* status, int num_sms, bool qk_bf16,
                                      cudaStream_t s, bool wait_late);
cudaError_t launch_attention_tma_long(const float* q, const float* k, const float* v,
                                      const int* cu, int B, int H, long T, int max_len, float* out,
                                      uint32_t* amax, uint32_t* status, int num_sms, bool qk_bf16,
                                      cudaStream_t s, bool wait_late);

cudaError_t launch_attention_varlen(const float* q, const float* k, const float* v,
                                    const int* cu, int B, int H, int dh, long T, int min_len,
                                    int max_len, float* out, uint32_t* amax, uint32_t* status,
                                    int num_sms, cudaStream_t s, bool qk_bf16) {
  if (B <= 0 || H <= 0 || max_len <= 0) return cudaSuccess;
  if (dh <= 0 || dh > 128 || (dh & 3)) return cudaErrorInvalidValue;
  // head_dim 64: tensor cores (3xTF32) -- one CTA per (sequence, head) for
  // L <= 128, a CTA pair for 129..256, one CTA per (sequence, head, 128-row
  // query tile) above; other head dims: FP32 SIMT.
  if (dh == 64 && status != nullptr) {
    // A kernel that follows another of these (same inputs, other sequences)
    // waits for it at its end, not its start (wait_late): it runs in the
    // earlier kernel's tail and still completes after it.
    bool after = false;
    if (min_len <= 128) {
      cudaError_t e =
          launch_attention_tma(q, k, v, cu, B, H, T, out, amax, status, num_sms, qk_bf16, s);
      if (e != cudaSuccess) return e;
      after = true;
    }
    if (max_len > 128 && min_len <= 256) {
      cudaError_t e = launch_attention_tma_pair(q, k, v, cu, B, H, T, out, amax, status, num_sms,
                                                qk_bf16, s, after);
      if (e != cudaSuccess) return e;
      after = true;
    }
    if (max_len > 256) {
      cudaError_t e = launch_attention_tma_long(q, k, v, cu, B, H, T, max_len, out, amax, status,
                                                num_sms, qk_bf16, s, after);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  const int min_len_simt = 0;
  dim3 grid(H, B);
  if (dh <= 16) attention_varlen_kernel<16><<<grid, QT, 0, s>>>(q, k, v, cu, H, dh, out, amax, min_len_simt);
  else if (dh <= 32) attention_varlen_kernel<32><<<grid, QT, 0, s>>>(q, k, v, cu, H, dh, out, amax, min_len_simt);
  else if (dh <= 64) attention_varlen_kernel<64><<<grid, QT, 0, s>>>(q, k, v, cu, H, dh, out, amax, min_len_simt);
  else attention_varlen_kernel<128><<<grid, QT, 0, s>>>(q, k, v, cu, H, dh, out, amax, min_len_simt);
  return cudaGetLastError();
}

}  // namespace esmb200

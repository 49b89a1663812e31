// Elementwise glue of the forward: GELU, residual add, Q scale, varlen RoPE,
// the q|k|v split for the FP32 path, token positions and the embedding
// gather with the per-sequence token-dropout rescale.
#include <cuda_bf16.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

inline int grid_for(long work, int block) {
  long g = (work + block - 1) / block;
  if (g > 148L * 32) g = 148L * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

// Two elements per thread and step through gelu_erf2 (the GEMM epilogue's
// form), the odd tail through gelu_erf.
__global__ void gelu_kernel(const float* __restrict__ x, float* __restrict__ out, long n) {
  const long np = n / 2;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < np;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    float a = x[2 * i], b = x[2 * i + 1];
    gelu_erf2(a, b);
    out[2 * i] = a;
    out[2 * i + 1] = b;
  }
  if ((n & 1) && blockIdx.x == 0 && threadIdx.x == 0) out[n - 1] = gelu_erf(x[n - 1]);
}

__global__ void residual_kernel(float* __restrict__ y, const float* __restrict__ x, long n) {
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    y[i] = __fadd_rn(y[i], x[i]);
}

// y = float(bf16(x)), round to nearest even: the Q and K of the reference's
// opt-in BF16 attention (attention.cpp:686-700, 707-768 converts them with
// _mm512_cvtne2ps_pbh).
__global__ void round_bf16_kernel(const float* x, float* y, long n) {
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    y[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
}

// lo = x - tf32(x): the part of an fp32 operand a tf32 MMA drops (it reads
// the fp32 word with its low 13 mantissa bits cleared).
__global__ void tf32_lo_kernel(const float* __restrict__ x, float* __restrict__ lo, long n) {
  pdl_wait();
  pdl_trigger();
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    lo[i] = __fsub_rn(v, __uint_as_float(__float_as_uint(v) & 0xFFFFE000u));
  }
}

__global__ void scale_kernel(float* __restrict__ x, long n, float s) {
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    x[i] = __fmul_rn(x[i], s);
}

// Sequence index of token t: the last b with cu[b] <= t (cu has B+1 entries).
__device__ __forceinline__ int seq_of(const int* cu, int B, int t) {
  int lo = 0, hi = B;  // invariant: cu[lo] <= t < cu[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

// rope.cpp:90-152 (AVX-512 form): in place on [T, H, dh]; one thread per
// (token, head, i < dh/2).
__global__ void rope_varlen_kernel(float* __restrict__ x, const float* __restrict__ cos_t,
                                   const float* __restrict__ sin_t, const int* __restrict__ cu,
                                   int B, int H, int dh) {
  const int half = dh / 2;
  const int T = __ldg(cu + B);
  const long total = static_cast<long>(T) * H * half;
  for (long w = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(w % half);
    const long th = w / half;
    const int t = static_cast<int>(th / H);
    const int p = t - __ldg(cu + seq_of(cu, B, t));
    float* xr = x + th * dh;
    const float c = __ldg(cos_t + static_cast<long>(p) * dh + i);
    const float s = __ldg(sin_t + static_cast<long>(p) * dh + i);
    const float lo = xr[i], hi = xr[i + half];
    xr[i] = __fmaf_rn(-hi, s, __fmul_rn(lo, c));
    xr[i + half] = __fmaf_rn(hi, c, __fmul_rn(lo, s));
  }
}

// qkv [T, 3d] -> q, k, v [T, d] with q *= q_scale then RoPE on q, k.
__global__ void split_qkv_rope_kernel(const float* __restrict__ qkv, float* __restrict__ q,
                                      float* __restrict__ k, float* __restrict__ v, int T, int d,
                                      int H, int dh, const int* __restrict__ pos,
                                      const float* __restrict__ cos_t,
                                      const float* __restrict__ sin_t, float q_scale, int qk_bf16) {
  const int half = dh / 2;
  const long total = static_cast<long>(T) * H * half;
  for (long w = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; w < total;
       w += static_cast<long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(w % half);
    const long th = w / half;
    const long t = th / H;
    const int h = static_cast<int>(th - t * H);
    const float* src = qkv + t * 3L * d + static_cast<long>(h) * dh;
    const long o = t * d + static_cast<long>(h) * dh;
    const int p = __ldg(pos + t);
    const float c = __ldg(cos_t + static_cast<long>(p) * dh + i);
    const float s = __ldg(sin_t + static_cast<long>(p) * dh + i);
    // q: scale before RoPE (model.cpp:976-988)
    // ESM_AMX_ATTENTION: q and k stored rounded to bf16.
    auto st = [qk_bf16](float x) { return qk_bf16 ? __bfloat162float(__float2bfloat16_rn(x)) : x; };
    float lo = __fmul_rn(src[i], q_scale), hi = __fmul_rn(src[i + half], q_scale);
    q[o + i] = st(__fmaf_rn(-hi, s, __fmul_rn(lo, c)));
    q[o + i + half] = st(__fmaf_rn(hi, c, __fmul_rn(lo, s)));
    lo = src[d + i];
    hi = src[d + i + half];
    k[o + i] = st(__fmaf_rn(-hi, s, __fmul_rn(lo, c)));
    k[o + i + half] = st(__fmaf_rn(hi, c, __fmul_rn(lo, s)));
    v[o + i] = src[2 * d + i];
    v[o + i + half] = src[2 * d + i + half];
  }
}

__global__ void positions_kernel(const int* __restrict__ cu, int B, int* __restrict__ pos) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  if (b >= B) return;
  const int s0 = cu[b], s1 = cu[b + 1];
  for (int t = s0 + threadIdx.x; t < s1; t += blockDim.x) pos[t] = t - s0;
}

// model.cpp:737-778 Embed: one block per sequence.  scale =
// (1 - 0.15f*0.8f) / max(1 - masks_seen/real_tokens, 1e-12); mask-token and
// pad rows are zero.
__global__ void embed_kernel(const float* __restrict__ embed_w, int d, const int* __restrict__ ids,
                             const int* __restrict__ masks, const int* __restrict__ cu, int B,
                             int mask_id, float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ int s_counts[2];
  const int b = blockIdx.x;
  if (b >= B) return;
  const int s0 = cu[b], s1 = cu[b + 1];
  if (threadIdx.x == 0) {
    s_counts[0] = 0;
    s_counts[1] = 0;
  }
  __syncthreads();
  int src = 0, obs = 0;
  for (int t = s0 + threadIdx.x; t < s1; t += blockDim.x) {
    if (masks == nullptr || masks[t] != 0) ++src;
    if (ids[t] == mask_id) ++obs;
  }
  atomicAdd(&s_counts[0], src);
  atomicAdd(&s_counts[1], obs);
  __syncthreads();
  const int src_len = s_counts[0], observed = s_counts[1];
  const float ratio_train = __fmul_rn(0.15f, 0.8f);
  const float obs_ratio =
      src_len > 0 ? __fdiv_rn(static_cast<float>(observed), static_cast<float>(src_len)) : 0.0f;
  const float denom = fmaxf(__fsub_rn(1.0f, obs_ratio), 1e-12f);
  const float scale = __fdiv_rn(__fsub_rn(1.0f, ratio_train), denom);
  // Rows: one warp per token, blockIdx.y splitting the sequence's tokens over
  // gridDim.y blocks (each recomputes the sequence's counts above), float4
  // columns when d % 4 == 0 and the tables are 16-byte aligned.
  const int nw = static_cast<int>(blockDim.x >> 5), warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int step = nw * static_cast<int>(gridDim.y);
  const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(embed_w) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  for (int t = s0 + static_cast<int>(blockIdx.y) * nw + warp; t < s1; t += step) {
    const int id = ids[t];
    const bool zero = (id == mask_id) || (masks != nullptr && masks[t] == 0);
    const float* src = embed_w + static_cast<long>(id) * d;
    float* dst = out + static_cast<long>(t) * d;
    if (vec) {
      for (int c4 = lane; c4 < d / 4; c4 += 32) {
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (!zero) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(src) + c4);
          v = make_float4(__fmul_rn(w.x, scale), __fmul_rn(w.y, scale), __fmul_rn(w.z, scale),
                          __fmul_rn(w.w, scale));
        }
        reinterpret_cast<float4*>(dst)[c4] = v;
      }
    } else {
      for (int c = lane; c < d; c += 32) dst[c] = zero ? 0.0f : __fmul_rn(__ldg(src + c), scale);
    }
  }
}

// out[r] = x[rows[r]] for rows of d floats: the masked positions that the
// masked-marginal head scores (eval/proteingym.py:84-88 reads logits[p + 1]
// of each masked copy).  One block per selected row.
__global__ void gather_rows_kernel(const float* __restrict__ x, const int* __restrict__ rows, int d,
                                   float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const float* src = x + static_cast<long>(__ldg(rows + blockIdx.x)) * d;
  float* dst = out + static_cast<long>(blockIdx.x) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
}

// In place, each row of x [R, V]: (x - max) - log(sum(exp(x - max))), the
// order of eval/proteingym.py:48-50.  One warp per row.
__global__ void log_softmax_rows_kernel(float* __restrict__ x, int R, int V) {
  pdl_wait();
  pdl_trigger();
  const long row = (blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  float* xr = x + row * V;
  float mx = -INFINITY;
  for (int j = lane; j < V; j += 32) mx = fmaxf(mx, xr[j]);
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.0f;
  for (int j = lane; j < V; j += 32) sum = __fadd_rn(sum, expf(__fsub_rn(xr[j], mx)));
  for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  const float lse = logf(sum);
  for (int j = lane; j < V; j += 32) xr[j] = __fsub_rn(__fsub_rn(xr[j], mx), lse);
}

}  // namespace

cudaError_t launch_gelu(const float* x, float* out, long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  gelu_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, out, n);
  return cudaGetLastError();
}

cudaError_t launch_residual_add(float* y, const float* x, long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  residual_kernel<<<grid_for(n, 256), 256, 0, s>>>(y, x, n);
  return cudaGetLastError();
}

cudaError_t launch_round_bf16(const float* x, float* y, long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  round_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, y, n);
  return cudaGetLastError();
}

cudaError_t launch_tf32_lo(const float* x, float* lo, long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  return launch_pdl(tf32_lo_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, x, lo, n);
}

cudaError_t launch_scale(float* x, long n, float sc, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  scale_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, sc);
  return cudaGetLastError();
}

cudaError_t launch_rope_varlen(float* x, const float* cos_t, const float* sin_t, const int* cu,
                               int B, int H, int dh, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  // T is read on the device from cu[B]; size the grid for a generous bound.
  rope_varlen_kernel<<<148 * 8, 256, 0, s>>>(x, cos_t, sin_t, cu, B, H, dh);
  return cudaGetLastError();
}

cudaError_t launch_split_qkv_rope(const float* qkv, float* q, float* k, float* v, int T, int d,
                                  int H, int dh, const int* pos, const float* cos_t,
                                  const float* sin_t, float q_scale, cudaStream_t s,
                                  bool qk_bf16) {
  if (T <= 0) return cudaSuccess;
  const long work = static_cast<long>(T) * H * (dh / 2);
  split_qkv_rope_kernel<<<grid_for(work, 256), 256, 0, s>>>(qkv, q, k, v, T, d, H, dh, pos,
                                                            cos_t, sin_t, q_scale, qk_bf16 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_positions(const int* cu, int B, int* pos, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  return launch_pdl(positions_kernel, dim3(B), dim3(128), 0, s, cu, B, pos);
}

cudaError_t launch_embed(const float* embed_w, int d, const int* ids, const int* masks,
                         const int* cu, int B, int mask_id, float* out, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  return launch_pdl(embed_kernel, dim3(B, 4), dim3(256), 0, s, embed_w, d, ids, masks, cu, B, mask_id,
                    out);
}

cudaError_t launch_gather_rows(const float* x, const int* rows, int R, int d, float* out,
                               cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  return launch_pdl(gather_rows_kernel, dim3(R), dim3(128), 0, s, x, rows, d, out);
}

cudaError_t launch_log_softmax_rows(float* x, int R, int V, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  const long threads = static_cast<long>(R) * 32;  // one warp per row
  return launch_pdl(log_softmax_rows_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)),
                    dim3(256), 0, s, x, R, V);
}

}  // namespace esmb200

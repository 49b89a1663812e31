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
#include <algorithm>
#include <atomic>

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
  pdl_wait();
  pdl_trigger();
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

// ------------------------------------------------ LayerNorm + quantisation
// The per-tensor W8A8 path only needs LN(x) as int8 with one scale over the
// whole [rows, d] output, so the fp32 output is never written: phase 1 finds
// every row's statistics and the absmax of y; after a grid-wide barrier
// phase 2 recomputes y from x (still in L2) and quantises it.  One warp per
// row, lane l holding columns 4 l + 128 i (d = 128 NV).

// Grid-wide barrier for a cooperative launch, used once per launch: `counter`
// is zero before the launch; the wait is bounded like the mbarrier waits.
__device__ __forceinline__ void grid_barrier_once(uint32_t* counter, uint32_t* status) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(counter, 1u);
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
      uint32_t cur;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(counter) : "memory");
      if (cur >= gridDim.x) break;
      if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitNs) {
        atomicOr(status, kStatusTimeout);
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
  }
  __syncthreads();
}

// y = fma((x - mean) * inv_std, g, b) on four columns.
__device__ __forceinline__ float4 ln_y4(float4 v, float meanf, float inv_std, float4 gg, float4 bv) {
  return make_float4(__fmaf_rn(__fmul_rn(__fsub_rn(v.x, meanf), inv_std), gg.x, bv.x),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.y, meanf), inv_std), gg.y, bv.y),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.z, meanf), inv_std), gg.z, bv.z),
                     __fmaf_rn(__fmul_rn(__fsub_rn(v.w, meanf), inv_std), gg.w, bv.w));
}

__device__ __forceinline__ uint32_t quant4(float4 y, float inv) {
  const int a0 = max(-127, min(127, __float2int_rn(__fmul_rn(y.x, inv))));
  const int a1 = max(-127, min(127, __float2int_rn(__fmul_rn(y.y, inv))));
  const int a2 = max(-127, min(127, __float2int_rn(__fmul_rn(y.z, inv))));
  const int a3 = max(-127, min(127, __float2int_rn(__fmul_rn(y.w, inv))));
  return (static_cast<uint32_t>(a0) & 0xffu) | ((static_cast<uint32_t>(a1) & 0xffu) << 8) |
         ((static_cast<uint32_t>(a2) & 0xffu) << 16) | ((static_cast<uint32_t>(a3) & 0xffu) << 24);
}

// 12 warps per block, a row per warp.  Up to d = 2048 (NV <= 16) two blocks
// share an SM (at most 80 registers: gamma and beta come from shared memory
// and the statistics take one pass); d = 2560 (ESM-2 3B, NV = 20) holds 80
// floats of the row per lane and runs one block per SM.
constexpr int kLqThreads = 384;

template <int NV>
__global__ void __launch_bounds__(kLqThreads, NV <= 16 ? 2 : 1)
    ln_quant_kernel(const float* __restrict__ x, const float* __restrict__ g,
                    const float* __restrict__ b, float eps, int rows, int d, uint32_t* amax,
                    float2* stats, uint32_t* counter, int8_t* __restrict__ q, long ldq,
                    float* scale_out, uint32_t* status) {
  const int lane = threadIdx.x & 31;
  const long warp_g = static_cast<long>(blockIdx.x) * (kLqThreads / 32) + (threadIdx.x >> 5);
  const long nwarps = static_cast<long>(gridDim.x) * (kLqThreads / 32);
  __shared__ __align__(16) float s_gb[2 * 128 * NV];  // gamma | beta
  for (int i = threadIdx.x; i < d; i += kLqThreads) {
    s_gb[i] = __ldg(g + i);
    s_gb[128 * NV + i] = __ldg(b + i);
  }
  // x, the absmax slots and the barrier counter come from earlier work of
  // the stream (the weights above do not).
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const uint32_t sg = smem_u32(s_gb), sb = sg + 128u * NV * 4u;
  auto load_row = [&](long r, float4 (&v)[NV]) {
    const float* xr = x + r * d;
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = __ldg(reinterpret_cast<const float4*>(xr + 4 * lane + 128 * i));
  };
  // ---- phase 1: statistics and absmax of y
  float tmax = 0.0f;
  // Mean and variance in double in one pass (sum and sum of squares, two
  // partial chains each, one combined warp reduction): var = E[x^2] - mean^2
  // differs from the two-pass double variance by ~1e-12 relative, far below
  // the float rounding of var that follows.
  auto stats_row = [&](long r, const float4 (&v)[NV]) {
    double s0 = 0.0, s1 = 0.0, q0 = 0.0, q1 = 0.0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const double a = v[i].x, bb = v[i].y, cc = v[i].z, dd = v[i].w;
      s0 += a + bb;
      s1 += cc + dd;
      q0 = fma(a, a, fma(bb, bb, q0));
      q1 = fma(cc, cc, fma(dd, dd, q1));
    }
    double sum = s0 + s1, sq = q0 + q1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
    }
    const double mean = sum / d;
    const double var = fmax(sq / d - mean * mean, 0.0);
    const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(var), eps)));
    const float meanf = static_cast<float>(mean);
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * lane + 128 * i;
      const float4 y = ln_y4(v[i], meanf, inv_std, lds128(sg + c * 4u), lds128(sb + c * 4u));
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
    }
    if (lane == 0) stats[r] = make_float2(meanf, inv_std);
    tmax = fmaxf(tmax, mx);
  };
  for (long r = warp_g; r < rows; r += nwarps) {
    float4 va[NV];
    load_row(r, va);
    stats_row(r, va);
  }
  amax_publish(amax, tmax);
  grid_barrier_once(counter, status);
  // ---- phase 2: scale from the finished absmax, then y -> int8
  __shared__ float s_inv;
  if (threadIdx.x < 32) {
    uint32_t m0, m1;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(m0) : "l"(amax + threadIdx.x) : "memory");
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(m1) : "l"(amax + 32 + threadIdx.x) : "memory");
    const float am = warp_max(__uint_as_float(max(m0, m1)));
    if (threadIdx.x == 0) {
      const float sc = am > 0.0f ? __fdiv_rn(am, 127.0f) : 1.0f;
      s_inv = __fdiv_rn(1.0f, sc);
      if (blockIdx.x == 0) *scale_out = sc;
    }
  }
  __syncthreads();
  const float inv = s_inv;
  auto quant_row = [&](long r, const float4 (&v)[NV]) {
    const float2 st = __ldcg(stats + r);
    int8_t* qr = q + r * ldq;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * lane + 128 * i;
      const float4 y = ln_y4(v[i], st.x, st.y, lds128(sg + c * 4u), lds128(sb + c * 4u));
      *reinterpret_cast<uint32_t*>(qr + c) = quant4(y, inv);
    }
    for (long c = d + lane; c < ldq; c += 32) qr[c] = 0;
  };
  for (long r = warp_g; r < rows; r += nwarps) {
    float4 va[NV];
    load_row(r, va);
    quant_row(r, va);
  }
}

template <int NV>
cudaError_t launch_lq(const float* x, const float* g, const float* b, float eps, int rows, int d,
                      uint32_t* amax, float2* stats, uint32_t* counter, int8_t* q, long ldq,
                      float* scale_out, uint32_t* status, cudaStream_t s) {
  static std::atomic<int> blocks_per_sm[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = blocks_per_sm[dev & 63].load();
  int sms = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (per_sm == 0) {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ln_quant_kernel<NV>, kLqThreads, 0);
    if (e != cudaSuccess) return e;
    if (per_sm <= 0) return cudaErrorNotSupported;
    blocks_per_sm[dev & 63].store(per_sm);
  }
  const long want = (static_cast<long>(rows) + kLqThreads / 32 - 1) / (kLqThreads / 32);
  const int grid = static_cast<int>(std::max(1L, std::min<long>(want, static_cast<long>(per_sm) * sms)));
  // Cooperative (for the grid barrier) and with programmatic dependent
  // launch, so the launch and the gamma / beta loads overlap the previous
  // kernel's tail.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kLqThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1] = pdl_attribute();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, ln_quant_kernel<NV>, x, g, b, eps, rows, d, amax, stats, counter, q,
                            ldq, scale_out, status);
}

}  // namespace

cudaError_t launch_layernorm_quant(const float* x, const float* g, const float* b, float eps,
                                   int rows, int d, uint32_t* amax, float2* stats,
                                   uint32_t* counter, int8_t* q, long ldq, float* scale_out,
                                   uint32_t* status, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) |
                         reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(q)) & 15) == 0;
  if (d % 128 != 0 || d > 2560 || !aligned || ldq < d || (ldq % 16) != 0 || status == nullptr)
    return cudaErrorNotSupported;
  switch (d / 128) {
    case 1: return launch_lq<1>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 2: return launch_lq<2>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 3: return launch_lq<3>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 4: return launch_lq<4>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 5: return launch_lq<5>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 6: return launch_lq<6>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 8: return launch_lq<8>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 10: return launch_lq<10>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 12: return launch_lq<12>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 16: return launch_lq<16>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    case 20: return launch_lq<20>(x, g, b, eps, rows, d, amax, stats, counter, q, ldq, scale_out, status, s);
    default: return cudaErrorNotSupported;
  }
}

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
      case 1: return launch_pdl(layernorm_kernel<1>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
      case 2: return launch_pdl(layernorm_kernel<2>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
      case 3: return launch_pdl(layernorm_kernel<3>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
      case 4: return launch_pdl(layernorm_kernel<4>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
      case 5: return launch_pdl(layernorm_kernel<5>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
      default: return launch_pdl(layernorm_kernel<8>, dim3(grid), dim3(kLnThreads), 0, s, x, g, b, eps, out, rows, d, amax, q, ldq, row_scales);
    }
  }
  if (q != nullptr || out == nullptr) return cudaErrorInvalidValue;
  const long threads = static_cast<long>(rows) * 32;
  layernorm_wide_kernel<<<static_cast<int>((threads + 255) / 256), 256, 0, s>>>(x, g, b, eps, out, rows, d, amax);
  return cudaGetLastError();
}

}  // namespace esmb200

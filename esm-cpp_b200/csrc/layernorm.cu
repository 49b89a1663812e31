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
        if (c < d) *reinterpret_cast<uint32_t*>(qr + c) = quant_pack4(v[i], inv);
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
// phase 2 recomputes y from x (in L2) and quantises it.  One warp per row,
// lane l holding columns 4 l + 128 i (d = 128 NV).

// Grid-wide barrier for a cooperative launch, used once per launch: `counter`
// is zero before the launch; the wait is bounded like the mbarrier waits.
// Each block's thread 0 publishes the block's writes with a fence before its
// arrival; the acquire load that sees every arrival orders thread 0's later
// reads after them, and the closing block barrier orders the other threads'
// reads after thread 0's acquire, so no second fence is needed.
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
  }
  __syncthreads();
}

// y = fma((x - mean) * inv_std, g, b) on four columns as two f32x2 pairs
// (each lane of a packed instruction rounds as the scalar form does).
__device__ __forceinline__ void ln_y4x2(float4 v, unsigned long long mean2, unsigned long long inv2,
                                        float4 gg, float4 bv, unsigned long long& y01,
                                        unsigned long long& y23) {
  y01 = f2_fma(f2_mul(f2_sub(f2_pack(v.x, v.y), mean2), inv2), f2_pack(gg.x, gg.y), f2_pack(bv.x, bv.y));
  y23 = f2_fma(f2_mul(f2_sub(f2_pack(v.z, v.w), mean2), inv2), f2_pack(gg.z, gg.w), f2_pack(bv.z, bv.w));
}

// 12 warps per block, a row per warp at a time.  Up to d = 2048 (NV <= 16)
// two blocks share an SM (at most 80 registers); d = 2560 (ESM-2 3B, NV = 20)
// holds 80 floats of the row per lane and runs one block per SM.  Warp w of
// block b takes rows w * grid + b, + 12 grid, ...: every block gets a near-
// equal share of the rows, so the SMs finish each phase together.  Each warp
// keeps its last row of phase 1 in registers across the grid barrier; phase 2
// quantises it first and re-reads the others (from L2) most recent first.
constexpr int kLqThreads = 384;
constexpr int kLqWarps = kLqThreads / 32;

template <int NV>
__global__ void __launch_bounds__(kLqThreads, NV <= 16 ? 2 : 1)
    ln_quant_kernel(const float* __restrict__ x, const float* __restrict__ g,
                    const float* __restrict__ b, float eps, int rows, int d, uint32_t* amax,
                    float2* stats, uint32_t* counter, int8_t* __restrict__ q, long ldq,
                    float* scale_out, uint32_t* status) {
  const int lane = threadIdx.x & 31;
  const long warp_g = static_cast<long>(threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  const long nwarps = static_cast<long>(gridDim.x) * kLqWarps;
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
  // the float rounding of var that follows.  Returns (mean, inv_std).
  auto stats_row = [&](const float4 (&v)[NV]) {
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
    const unsigned long long mean2 = f2_pack(meanf, meanf), inv2 = f2_pack(inv_std, inv_std);
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * lane + 128 * i;
      unsigned long long y01, y23;
      ln_y4x2(v[i], mean2, inv2, lds128(sg + c * 4u), lds128(sb + c * 4u), y01, y23);
      float y0, y1, y2, y3;
      f2_unpack(y01, y0, y1);
      f2_unpack(y23, y2, y3);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(y0), fabsf(y1)), fmaxf(fabsf(y2), fabsf(y3))));
    }
    tmax = fmaxf(tmax, mx);
    return make_float2(meanf, inv_std);
  };
  float4 va[NV];  // after the loop: the warp's last row
  float2 st_last = make_float2(0.0f, 0.0f);
  for (long r = warp_g; r < rows; r += nwarps) {
    load_row(r, va);
    st_last = stats_row(va);
    if (lane == 0) stats[r] = st_last;
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
  // q = rne(y * inv) through the float adder (quant_bits), packed f32x2.
  // The upper clamp of quant_bits is left out: y is recomputed here exactly
  // as phase 1 computed it, so |y| <= amax and |y * inv| < 127.5 (the scale
  // and its reciprocal each round by half an ulp).  The lower clamp stays so
  // that a NaN still maps to -127.
  const unsigned long long inv2 = f2_pack(inv, inv), round2 = f2_pack(12582912.0f, 12582912.0f);
  auto quant_row = [&](long r, float2 st, const float4 (&v)[NV]) {
    int8_t* qr = q + r * ldq;
    const unsigned long long mean2 = f2_pack(st.x, st.x), is2 = f2_pack(st.y, st.y);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * lane + 128 * i;
      unsigned long long y01, y23;
      ln_y4x2(v[i], mean2, is2, lds128(sg + c * 4u), lds128(sb + c * 4u), y01, y23);
      float t0, t1, t2, t3;
      f2_unpack(f2_mul(y01, inv2), t0, t1);
      f2_unpack(f2_mul(y23, inv2), t2, t3);
      float u0, u1, u2, u3;
      f2_unpack(f2_add(f2_pack(fmaxf(t0, -127.0f), fmaxf(t1, -127.0f)), round2), u0, u1);
      f2_unpack(f2_add(f2_pack(fmaxf(t2, -127.0f), fmaxf(t3, -127.0f)), round2), u2, u3);
      *reinterpret_cast<uint32_t*>(qr + c) =
          __byte_perm(__byte_perm(__float_as_uint(u0), __float_as_uint(u1), 0x0040),
                      __byte_perm(__float_as_uint(u2), __float_as_uint(u3), 0x0040), 0x5410);
    }
    for (long c = d + lane; c < ldq; c += 32) qr[c] = 0;
  };
  if (warp_g >= rows) return;
  const long r_last = warp_g + (rows - 1 - warp_g) / nwarps * nwarps;
  quant_row(r_last, st_last, va);
  for (long r = r_last - nwarps; r >= warp_g; r -= nwarps) {
    load_row(r, va);
    quant_row(r, __ldcg(stats + r), va);
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
  const long want = (static_cast<long>(rows) + kLqWarps - 1) / kLqWarps;
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

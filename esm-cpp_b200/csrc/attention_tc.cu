// Packed-varlen attention on the tcgen05 tensor cores, FP32-accurate
// (3xTF32), for head_dim 64 and sequences of up to 256 tokens -- every
// ESM-2 650M/150M batch of the reference's workloads.  Longer sequences go
// to the SIMT kernel in attention.cu.
//
// Same contract as the reference's AttentionVarlen (attention.cpp:99-144):
// q pre-scaled and RoPE'd, per-sequence softmax over cu_seqlens, exact
// (not online) softmax -- row max over all keys, exponentials, sum -- then
// out = (sum_j e_j v_j) / sum_j e_j.
//
// One CTA per (sequence, head, 128-query block), 256 threads, 1 CTA/SM:
//   1. Q [128 x 64] and K [L x 64] are loaded, split into tf32 hi/lo parts
//      (hi = top 19 bits, lo = x - hi, exact) and written K-major with the
//      128-byte swizzle.
//   2. One thread issues S = Q_hi K_hi^T + Q_hi K_lo^T + Q_lo K_hi^T
//      (kind::tf32, M=128, N=round16(L), 8 k-steps) into TMEM columns
//      [0, 256); the dropped lo*lo term and lo truncation leave ~2^-21
//      relative error per product, well inside the 1e-4 FP32 class.
//   3. V^T (hi/lo) replaces K in shared memory.  Two warps share each TMEM
//      lane quadrant (query rows); they split the 32-key chunks by parity:
//      row max over the S row, then per pair of chunks p = exp(s - max) ->
//      P chunks (hi/lo) in two buffers -> one thread issues
//      O += P_chunk V^T_chunk (3xTF32, N=64) into TMEM [256, 320).
//   4. O is read back (each warp of a quadrant one 32-column half), scaled
//      by 1/sum and stored; absmax folded for the next GEMM's per-tensor
//      activation scale.
// Barrier waits are bounded and block-uniform (a timeout sets the status
// word and the CTA skips to cleanup).
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int QB = 128;      // queries per CTA
constexpr int DH = 64;       // head dim on this path
constexpr int KMAX = 256;    // longest sequence on this path
constexpr int KC = 32;       // keys per P.V chunk (one swizzle row of tf32)
constexpr int kThreads = 256;  // 8 warps: two per TMEM lane quadrant
constexpr int kBatch = 4;     // independent float4 loads in flight per thread
constexpr uint32_t kRegionA = 0;        // Q hi|lo (32K each) -> P buffers
constexpr uint32_t kRegionB = 65536;    // K hi|lo (64K each) -> V^T hi|lo
constexpr uint32_t kSmemUsed = 196608;
constexpr int kSmemBytes = kSmemUsed + 1024 + 128;

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

__device__ __forceinline__ void split_store4(uint8_t* hi_base, uint8_t* lo_base, uint32_t off,
                                             float4 x) {
  const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
  const float4 l = make_float4(__fsub_rn(x.x, h.x), __fsub_rn(x.y, h.y), __fsub_rn(x.z, h.z),
                               __fsub_rn(x.w, h.w));
  *reinterpret_cast<float4*>(hi_base + off) = h;
  *reinterpret_cast<float4*>(lo_base + off) = l;
}

// Every thread waits (bounded); the result is made block-uniform.
__device__ __forceinline__ bool block_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
  const bool ok = mbar_wait(bar, parity, status);
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const float* __restrict__ q, const float* __restrict__ k,
                        const float* __restrict__ v, const int* __restrict__ cu, int H,
                        float* __restrict__ out, uint32_t* amax, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kSmemUsed);  // [0] S, [1..2] P buffers
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = __ldg(cu + b);
  const int L = __ldg(cu + b + 1) - s0;
  if (L <= 0 || L > KMAX || qb * QB >= L) return;  // CTA-uniform, before any barrier

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = qb * QB;
  const int Lk16 = (L + 15) & ~15;
  const int nchunk = (L + KC - 1) / KC;
  const int Lk32 = nchunk * KC;
  const long rs = static_cast<long>(H) * DH;  // token row stride (floats)
  const float* qg = q + static_cast<long>(s0) * rs + h * DH;
  const float* kg = k + static_cast<long>(s0) * rs + h * DH;
  const float* vg = v + static_cast<long>(s0) * rs + h * DH;
  uint8_t* A = smem + kRegionA;
  uint8_t* Bm = smem + kRegionB;

  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }

  // ---- 1. Q and K, split into tf32 hi/lo, K-major 128-byte swizzle.  One
  // index space (Q float4s, then K float4s); each thread issues kBatch
  // independent loads before it stores any, to keep loads in flight.
  const int nq = QB * 16, nqk = nq + Lk16 * 16;
  for (int base = tid; base < nqk; base += kThreads * kBatch) {
    float4 x[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int e = base + i * kThreads;
      x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < nq) {
        const int r = e >> 4;
        if (q0 + r < L) x[i] = __ldg(reinterpret_cast<const float4*>(qg + (q0 + r) * rs + (e & 15) * 4));
      } else if (e < nqk) {
        const int r = (e - nq) >> 4;
        if (r < L) x[i] = __ldg(reinterpret_cast<const float4*>(kg + r * rs + (e & 15) * 4));
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int e = base + i * kThreads;
      if (e < nq) split_store4(A, A + 32768, sw128_off4(e >> 4, (e & 15) * 4, QB), x[i]);
      else if (e < nqk) split_store4(Bm, Bm + 65536, sw128_off4((e - nq) >> 4, (e & 15) * 4, Lk16), x[i]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tS = tmem, tO = tmem + 256;

  // ---- 2. S = Q K^T (3xTF32)
  if (tid == 0) {
    const uint32_t idS = idesc_tf32(QB, Lk16);
    const uint32_t a_hi = smem_u32(A), a_lo = a_hi + 32768;
    const uint32_t b_hi = smem_u32(Bm), b_lo = b_hi + 65536;
#pragma unroll
    for (int kk = 0; kk < DH / 8; ++kk) {
      const uint32_t ao = (kk >> 2) * (QB * 128) + (kk & 3) * 32;
      const uint32_t bo = static_cast<uint32_t>((kk >> 2) * (Lk16 * 128) + (kk & 3) * 32);
      mma_tf32(tS, sw128_kmajor_desc(a_hi + ao), sw128_kmajor_desc(b_hi + bo), idS, kk > 0 ? 1u : 0u);
      mma_tf32(tS, sw128_kmajor_desc(a_hi + ao), sw128_kmajor_desc(b_lo + bo), idS, 1u);
      mma_tf32(tS, sw128_kmajor_desc(a_lo + ao), sw128_kmajor_desc(b_hi + bo), idS, 1u);
    }
    mma_commit(&bar[0]);
  }
  // V^T element e -> key j, dh group c4: a warp covers 32 consecutive keys of
  // one 4-wide dh group (conflict-free transposed stores).
  const int nv = Lk32 * 16;
  auto v_load = [&](int e) {
    const int j = (e & 31) + ((e >> 9) << 5), c4 = (e >> 5) & 15;
    return (e < nv && j < L) ? __ldg(reinterpret_cast<const float4*>(vg + j * rs + c4 * 4))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  auto v_store = [&](int e, float4 x) {
    if (e >= nv) return;
    const int j = (e & 31) + ((e >> 9) << 5), c4 = (e >> 5) & 15;
    const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t off = sw128_off4(c4 * 4 + i, j, DH);
      const float hv = tf32_hi(xs[i]);
      *reinterpret_cast<float*>(Bm + off) = hv;
      *reinterpret_cast<float*>(Bm + 65536 + off) = __fsub_rn(xs[i], hv);
    }
  };
  // The first V batch is fetched while the S MMAs run (K's region is only
  // overwritten after they complete).
  float4 vx[kBatch];
#pragma unroll
  for (int i = 0; i < kBatch; ++i) vx[i] = v_load(tid + i * kThreads);

  bool ok = block_wait(&bar[0], 0, status);
  tc_fence_after();

  // Warp w reads TMEM lane quadrant (w % 4) = query rows 32*(w%4)..+31 and
  // handles the 32-key chunks of parity par = w / 4 (even chunks go to P
  // buffer 0, odd chunks to buffer 1, both filled in the same iteration).
  __shared__ float red_max[2][QB], red_sum[2][QB];
  const int qd = warp & 3, par = warp >> 2;
  const int row = qd * 32 + lane;  // query row in the block = TMEM lane
  const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
  const int npairs = (nchunk + 1) >> 1;
  float total = 0.0f;
  if (ok) {
    // ---- 3a. V^T (hi/lo) over the consumed K region; keys >= L are zero.
    for (int base = tid;; base += kThreads * kBatch) {
#pragma unroll
      for (int i = 0; i < kBatch; ++i) v_store(base + i * kThreads, vx[i]);
      const int next = base + kThreads * kBatch;
      if (next >= nv) break;
#pragma unroll
      for (int i = 0; i < kBatch; ++i) vx[i] = v_load(next + i * kThreads);
    }
    // ---- 3b. row max over the valid keys (each warp over its parity)
    float mx = -INFINITY;
    for (int c = par; c < nchunk; c += 2) {
      uint32_t r32[32];
      tmem_ld32(tS + lane_off + c * 32, r32);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c * 32 + j < L) mx = fmaxf(mx, __uint_as_float(r32[j]));
    }
    red_max[par][row] = mx;
    __syncthreads();
    mx = fmaxf(red_max[0][row], red_max[1][row]);
    const float kLog2e = 1.4426950408889634f;
    float sum = 0.0f;
    // ---- 3c. P chunk pairs and O += P V^T
    for (int it = 0; it < npairs; ++it) {
      if (it > 0) {  // the MMAs of the previous pair released both buffers
        const bool a = mbar_wait(&bar[1], (it - 1) & 1, status);
        const bool b = (2 * (it - 1) + 1 >= nchunk) || mbar_wait(&bar[2], (it - 1) & 1, status);
        if (__syncthreads_and(a && b ? 1 : 0) == 0) {
          ok = false;
          break;
        }
      }
      const int c = 2 * it + par;
      if (c < nchunk) {  // warp-uniform
        uint32_t r32[32];
        tmem_ld32(tS + lane_off + c * 32, r32);
        tmem_ld_wait();
        uint8_t* P = A + par * 32768;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          float p4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = j4 * 4 + i;
            const float sv = __uint_as_float(r32[j]);
            p4[i] = (c * 32 + j < L) ? exp2f(__fmul_rn(__fsub_rn(sv, mx), kLog2e)) : 0.0f;
            sum = __fadd_rn(sum, p4[i]);
          }
          split_store4(P, P + 16384, sw128_off4(row, j4 * 4, QB), make_float4(p4[0], p4[1], p4[2], p4[3]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == 0) {
        const uint32_t idO = idesc_tf32(QB, DH);
        for (int pc = 0; pc < 2 && 2 * it + pc < nchunk; ++pc) {
          const int cc = 2 * it + pc;
          const uint32_t p_hi = smem_u32(A) + pc * 32768, p_lo = p_hi + 16384;
          const uint32_t v_hi = smem_u32(Bm) + static_cast<uint32_t>(cc * DH * 128), v_lo = v_hi + 65536;
#pragma unroll
          for (int kk = 0; kk < KC / 8; ++kk) {
            const uint32_t o = kk * 32;
            mma_tf32(tO, sw128_kmajor_desc(p_hi + o), sw128_kmajor_desc(v_hi + o), idO,
                     (cc | kk) != 0 ? 1u : 0u);
            mma_tf32(tO, sw128_kmajor_desc(p_hi + o), sw128_kmajor_desc(v_lo + o), idO, 1u);
            mma_tf32(tO, sw128_kmajor_desc(p_lo + o), sw128_kmajor_desc(v_hi + o), idO, 1u);
          }
          mma_commit(&bar[1 + pc]);
        }
      }
    }
    if (ok) {  // the last pair's MMAs (and so all of them) are done
      const int it = npairs - 1;
      const bool a = mbar_wait(&bar[1], it & 1, status);
      const bool b = (2 * it + 1 >= nchunk) || mbar_wait(&bar[2], it & 1, status);
      ok = __syncthreads_and(a && b ? 1 : 0) != 0;
    }
    red_sum[par][row] = sum;
    __syncthreads();
    total = __fadd_rn(red_sum[0][row], red_sum[1][row]);
  }

  float mx_out = 0.0f;
  if (ok) {
    // ---- 4. O / sum -> out; warp parity picks the 32-column half of O.
    tc_fence_after();
    uint32_t o[32];
    tmem_ld32(tO + lane_off + par * 32, o);
    tmem_ld_wait();
    if (q0 + row < L) {
      const float inv = __fdiv_rn(1.0f, total);
      float* op = out + (static_cast<long>(s0) + q0 + row) * rs + h * DH + par * 32;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 a = make_float4(__fmul_rn(__uint_as_float(o[j]), inv), __fmul_rn(__uint_as_float(o[j + 1]), inv),
                                     __fmul_rn(__uint_as_float(o[j + 2]), inv), __fmul_rn(__uint_as_float(o[j + 3]), inv));
        *reinterpret_cast<float4*>(op + j) = a;
        mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
      }
    }
    if (amax != nullptr) amax_publish(amax, mx_out);  // ok is block-uniform
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// Launches the tensor-core kernel for every sequence of length <= 256 (max
// 2 query blocks); longer sequences are skipped here.
cudaError_t launch_attention_tc(const float* q, const float* k, const float* v, const int* cu,
                                int B, int H, int max_len, float* out, uint32_t* amax,
                                uint32_t* status, cudaStream_t s) {
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const int qblocks = (std::min(max_len, KMAX) + QB - 1) / QB;
  if (qblocks <= 0) return cudaSuccess;
  dim3 grid(qblocks, H, B);
  attention_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(q, k, v, cu, H, out, amax, status);
  return cudaGetLastError();
}

}  // namespace esmb200

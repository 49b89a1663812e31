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
// Persistent: one CTA per SM strides over the work items (128-query block,
// sequence, head), query-block-major.  Eight softmax warps load, split and
// normalise; a ninth warp issues every MMA.  Per item:
//   1. Q [128 x 64] and K [L x 64] are split into tf32 hi/lo parts (hi = top
//      19 bits, lo = x - hi, exact) and written K-major with the 128-byte
//      swizzle.  Q and the first 128 K rows were loaded into registers
//      while the previous item was still in its softmax (cross-item
//      prefetch), so an item's HBM latency overlaps the math of the one
//      before; V is loaded while S is computed.
//   2. The issuer computes S = Q_hi K_hi^T + Q_hi K_lo^T + Q_lo K_hi^T
//      (kind::tf32, M=128, N=round16(L), 8 k-steps) into TMEM columns
//      [0, 256); the dropped lo*lo term and lo truncation leave ~2^-21
//      relative error per product, well inside the 1e-4 FP32 class.
//   3. V^T (hi/lo) replaces K in shared memory.  Two warps share each TMEM
//      lane quadrant (query rows) and split the 32-key chunks by parity: row
//      max over the S row, then per chunk p = exp(s - max), split into
//      P_hi (written over the chunk's S columns) and P_lo (one of six spare
//      32-column TMEM slots).  As each chunk lands, the issuer adds
//      P_chunk V^T_chunk (3xTF32, A operand from TMEM, N=64) into O at TMEM
//      [256, 320), so the softmax of chunk c+2 runs under the MMAs of c.
//   4. O is read back (each warp of a quadrant one 32-column half), scaled
//      by 1/sum and stored; absmax folded for the next GEMM's per-tensor
//      activation scale (published once per CTA).
// Barrier waits are bounded; a timeout sets the status word, the remaining
// waits of the item are skipped, and the next item-start vote (all warps)
// ends the loop everywhere.
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int QB = 128;      // queries per item
constexpr int DH = 64;       // head dim on this path
constexpr int KMAX = 256;    // longest sequence on this path
constexpr int KC = 32;       // keys per P.V chunk (one swizzle row of tf32)
constexpr int kSoftWarps = 8;  // two per TMEM lane quadrant
constexpr int kSoftThreads = kSoftWarps * 32;
constexpr int kThreads = kSoftThreads + 32;  // + the MMA-issue warp
constexpr uint32_t kRegionA = 0;        // Q hi|lo (32K each)
constexpr uint32_t kRegionB = 65536;    // K hi|lo (64K each) -> V^T hi|lo
constexpr uint32_t kSmemUsed = 196608;
constexpr int kSmemBytes = kSmemUsed + 1024 + 128;
// TMEM columns (512 allocated): S and then P_hi in place, O, P_lo slots.
constexpr uint32_t kColS = 0, kColO = 256, kColLo = 320;
constexpr int kLoSlots = 6;  // chunks 6, 7 reuse the slots of chunks 0, 1

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

// Named barrier 1 over the softmax warps only.
__device__ __forceinline__ void soft_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kSoftThreads) : "memory");
}

// One work item: query block qb of sequence b (tokens [s0, s0+L)), head h.
struct Item {
  int h, qb, s0, L;
};

// Items are numbered query-block-major, then sequence, then head, so the
// second query blocks (only sequences longer than 128) come last.  Returns
// whether item `it` has work on this path.
__device__ __forceinline__ bool decode_item(int it, int B, int H, int min_len,
                                            const int* __restrict__ cu, Item& w) {
  const int per_qb = B * H;
  const int qb = it / per_qb;
  const int rem = it - qb * per_qb;
  const int b = rem / H;
  w.h = rem - b * H;
  w.qb = qb;
  w.s0 = __ldg(cu + b);
  w.L = __ldg(cu + b + 1) - w.s0;
  return w.L >= min_len && w.L > 0 && w.L <= KMAX && qb * QB < w.L;
}

// First item with work at or after `it` in steps of `stride` (n_items if none).
__device__ __forceinline__ int next_item(int it, int stride, int n_items, int B, int H,
                                         int min_len, const int* __restrict__ cu, Item& w) {
  for (; it < n_items; it += stride)
    if (decode_item(it, B, H, min_len, cu, w)) return it;
  return n_items;
}

// 168 registers: nine warps put three on one SM sub-partition (16K
// registers each); the prefetch buffer (64 registers) stays live through the
// softmax.
__global__ void __maxnreg__(168)
    attention_tc_kernel(const float* __restrict__ q, const float* __restrict__ k,
                        const float* __restrict__ v, const int* __restrict__ cu, int B, int H,
                        int min_len, int n_items, float* __restrict__ out, uint32_t* amax,
                        uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // [0] S done, [1 + c] P chunk c written (4 warp arrivals, once per item),
  // [9] P_lo slots of chunks 0-1 free, [10] O done
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kSmemUsed);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 12);
  __shared__ float red_max[2][QB], red_sum[2][QB];

  const int stride = gridDim.x;
  Item cur;
  int it = next_item(blockIdx.x, stride, n_items, B, H, min_len, cu, cur);
  if (it >= n_items) return;  // CTA-uniform, before any barrier

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long rs = static_cast<long>(H) * DH;  // token row stride (floats)
  uint8_t* A = smem + kRegionA;
  uint8_t* Bm = smem + kRegionB;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    for (int c = 0; c < KMAX / KC; ++c) mbar_init(&bar[1 + c], 4);
    mbar_init(&bar[9], 1);
    mbar_init(&bar[10], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }

  bool ok = true;
  float mx_out = 0.0f;

  if (warp < kSoftWarps) {
    // ======================= softmax / load warps =======================
    // Loader mapping of a 128-row block: row (tid >> 4) + 16 i, 4 floats at col4.
    const int lrow = tid >> 4, col4 = (tid & 15) * 4;
    const int qd = warp & 3, par = warp >> 2;
    const int row = qd * 32 + lane;  // query row in the block = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    uint32_t nS = 0, nLo = 0, nO = 0;  // completions consumed on bar[0], [9], [10]

    // V^T element e -> key j, dh group c4: a warp covers 32 consecutive keys
    // of one 4-wide dh group (conflict-free transposed stores).
    auto v_key = [](int e) { return (e & 31) + ((e >> 9) << 5); };
    auto v_c4 = [](int e) { return (e >> 5) & 15; };
    // Row-major staging in region A (free once S is done) for V on its way
    // in and O on its way out: 256-byte rows, 16-byte group c4 of row j at
    // slot c4 ^ (j & 15), conflict-free both for a warp covering two whole
    // rows and for one covering 32 rows at one c4.
    auto stage_off = [](int j, int c4) {
      return static_cast<uint32_t>(j * 256 + ((c4 ^ (j & 15)) << 4));
    };
    // Q block and the first 128 K rows of item w.
    auto prefetch = [&](const Item& w, float4 (&x)[16]) {
      const long base = static_cast<long>(w.s0) * rs + w.h * DH;
      const int q0 = w.qb * QB;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = lrow + (i & 7) * 16;
        x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < 8) {
          if (q0 + r < w.L) x[i] = __ldg(reinterpret_cast<const float4*>(q + base + (q0 + r) * rs + col4));
        } else if (r < w.L) {
          x[i] = __ldg(reinterpret_cast<const float4*>(k + base + r * rs + col4));
        }
      }
    };
    auto vt_store = [&](int e, float4 xv) {
      const int j = v_key(e), c4 = v_c4(e);
      const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t off = sw128_off4(c4 * 4 + u, j, DH);
        const float hv = tf32_hi(xs[u]);
        *reinterpret_cast<float*>(Bm + off) = hv;
        *reinterpret_cast<float*>(Bm + 65536 + off) = __fsub_rn(xs[u], hv);
      }
    };

    float4 x[16];
    prefetch(cur, x);
    while (true) {
      const int L = cur.L, q0 = cur.qb * QB;
      const int Lk16 = (L + 15) & ~15;
      const int nchunk = (L + KC - 1) / KC;
      const int Lk32 = nchunk * KC;
      const long base = static_cast<long>(cur.s0) * rs + cur.h * DH;

      // ---- 1. Q / K split (prefetched rows), then K rows [128, Lk16).
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = lrow + (i & 7) * 16;
        if (i < 8) split_store4(A, A + 32768, sw128_off4(r, col4, QB), x[i]);
        else if (r < Lk16) split_store4(Bm, Bm + 65536, sw128_off4(r, col4, Lk16), x[i]);
      }
      if (Lk16 > 128) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 128 + lrow + i * 16;
          x[i] = r < L ? __ldg(reinterpret_cast<const float4*>(k + base + r * rs + col4))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 128 + lrow + i * 16;
          if (r < Lk16) split_store4(Bm, Bm + 65536, sw128_off4(r, col4, Lk16), x[i]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (__syncthreads_and(ok ? 1 : 0) == 0) {  // item start: all warps vote
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tmem = *tslot;

      // V rows [0, Lk32) while S runs, row-coalesced (16 threads per row).
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = lrow + i * 16;
        x[i] = r < L ? __ldg(reinterpret_cast<const float4*>(v + base + r * rs + col4))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (ok) ok = mbar_wait(&bar[0], nS & 1, status);
      ++nS;
      tc_fence_after();

      // ---- 3a. V -> staging (region A, Q consumed) -> V^T (hi/lo) over the
      // consumed K region; keys >= L are zero.
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int r = lrow + i * 16;
        if (r < Lk32) *reinterpret_cast<float4*>(A + stage_off(r, col4 >> 2)) = x[i];
      }
      soft_sync();
      const int nv = Lk32 * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = tid + i * kSoftThreads;
        if (e < nv) vt_store(e, *reinterpret_cast<const float4*>(A + stage_off(v_key(e), v_c4(e))));
      }
      fence_proxy_async_smem();
      // Next item's loads fly during this item's softmax and P.V.
      Item nxt;
      const int it_next = next_item(it + stride, stride, n_items, B, H, min_len, cu, nxt);
      if (it_next < n_items) prefetch(nxt, x);

      // ---- 3b. row max over the valid keys (each warp over its parity)
      float mx = -INFINITY;
      for (int c = par; c < nchunk; c += 2) {
        uint32_t r32[32];
        tmem_ld32(tmem + kColS + lane_off + c * 32, r32);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c * 32 + j < L) mx = fmaxf(mx, __uint_as_float(r32[j]));
      }
      red_max[par][row] = mx;
      soft_sync();  // also: every V^T store precedes every chunk-ready arrive
      mx = fmaxf(red_max[0][row], red_max[1][row]);

      // ---- 3c. P chunks into TMEM; each chunk's arrive lets the issuer add
      // P_chunk V^T_chunk into O.
      const float kLog2e = 1.4426950408889634f;
      float sum = 0.0f;
      for (int c = par; c < nchunk; c += 2) {
        if (c == kLoSlots || c == kLoSlots + 1) {  // slot reuse: chunks 0, 1 consumed
          if (ok) ok = mbar_wait(&bar[9], nLo & 1, status);
          tc_fence_after();
        }
        uint32_t hi[32];
        tmem_ld32(tmem + kColS + lane_off + c * 32, hi);
        tmem_ld_wait();
        const int slot = c < kLoSlots ? c : c - kLoSlots;
#pragma unroll
        for (int h16 = 0; h16 < 2; ++h16) {  // P_lo in two 16-column halves
          uint32_t lo[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = h16 * 16 + jj;
            const float sv = __uint_as_float(hi[j]);
            const float pv = (c * 32 + j < L) ? exp2f(__fmul_rn(__fsub_rn(sv, mx), kLog2e)) : 0.0f;
            sum = __fadd_rn(sum, pv);
            const float ph = tf32_hi(pv);
            hi[j] = __float_as_uint(ph);
            lo[jj] = __float_as_uint(__fsub_rn(pv, ph));
          }
          tmem_st16(tmem + kColLo + lane_off + slot * 32 + h16 * 16, lo);
        }
        tmem_st32(tmem + kColS + lane_off + c * 32, hi);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[1 + c]);
      }
      if (nchunk > kLoSlots) ++nLo;  // the phase completes for every thread
      red_sum[par][row] = sum;
      soft_sync();
      const float total = __fadd_rn(red_sum[0][row], red_sum[1][row]);

      // ---- 4. O / sum -> out; warp parity picks the 32-column half of O.
      if (ok) ok = mbar_wait(&bar[10], nO & 1, status);
      ++nO;
      tc_fence_after();
      uint32_t o[32];
      tmem_ld32(tmem + kColO + lane_off + par * 32, o);
      tmem_ld_wait();
      {  // O / sum -> staging (region A) -> row-coalesced stores
        const float inv = __fdiv_rn(1.0f, total);
        const bool live = q0 + row < L;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 a = make_float4(__fmul_rn(__uint_as_float(o[j]), inv), __fmul_rn(__uint_as_float(o[j + 1]), inv),
                                       __fmul_rn(__uint_as_float(o[j + 2]), inv), __fmul_rn(__uint_as_float(o[j + 3]), inv));
          *reinterpret_cast<float4*>(A + stage_off(row, par * 8 + (j >> 2))) = a;
          if (live)
            mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
        }
        soft_sync();
        if (ok) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = lrow + i * 16;
            if (q0 + r < L)
              *reinterpret_cast<float4*>(out + base + static_cast<long>(q0 + r) * rs + col4) =
                  *reinterpret_cast<const float4*>(A + stage_off(r, col4 >> 2));
          }
        }
        soft_sync();  // staging read out before the next item's Q lands in A
      }
      if (it_next >= n_items) break;
      it = it_next;
      cur = nxt;
    }
  } else {
    // ============================ MMA issuer ============================
    uint32_t cpar = 0;  // bit c: parity of the next completion of bar[1 + c]
    while (true) {
      if (__syncthreads_and(ok ? 1 : 0) == 0) {  // item start: Q / K in shared memory
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tmem = *tslot;
      const int L = cur.L;
      const int Lk16 = (L + 15) & ~15;
      const int nchunk = (L + KC - 1) / KC;
      if (lane == 0) {
        // ---- 2. S = Q K^T (3xTF32)
        const uint32_t idS = idesc_tf32(QB, Lk16);
        const uint32_t a_hi = smem_u32(A), a_lo = a_hi + 32768;
        const uint32_t b_hi = smem_u32(Bm), b_lo = b_hi + 65536;
#pragma unroll
        for (int kk = 0; kk < DH / 8; ++kk) {
          const uint32_t ao = (kk >> 2) * (QB * 128) + (kk & 3) * 32;
          const uint32_t bo = static_cast<uint32_t>((kk >> 2) * (Lk16 * 128) + (kk & 3) * 32);
          mma_tf32(tmem + kColS, sw128_kmajor_desc(a_hi + ao), sw128_kmajor_desc(b_hi + bo), idS, kk > 0 ? 1u : 0u);
          mma_tf32(tmem + kColS, sw128_kmajor_desc(a_hi + ao), sw128_kmajor_desc(b_lo + bo), idS, 1u);
          mma_tf32(tmem + kColS, sw128_kmajor_desc(a_lo + ao), sw128_kmajor_desc(b_hi + bo), idS, 1u);
        }
        mma_commit(&bar[0]);
        // ---- 3c. O += P_chunk V^T_chunk as the chunks land
        const uint32_t idO = idesc_tf32(QB, DH);
        for (int c = 0; c < nchunk; ++c) {
          if (ok) ok = mbar_wait(&bar[1 + c], (cpar >> c) & 1u, status);
          cpar ^= 1u << c;
          tc_fence_after();
          const uint32_t p_hi = tmem + kColS + c * 32;
          const uint32_t p_lo = tmem + kColLo + (c < kLoSlots ? c : c - kLoSlots) * 32;
          const uint32_t v_hi = smem_u32(Bm) + static_cast<uint32_t>(c * DH * 128), v_lo = v_hi + 65536;
#pragma unroll
          for (int kk = 0; kk < KC / 8; ++kk) {
            const uint32_t o = kk * 32;
            mma_tf32_ts(tmem + kColO, p_hi + kk * 8, sw128_kmajor_desc(v_hi + o), idO,
                        (c | kk) != 0 ? 1u : 0u);
            mma_tf32_ts(tmem + kColO, p_hi + kk * 8, sw128_kmajor_desc(v_lo + o), idO, 1u);
            mma_tf32_ts(tmem + kColO, p_lo + kk * 8, sw128_kmajor_desc(v_hi + o), idO, 1u);
          }
          if (c == 1 && nchunk > kLoSlots) mma_commit(&bar[9]);
        }
        mma_commit(&bar[10]);
      }
      __syncwarp();
      Item nxt;
      const int it_next = next_item(it + stride, stride, n_items, B, H, min_len, cu, nxt);
      if (it_next >= n_items) break;
      it = it_next;
      cur = nxt;
    }
  }

  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (all_ok && amax != nullptr) amax_publish(amax, mx_out);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*tslot, 512);
  }
}

}  // namespace

// Launches the persistent tensor-core kernel (one CTA per SM) over every
// sequence with min_len <= L <= 256 (at most 2 query blocks); other
// sequences are skipped here.
cudaError_t launch_attention_tc(const float* q, const float* k, const float* v, const int* cu,
                                int B, int H, int min_len, int max_len, float* out,
                                uint32_t* amax, uint32_t* status, cudaStream_t s) {
  static std::atomic<uint64_t> attr_set{0};
  static std::atomic<int> sm_count[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sm_count[dev & 63].store(n);
    attr_set.fetch_or(bit);
  }
  const int qblocks = (std::min(max_len, KMAX) + QB - 1) / QB;
  if (qblocks <= 0) return cudaSuccess;
  const long n_items = static_cast<long>(qblocks) * B * H;
  if (n_items > (1L << 30)) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long>(n_items, sm_count[dev & 63].load()));
  attention_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(q, k, v, cu, B, H, min_len,
                                                         static_cast<int>(n_items), out, amax,
                                                         status);
  return cudaGetLastError();
}

}  // namespace esmb200

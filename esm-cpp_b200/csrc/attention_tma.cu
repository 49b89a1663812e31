// Packed-varlen attention (head_dim 64) on the tcgen05 tensor cores,
// FP32-accurate (3xTF32), fed by TMA.  Three kernels by sequence length:
//   attention_tma_kernel       L <= 128: one CTA per (sequence, head)
//   attention_tma_pair_kernel  129..256: one CTA pair (cta_group::2) per
//                              (sequence, head)
//   attention_tma_long_kernel  > 256: one CTA per (sequence, head, 128-row
//                              query tile), two passes over 128-key blocks
// With qk_bf16 (the reference's opt-in BF16 attention) Q and K already hold
// bf16 values, which tf32 represents exactly: S needs no lo terms.  The
// description below is the single-CTA kernel's; the other two follow it and
// say where they differ.
//
// Same contract as the reference's AttentionVarlen (attention.cpp:99-144):
// q pre-scaled and RoPE'd, per-sequence softmax over cu_seqlens, exact
// (not online) softmax -- row max over all keys, exponentials, sum -- then
// out = (sum_j e_j v_j) / sum_j e_j.
//
// 3xTF32 without a hi copy: the tensor core reads an fp32 operand as tf32 by
// dropping its low 13 bits, so the raw fp32 word is the hi part and only
// lo = x - hi is formed (in shared memory for K and V, in TMEM for Q).
//   S = Q K^T  = Q_raw K_raw^T + Q_raw K_lo^T + Q_lo K_raw^T
//   O = P V    = P_hi V_raw + P_hi V_lo + P_lo V_raw
// V is used in its natural [key][dh] layout as an MN-major B operand (TMA
// writes it in the 128-byte swizzle with 32-byte atoms, the MN-major layout
// kind::tf32 accepts).
//
// Persistent, one CTA per SM, items = (sequence, head) with L <= 128,
// double-buffered: while item n is in its softmax, item n+1's Q and K land
// in the other 96 KB slot, are split, and its S is computed.
//   warp 0      TMA producer (Q, K into the slot; V into a prefetch buffer)
//   warp 1      TMEM owner + MMA issuer (S into one of two TMEM buffers,
//               then O += P_chunk V_chunk as the softmax finishes chunks)
//   warps 2-5   prep, one per TMEM lane quadrant: K_lo, Q_lo (TMEM), then V
//               and V_lo into the slot once S has consumed K (rows >= L
//               zeroed)
//   warps 6-13  softmax (two per lane quadrant, 32-key chunks by parity) and
//               the epilogue (O / sum staged in the slot, stored in rows)
// TMEM (CTA-pair kernel): S [0,256) O [256,320) P_lo [320,448) Q_lo [448,512);
// the single-CTA kernel's layout is next to its shared-memory constants.
// Every mbarrier is used at most once per item (or per use of its slot), so
// no parity wait can alias a later phase.  Waits are bounded; a timeout (or
// another waiter's) ends all roles' loops.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int QB = 128;    // query rows per item (all of a short sequence)
constexpr int DH = 64;     // head dim on this path
constexpr int KC = 32;     // keys per P.V chunk
constexpr int LMAX = 128;  // longest sequence on this path
constexpr int kThreads = 448;
constexpr int kPrepWarp0 = 2, kSoftWarp0 = 6;
constexpr uint32_t kSlotBytes = 98304;  // Q raw | K or V raw | K or V lo, 32 KB each
constexpr uint32_t kOffQ = 0, kOffKV = 32768, kOffLo = 65536;
// Both kernels: a 32 KB V prefetch buffer after the two slots, then the
// barriers.  Single-CTA TMEM: S [0,128), O [128,256) as two halves (P_hi V +
// P_lo V, P_hi V_lo; summed by the epilogue), four P_lo slots [256,384), Q_lo
// [384,448).
constexpr uint32_t kSVpre = 2 * kSlotBytes, kSBarOff = kSVpre + 32768;
constexpr int kSSmemBytes = static_cast<int>(kSBarOff) + 256 + 1024;
constexpr uint32_t kSColO = 128, kSColPlo = 256, kSColQlo = 384;
constexpr uint32_t kColO = 256, kColPlo = 384, kColQlo = 448;  // CTA-pair and long kernels
// CTA-pair kernel: the V buffer first (it is the raw V operand, and V_lo in
// a slot's third region sits one positive LBO above it), the two slots, a
// 1 KB zero block (the B operand's second half in P_lo [V | 0]), barriers.
constexpr uint32_t kPVbuf = 0, kPSlot0 = 32768;
constexpr uint32_t kPZero = kPSlot0 + 2 * kSlotBytes, kPBarOff = kPZero + 1024;
constexpr int kPSmemBytes = static_cast<int>(kPBarOff) + 256 + 1024;

enum : int {
  kFullQK = 0,     // [2] TMA Q + K landed in slot s
  kFullV = 2,      // [2] TMA V landed
  kQKReady = 4,    // [2] K_lo and Q_lo written (4 prep warps)
  kVReady = 6,     // [2] V_lo written (4 prep warps)
  kSDone = 8,      // [2] S MMAs of the slot's item done
  kODone = 10,     // [2] P.V MMAs done (by item parity)
  kSlotFree = 12,  // [2] epilogue done with the slot (8 softmax warps)
  kChunk = 14,     // [4] P chunk c written (4 softmax warps)
  kFullVpre = 18,  // TMA V landed in the prefetch buffer (once per item)
  kVpreFree = 19,  // prep has copied it into the slot (4 prep warps)
  kNumBars = 20
};

struct Item {
  int h, s0, L;
};

__device__ __forceinline__ bool decode_item(int it, int H, const int* __restrict__ cu, Item& w) {
  const int b = it / H;
  w.h = it - b * H;
  w.s0 = __ldg(cu + b);
  w.L = __ldg(cu + b + 1) - w.s0;
  return w.L > 0 && w.L <= LMAX;
}

__device__ __forceinline__ int next_item(int it, int stride, int n_items, int H,
                                         const int* __restrict__ cu, Item& w) {
  for (; it < n_items; it += stride)
    if (decode_item(it, H, cu, w)) return it;
  return n_items;
}

__device__ __forceinline__ float tf32_lo(float x) {
  return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
}
__device__ __forceinline__ float4 tf32_lo4(float4 x) {
  return make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
}

// lo = x - tf32(x) over a 32 KB tile, 128 threads, 16 bytes per thread per
// 2 KB step, eight loads in flight.
__device__ __forceinline__ void tile_lo_32k(uint32_t src, uint32_t dst, int ptid) {
  src += static_cast<uint32_t>(ptid) * 16u;
  dst += static_cast<uint32_t>(ptid) * 16u;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float4 x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = lds128(src + (h * 8 + i) * 2048u);
#pragma unroll
    for (int i = 0; i < 8; ++i) sts128(dst + (h * 8 + i) * 2048u, tf32_lo4(x[i]));
  }
}

// Named barrier 2 over the softmax warps, with an AND-vote.
__device__ __forceinline__ bool soft_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "barrier.cta.red.and.pred po, 2, 256, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void soft_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

// Row-major staging of O in a slot: 256-byte rows, 16-byte group c4 of row j
// at slot c4 ^ (j & 15) (conflict-free for row-per-thread writes and for
// two-rows-per-warp reads).
__device__ __forceinline__ uint32_t stage_off(int j, int c4) {
  return static_cast<uint32_t>(j * 256 + ((c4 ^ (j & 15)) << 4));
}

// Row max over the valid keys of one softmax warp's chunks (c = par, par+2,
// ...; 32 keys each, S chunk c at TMEM column tS + 32 c).
__device__ __forceinline__ float s_row_max(uint32_t tS, int par, int nchunk, int L) {
  float m0 = -INFINITY, m1 = -INFINITY;  // two chains (max is order-free)
  for (int c = par; c < nchunk; c += 2) {
    uint32_t r[32];
    tmem_ld32(tS + 32u * c, r);
    tmem_ld_wait();
    if (c * 32 + 32 <= L) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        m0 = fmaxf(m0, __uint_as_float(r[j]));
        m1 = fmaxf(m1, __uint_as_float(r[j + 1]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c * 32 + j < L) m0 = fmaxf(m0, __uint_as_float(r[j]));
    }
  }
  return fmaxf(m0, m1);
}

// One softmax warp's P chunks (c = par, par+2, ...): P = 2^((S - mx) log2 e)
// over the valid keys (0 past L), P_hi = P with its low 13 bits cleared
// written over S, P_lo = P - P_hi into P_lo slot c & slot_mask (32 columns),
// then arrive(c).  Returns this warp's row sum of P.  wait_lo(c) runs once P
// is computed and P_hi stored, before chunk c's P_lo slot is written, so the
// conversion overlaps the MMAs still reading that slot.  The exponential is
// taken for every key
// and masked afterwards: a select, where a guarded exponential would branch.
template <class WaitLo, class Arrive>
__device__ __forceinline__ float p_chunks(uint32_t tS, uint32_t tPlo, uint32_t slot_mask, int par,
                                          int nchunk, int L, float mx, WaitLo&& wait_lo,
                                          Arrive&& arrive) {
  const float kLog2e = 1.4426950408889634f;
  // Two keys per packed f32x2 instruction (each rounded as its scalar form);
  // the row sum is kept as two interleaved partial sums.
  const unsigned long long mx2 = f2_pack(mx, mx), l2e2 = f2_pack(kLog2e, kLog2e);
  unsigned long long sum2 = f2_pack(0.0f, 0.0f);
  for (int c = par; c < nchunk; c += 2) {
    uint32_t hi[32], lo[32];
    tmem_ld32(tS + 32u * c, hi);
    tmem_ld_wait();
    const int nvalid = L - c * 32;  // keys j < nvalid are valid
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float t0, t1;
      f2_unpack(f2_mul(f2_sub(f2_pack(__uint_as_float(hi[j]), __uint_as_float(hi[j + 1])), mx2), l2e2),
                t0, t1);
      float p0 = ex2_ftz(t0), p1 = ex2_ftz(t1);  // masked after, not guarded
      p0 = j < nvalid ? p0 : 0.0f;
      p1 = j + 1 < nvalid ? p1 : 0.0f;
      const unsigned long long pv = f2_pack(p0, p1);
      sum2 = f2_add(sum2, pv);
      const float h0 = __uint_as_float(__float_as_uint(p0) & 0xFFFFE000u);
      const float h1 = __uint_as_float(__float_as_uint(p1) & 0xFFFFE000u);
      hi[j] = __float_as_uint(h0);
      hi[j + 1] = __float_as_uint(h1);
      float l0, l1;
      f2_unpack(f2_sub(pv, f2_pack(h0, h1)), l0, l1);
      lo[j] = __float_as_uint(l0);
      lo[j + 1] = __float_as_uint(l1);
    }
    tmem_st32(tS + 32u * c, hi);  // S chunk c is this warp's alone once read
    wait_lo(c);
    tmem_st32(tPlo + 32u * (c & slot_mask), lo);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    arrive(c);
  }
  float s0, s1;
  f2_unpack(sum2, s0, s1);
  return __fadd_rn(s0, s1);
}

__global__ void __maxnreg__(128)
    attention_tma_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const int* __restrict__ cu,
                         int H, int n_items, float* __restrict__ out, uint32_t* amax,
                         uint32_t* status, int qk_bf16) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kSBarOff);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile uint32_t* abort_flag = tslot + 1;
  uint8_t* vpre = smem + kSVpre;
  pdl_wait();  // cu and the inputs come from earlier work of the stream
  pdl_trigger();

  const int stride = gridDim.x;
  Item first;
  const int it0 = next_item(blockIdx.x, stride, n_items, H, cu, first);
  if (it0 >= n_items) return;  // CTA-uniform, before any barrier

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long rs = static_cast<long>(H) * DH;  // token row stride (floats)

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kFullQK + i], 1);
      mbar_init(&bar[kFullV + i], 1);
      mbar_init(&bar[kQKReady + i], 4);
      mbar_init(&bar[kVReady + i], 4);
      mbar_init(&bar[kSDone + i], 1);
      mbar_init(&bar[kODone + i], 1);
      mbar_init(&bar[kSlotFree + i], 8);
    }
    for (int c = 0; c < LMAX / KC; ++c) mbar_init(&bar[kChunk + c], 4);
    mbar_init(&bar[kFullVpre], 1);
    mbar_init(&bar[kVpreFree], 4);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  float mx_out = 0.0f;
  Item cur = first;
  int it = it0;
  int n = 0;  // this CTA's item counter

  if (warp == 0) {
    // ================================================== TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      while (true) {
        const int s = n & 1;
        uint8_t* slot = smem + s * kSlotBytes;
        if (n >= 2 && !(ok = mbar_wait_abort(&bar[kSlotFree + s], ((n >> 1) + 1) & 1, status, abort_flag)))
          break;
        mbar_arrive_expect_tx(&bar[kFullQK + s], 4 * 16384);
        for (int blk = 0; blk < 2; ++blk) {
          tma_load_2d(slot + kOffQ + blk * 16384, &tmQ, &bar[kFullQK + s], cur.h * DH + 32 * blk, cur.s0);
          tma_load_2d(slot + kOffKV + blk * 16384, &tmK, &bar[kFullQK + s], cur.h * DH + 32 * blk, cur.s0);
        }
        // The next item, looked up while this one's wait is pending.
        Item nxt;
        const int itn = next_item(it + stride, stride, n_items, H, cu, nxt);
        // V right behind, into the prefetch buffer once prep has moved item
        // n-1's V out of it.
        if (n >= 1 && !(ok = mbar_wait_abort(&bar[kVpreFree], (n - 1) & 1, status, abort_flag))) break;
        mbar_arrive_expect_tx(&bar[kFullVpre], 2 * 16384);
        for (int blk = 0; blk < 2; ++blk)
          tma_load_2d(vpre + blk * 16384, &tmV, &bar[kFullVpre], cur.h * DH + 32 * blk, cur.s0);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp == 1) {
    // ==================================================== MMA issuer
    if (lane == 0) {
      uint32_t cpar = 0;  // bit c: parity of the next completion of chunk barrier c
      const uint32_t idO = idesc_tf32_bmn(QB, DH);
      const uint32_t idO2 = idesc_tf32_bmn(QB, 2 * DH);
      while (true) {
        const int s = n & 1;
        const uint32_t slot = smem_u32(smem + s * kSlotBytes);
        const int L = cur.L, Lk16 = (L + 15) & ~15, nchunk = (L + KC - 1) / KC;
        if (!(ok = mbar_wait_abort(&bar[kQKReady + s], (n >> 1) & 1, status, abort_flag))) break;
        // The single S buffer still holds item n-1's P_hi, read by the P.V
        // MMAs this thread issued before: tcgen05.mma from one thread execute
        // in issue order, so S(n) is issued without waiting for them to finish
        // (the same reuse of P's TMEM by the next S as in CUTLASS's sm100 FMHA).
        tc_fence_after();
        const uint32_t tS = tmem;
        const uint32_t idS = idesc_tf32(QB, Lk16);
#pragma unroll
        for (int kk = 0; kk < DH / 8; ++kk) {
          const uint32_t o = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
          const uint64_t a_raw = sw128_kmajor_desc(slot + kOffQ + o);
          const uint64_t b_raw = sw128_kmajor_desc(slot + kOffKV + o);
          const uint64_t b_lo = sw128_kmajor_desc(slot + kOffLo + o);
          mma_tf32(tS, a_raw, b_raw, idS, kk > 0 ? 1u : 0u);
          if (!qk_bf16) {  // bf16-valued Q and K are exact in tf32: no lo terms
            mma_tf32(tS, a_raw, b_lo, idS, 1u);
            mma_tf32_ts(tS, tmem + kSColQlo + 8u * kk, b_raw, idS, 1u);
          }
        }
        mma_commit(&bar[kSDone + s]);
        // The next item, looked up while this one's wait is pending.
        Item nxt;
        const int itn = next_item(it + stride, stride, n_items, H, cu, nxt);
        if (!(ok = mbar_wait_abort(&bar[kVReady + s], (n >> 1) & 1, status, abort_flag))) break;
        for (int c = 0; c < nchunk; ++c) {
          if (!(ok = mbar_wait_abort(&bar[kChunk + c], (cpar >> c) & 1u, status, abort_flag))) break;
          cpar ^= 1u << c;
          tc_fence_after();
          // P_hi [V | V_lo] as one N = 128 MMA (V's two 32-column blocks and
          // V_lo's follow one another 16 KB apart, the LBO stride), then
          // P_lo V at N = 64 into the first half.
#pragma unroll
          for (int kk = 0; kk < KC / 8; ++kk) {
            const uint32_t vo = static_cast<uint32_t>(c * 4096 + kk * 1024);
            const uint64_t v_all = sw128b32_mnmajor_desc(slot + kOffKV + vo, 16384);
            const uint32_t p_hi = tS + 32u * c + 8u * kk;
            const uint32_t p_lo = tmem + kSColPlo + 32u * c + 8u * kk;
            mma_tf32_ts(tmem + kSColO, p_hi, v_all, idO2, (c | kk) != 0 ? 1u : 0u);
            mma_tf32_ts(tmem + kSColO, p_lo, v_all, idO, 1u);
          }
        }
        if (!ok) break;
        mma_commit(&bar[kODone + s]);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp < kSoftWarp0) {
    // ================================================== prep warps
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int ptid = (warp - kPrepWarp0) * 32 + lane;  // 0..127
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    while (true) {
      const int s = n & 1;
      uint8_t* slot = smem + s * kSlotBytes;
      const int L = cur.L;
      if (!(ok = mbar_wait_abort(&bar[kFullQK + s], (n >> 1) & 1, status, abort_flag))) break;
      // K_lo over the K tile (both 32-column blocks, all 128 rows).
      tile_lo_32k(smem_u32(slot + kOffKV), smem_u32(slot + kOffLo), ptid);
      // Q_lo of this thread's row into TMEM, once S of item n-1 has read the
      // previous Q_lo.
      if (n >= 1 && !(ok = mbar_wait_abort(&bar[kSDone + ((n - 1) & 1)], ((n - 1) >> 1) & 1, status, abort_flag)))
        break;
      tc_fence_after();
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        uint32_t lo[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 x = lds128(smem_u32(slot + kOffQ + blk * 16384 + row * 128) +
                                  static_cast<uint32_t>((c4 ^ (row & 7)) << 4));
          const float4 l = tf32_lo4(x);
          lo[4 * c4] = __float_as_uint(l.x);
          lo[4 * c4 + 1] = __float_as_uint(l.y);
          lo[4 * c4 + 2] = __float_as_uint(l.z);
          lo[4 * c4 + 3] = __float_as_uint(l.w);
        }
        tmem_st32(tmem + kSColQlo + 32u * blk + lane_off, lo);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kQKReady + s]);
      // The next item, looked up while this one's wait is pending.
      Item nxt;
      const int itn = next_item(it + stride, stride, n_items, H, cu, nxt);
      // V (prefetched) into the slot once S has consumed K, with V_lo;
      // rows (keys) >= L are zeroed in both parts.
      if (!(ok = mbar_wait_abort(&bar[kSDone + s], (n >> 1) & 1, status, abort_flag))) break;
      if (!(ok = mbar_wait_abort(&bar[kFullVpre], n & 1, status, abort_flag))) break;
      {
        const uint32_t src = smem_u32(vpre), kv = smem_u32(slot + kOffKV), lo = smem_u32(slot + kOffLo);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float4 x[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            x[i] = lds128(src + static_cast<uint32_t>((ptid + (h * 8 + i) * 128) * 16));
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t o = static_cast<uint32_t>((ptid + (h * 8 + i) * 128) * 16);
            if (static_cast<int>((o & 16383u) >> 7) >= L) x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            sts128(kv + o, x[i]);
            sts128(lo + o, tf32_lo4(x[i]));
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar[kVReady + s]);
        mbar_arrive(&bar[kVpreFree]);
      }
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
  } else {
    // ================================================ softmax warps
    const int sw = warp - kSoftWarp0;  // 0..7
    const int quad = warp & 3, par = sw >> 2;
    const int row = quad * 32 + lane;  // query row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int stid = sw * 32 + lane;  // 0..255
    const int lrow = stid >> 4, col4 = (stid & 15) * 4;
    while (true) {
      const int s = n & 1;
      uint8_t* slot = smem + s * kSlotBytes;
      // Row max / sum exchange in the slot's Q region (dead once S is done).
      float (*red_max)[QB] = reinterpret_cast<float (*)[QB]>(slot + kOffQ);
      float (*red_sum)[QB] = reinterpret_cast<float (*)[QB]>(slot + kOffQ + 1024);
      const int L = cur.L, nchunk = (L + KC - 1) / KC;
      const bool w0 = ok && mbar_wait_abort(&bar[kSDone + s], (n >> 1) & 1, status, abort_flag);
      tc_fence_after();
      const uint32_t tS = tmem + lane_off;
      // ---- row max over the valid keys (each warp over its parity's chunks)
      float mx = s_row_max(tS, par, nchunk, L);
      red_max[par][row] = mx;
      if (!soft_all(w0)) {
        ok = false;
        break;
      }
      mx = fmaxf(red_max[0][row], red_max[1][row]);
      // ---- P chunks into TMEM (P_hi over S, P_lo into its slot)
      const float sum = p_chunks(
          tS, tmem + kSColPlo + lane_off, 3u, par, nchunk, L, mx, [](int) {},
          [&](int c) {
            if (lane == 0) mbar_arrive(&bar[kChunk + c]);
          });
      red_sum[par][row] = sum;
      // The next item, looked up while this one's wait is pending.
      Item nxt;
      const int itn = next_item(it + stride, stride, n_items, H, cu, nxt);
      soft_sync();
      const float total = __fadd_rn(red_sum[0][row], red_sum[1][row]);
      // ---- O / sum -> staging (the slot's V region, free once P.V is done)
      const bool w1 = ok && mbar_wait_abort(&bar[kODone + s], (n >> 1) & 1, status, abort_flag);
      tc_fence_after();
      uint32_t o[32], ob[32];
      tmem_ld32(tmem + kSColO + lane_off + 32u * par, o);
      tmem_ld32(tmem + kSColO + 64u + lane_off + 32u * par, ob);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j)
        o[j] = __float_as_uint(__fadd_rn(__uint_as_float(o[j]), __uint_as_float(ob[j])));
      {
        const float inv = __fdiv_rn(1.0f, total);
        const bool live = row < L;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 a = make_float4(__fmul_rn(__uint_as_float(o[j]), inv), __fmul_rn(__uint_as_float(o[j + 1]), inv),
                                       __fmul_rn(__uint_as_float(o[j + 2]), inv), __fmul_rn(__uint_as_float(o[j + 3]), inv));
          *reinterpret_cast<float4*>(slot + kOffKV + stage_off(row, par * 8 + (j >> 2))) = a;
          if (live)
            mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
        }
      }
      tc_fence_before();
      if (!soft_all(w1)) {  // also: staging complete
        ok = false;
        break;
      }
      {
        float* ob = out + static_cast<long>(cur.s0) * rs + cur.h * DH + col4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = lrow + i * 16;
          if (r < L)
            *reinterpret_cast<float4*>(ob + static_cast<long>(r) * rs) =
                *reinterpret_cast<const float4*>(slot + kOffKV + stage_off(r, col4 >> 2));
        }
      }
      fence_proxy_async_smem();  // generic writes in the slot precede its next TMA fill
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kSlotFree + s]);
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
  }

  __syncwarp();
  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (all_ok && amax != nullptr) amax_publish(amax, mx_out);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ===================================================================== pairs
// Sequences of 129..256 tokens: one CTA pair (2-CTA cluster) per (sequence,
// head), M = 256 MMAs (tcgen05 cta_group::2) issued by CTA 0.  CTA r owns
// query rows [128 r, 128 r + 128), keys [r N/2, (r+1) N/2) of K
// (N = round16(L)) and dh columns [32 r, 32 r + 32) of V for all keys, so
// each CTA keeps the same 96 KB double-buffered slots as the single-CTA
// kernel.  Prep and softmax warps of both CTAs arrive on CTA 0's ready
// barriers; CTA 0's MMA completions are committed to both CTAs' barriers.
// TMEM (each CTA): S [0,256) O [256,384) P_lo [384,448) Q_lo [448,512);
// chunk c >= 2 reuses P_lo slot c & 1 once chunk c - 2's P.V is done.
// P.V is two N = 128 MMAs per 8 keys, B in each CTA = its 32 dh columns of
// V and one LBO further V_lo (P_hi [V | V_lo]) or a zero block (P_lo [V | 0]):
// pair MMAs of N = 64 run at about 40% of the tensor rate, N = 128 at 66%.
// Each CTA's V lands in a 32 KB buffer while S runs and is the raw V operand
// itself; V_lo goes into the slot once S has consumed K_lo, and the next
// item's V loads once this item's P.V is done.
constexpr int LMAX2 = 256;
enum : int {
  kPFullQK = 0,    // [2] own TMA Q + K landed
  kPFullV = 2,     // own TMA V landed in the V buffer (once per item)
  kPQKReady = 3,   // [2] CTA 0: K_lo + Q_lo of both CTAs (8 prep warps)
  kPVReady = 5,    // [2][2] CTA 0: V_lo of keys [128 h, 128 h + 128), both CTAs (8 prep warps)
  kPSDone = 9,     // S MMAs done (both CTAs, once per item)
  kPODone = 10,    // P.V MMAs done (both CTAs, once per item): V buffer free
  kPLoFree = 11,   // [2] chunk c's P.V done: P_lo slot c & 1 free for c + 2 (both CTAs)
  kPSlotFree = 13, // [2] own epilogue done with the slot (8 softmax warps)
  kPChunk = 15,    // [8] CTA 0: P chunk c written in both CTAs (8 softmax warps)
  kPNumBars = 23
};

__device__ __forceinline__ bool decode_long(int it, int H, const int* __restrict__ cu, Item& w) {
  const int b = it / H;
  w.h = it - b * H;
  w.s0 = __ldg(cu + b);
  w.L = __ldg(cu + b + 1) - w.s0;
  return w.L > LMAX && w.L <= LMAX2;
}
__device__ __forceinline__ int next_long(int it, int stride, int n_items, int H,
                                         const int* __restrict__ cu, Item& w) {
  for (; it < n_items; it += stride)
    if (decode_long(it, H, cu, w)) return it;
  return n_items;
}

__global__ void __maxnreg__(128)
    attention_tma_pair_kernel(const __grid_constant__ CUtensorMap tmQ,
                              const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const int* __restrict__ cu,
                              int H, int n_items, float* __restrict__ out, uint32_t* amax,
                              uint32_t* status, int qk_bf16, int wait_late) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kPBarOff);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + kPNumBars);
  volatile uint32_t* abort_flag = tslot + 1;
  uint8_t* vbuf = smem + kPVbuf;
  // wait_late: the previous kernel is another attention kernel of the same
  // call (disjoint sequences, same inputs), which passed its own wait before
  // this grid could launch -- q, k, v and cu are complete.  Waiting for it at
  // the end instead lets these CTAs fill its tail, and this grid still
  // completes after it, so the next kernel's wait covers both.
  if (!wait_late) pdl_wait();
  pdl_trigger();

  const uint32_t rank = cluster_ctarank();
  const int stride = static_cast<int>(gridDim.x >> 1);
  Item first;
  const int it0 = next_long(static_cast<int>(blockIdx.x >> 1), stride, n_items, H, cu, first);
  if (it0 >= n_items) {  // uniform over the pair, before any barrier
    if (wait_late) pdl_wait();
    return;
  }

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long rs = static_cast<long>(H) * DH;
  // CTA 0's copy of a barrier (cluster address) for arrivals from either CTA.
  auto leader = [&](int i) { return mapa_shared(smem_u32(&bar[i]), 0); };
  auto arrive_leader = [&](int i) {
    if (rank == 0) mbar_arrive(&bar[i]);
    else mbar_arrive_cluster(leader(i));
  };

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kPFullQK + i], 1);
      mbar_init(&bar[kPQKReady + i], 8);
      mbar_init(&bar[kPVReady + 2 * i], 8);
      mbar_init(&bar[kPVReady + 2 * i + 1], 8);
      mbar_init(&bar[kPSlotFree + i], 8);
    }
    mbar_init(&bar[kPSDone], 1);
    mbar_init(&bar[kPODone], 1);
    for (int j = 0; j < 2; ++j) mbar_init(&bar[kPLoFree + j], 1);
    for (int c = 0; c < LMAX2 / KC; ++c) mbar_init(&bar[kPChunk + c], 8);
    mbar_init(&bar[kPFullV], 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (tid < 64) {
    reinterpret_cast<uint4*>(smem + kPZero)[tid] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tslot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  float mx_out = 0.0f;
  Item cur = first;
  int it = it0;
  int n = 0;

  if (warp == 0) {
    // ================================================== TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      while (true) {
        const int s = n & 1;
        uint8_t* slot = smem + kPSlot0 + s * kSlotBytes;
        const int half = ((cur.L + 15) & ~15) >> 1;  // this CTA's K rows start at rank * half
        if (n >= 2 && !(ok = mbar_wait_abort(&bar[kPSlotFree + s], ((n >> 1) + 1) & 1, status, abort_flag)))
          break;
        mbar_arrive_expect_tx(&bar[kPFullQK + s], 4 * 16384);
        for (int blk = 0; blk < 2; ++blk) {
          tma_load_2d(slot + kOffQ + blk * 16384, &tmQ, &bar[kPFullQK + s], cur.h * DH + 32 * blk,
                      cur.s0 + 128 * static_cast<int>(rank));
          tma_load_2d(slot + kOffKV + blk * 16384, &tmK, &bar[kPFullQK + s], cur.h * DH + 32 * blk,
                      cur.s0 + half * static_cast<int>(rank));
        }
        // The next item, looked up while this one's wait is pending.
        Item nxt;
        const int itn = next_long(it + stride, stride, n_items, H, cu, nxt);
        // V right behind, into the V buffer once item n-1's P.V is done.
        if (n >= 1 && !(ok = mbar_wait_abort(&bar[kPODone], (n - 1) & 1, status, abort_flag))) break;
        mbar_arrive_expect_tx(&bar[kPFullV], 2 * 16384);
        for (int kb = 0; kb < 2; ++kb)
          tma_load_2d(vbuf + kb * 16384, &tmV, &bar[kPFullV],
                      cur.h * DH + 32 * static_cast<int>(rank), cur.s0 + 128 * kb);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp == 1) {
    // ============================================ MMA issuer (CTA 0)
    if (lane == 0 && rank == 0) {
      uint32_t cpar = 0;
      const uint32_t idO2 = idesc_tf32_bmn(2 * QB, 2 * DH);
      const uint32_t zero = smem_u32(smem + kPZero), vb = smem_u32(vbuf);
      auto commit_both = [&](int i) {
        mma_commit_pair(smem_u32(&bar[i]));
        mma_commit_pair(mapa_shared(smem_u32(&bar[i]), 1));
      };
      while (true) {
        const int s = n & 1;
        const uint32_t slot = smem_u32(smem + kPSlot0 + s * kSlotBytes);
        const int L = cur.L, Lk16 = (L + 15) & ~15, nchunk = (L + KC - 1) / KC;
        if (!(ok = mbar_wait_cluster_abort(&bar[kPQKReady + s], (n >> 1) & 1, status, abort_flag))) break;
        // The single S buffer still holds item n-1's P_hi: issued after that
        // item's P.V MMAs by this thread, S(n) executes after them (in-order
        // tcgen05.mma), so no wait on their completion.
        tc_fence_after();
        const uint32_t idS = idesc_tf32(2 * QB, Lk16);
#pragma unroll
        for (int kk = 0; kk < DH / 8; ++kk) {
          const uint32_t o = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
          const uint64_t a_raw = sw128_kmajor_desc(slot + kOffQ + o);
          const uint64_t b_raw = sw128_kmajor_desc(slot + kOffKV + o);
          const uint64_t b_lo = sw128_kmajor_desc(slot + kOffLo + o);
          mma_tf32_pair(tmem, a_raw, b_raw, idS, kk > 0 ? 1u : 0u);
          if (!qk_bf16) {  // bf16-valued Q and K are exact in tf32: no lo terms
            mma_tf32_pair(tmem, a_raw, b_lo, idS, 1u);
            mma_tf32_ts_pair(tmem, tmem + kColQlo + 8u * kk, b_raw, idS, 1u);
          }
        }
        commit_both(kPSDone);
        // The next item, looked up while this one's wait is pending.
        Item nxt;
        const int itn = next_long(it + stride, stride, n_items, H, cu, nxt);
        for (int c = 0; c < nchunk; ++c) {
          if ((c & 3) == 0 &&  // V_lo of keys [32 c, 32 c + 128)
              !(ok = mbar_wait_cluster_abort(&bar[kPVReady + 2 * s + (c >> 2)], (n >> 1) & 1, status, abort_flag)))
            break;
          if (!(ok = mbar_wait_cluster_abort(&bar[kPChunk + c], (cpar >> c) & 1u, status, abort_flag))) break;
          cpar ^= 1u << c;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < KC / 8; ++kk) {
            // Each CTA's B: its 32 dh columns of V (8 keys) and, one LBO
            // further, of V_lo -- or the zero block for the P_lo term.
            const uint32_t vs = vb + static_cast<uint32_t>(c * 4096 + kk * 1024);
            const uint64_t v_all = sw128b32_mnmajor_desc(vs, slot + kOffLo - vb);
            const uint64_t v_zero = sw128b32_mnmajor_desc(vs, zero - vs);
            const uint32_t p_hi = tmem + 32u * c + 8u * kk;
            const uint32_t p_lo = tmem + kColPlo + 32u * (c & 1) + 8u * kk;
            mma_tf32_ts_pair(tmem + kColO, p_hi, v_all, idO2, (c | kk) != 0 ? 1u : 0u);
            mma_tf32_ts_pair(tmem + kColO, p_lo, v_zero, idO2, 1u);
          }
          if (c + 2 < nchunk) commit_both(kPLoFree + (c & 1));
        }
        if (!ok) break;
        commit_both(kPODone);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp < kSoftWarp0) {
    // ================================================== prep warps
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int ptid = (warp - kPrepWarp0) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    while (true) {
      const int s = n & 1;
      uint8_t* slot = smem + kPSlot0 + s * kSlotBytes;
      const int L = cur.L;
      if (!(ok = mbar_wait_abort(&bar[kPFullQK + s], (n >> 1) & 1, status, abort_flag))) break;
      tile_lo_32k(smem_u32(slot + kOffKV), smem_u32(slot + kOffLo), ptid);
      if (n >= 1 && !(ok = mbar_wait_abort(&bar[kPSDone], (n - 1) & 1, status, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        uint32_t lo[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 x = lds128(smem_u32(slot + kOffQ + blk * 16384 + row * 128) +
                                  static_cast<uint32_t>((c4 ^ (row & 7)) << 4));
          const float4 l = tf32_lo4(x);
          lo[4 * c4] = __float_as_uint(l.x);
          lo[4 * c4 + 1] = __float_as_uint(l.y);
          lo[4 * c4 + 2] = __float_as_uint(l.z);
          lo[4 * c4 + 3] = __float_as_uint(l.w);
        }
        tmem_st32(tmem + kColQlo + 32u * blk + lane_off, lo);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(kPQKReady + s);
      // The next item, looked up while this one's wait is pending.
      Item nxt;
      const int itn = next_long(it + stride, stride, n_items, H, cu, nxt);
      // V_lo (this CTA's 32 dh columns x 256 keys) into the slot once S has
      // consumed K_lo; keys >= L zeroed in the V buffer too.
      if (!(ok = mbar_wait_abort(&bar[kPSDone], n & 1, status, abort_flag))) break;
      if (!(ok = mbar_wait_abort(&bar[kPFullV], n & 1, status, abort_flag))) break;
      {
        const uint32_t vb = smem_u32(vbuf), lo = smem_u32(slot + kOffLo);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float4 x[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            x[i] = lds128(vb + static_cast<uint32_t>((ptid + (h * 8 + i) * 128) * 16));
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t o = static_cast<uint32_t>((ptid + (h * 8 + i) * 128) * 16);
            if (static_cast<int>(o >> 7) >= L) {
              x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
              sts128(vb + o, x[i]);
            }
            sts128(lo + o, tf32_lo4(x[i]));
          }
          fence_proxy_async_smem();  // keys [128 h, 128 h + 128) ready
          __syncwarp();
          if (lane == 0) arrive_leader(kPVReady + 2 * s + h);
        }
      }
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
  } else {
    // ================================================ softmax warps
    const int sw = warp - kSoftWarp0;
    const int quad = warp & 3, par = sw >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int stid = sw * 32 + lane;
    const int lrow = stid >> 4, col4 = (stid & 15) * 4;
    const int q0 = QB * static_cast<int>(rank);
    uint32_t lo_par = 0;  // phase bits of the two P_lo-free barriers
    while (true) {
      const int s = n & 1;
      uint8_t* slot = smem + kPSlot0 + s * kSlotBytes;
      // Row max / sum exchange in the slot's Q region (dead once S is done).
      float (*red_max)[QB] = reinterpret_cast<float (*)[QB]>(slot + kOffQ);
      float (*red_sum)[QB] = reinterpret_cast<float (*)[QB]>(slot + kOffQ + 1024);
      const int L = cur.L, nchunk = (L + KC - 1) / KC;
      const bool w0 = ok && mbar_wait_abort(&bar[kPSDone], n & 1, status, abort_flag);
      tc_fence_after();
      const uint32_t tS = tmem + lane_off;
      float mx = s_row_max(tS, par, nchunk, L);
      red_max[par][row] = mx;
      if (!soft_all(w0)) {
        ok = false;
        break;
      }
      mx = fmaxf(red_max[0][row], red_max[1][row]);
      // Chunk c >= 2 reuses P_lo slot c & 1 once chunk c - 2's P.V is done.
      const float sum = p_chunks(
          tS, tmem + kColPlo + lane_off, 1u, par, nchunk, L, mx,
          [&](int c) {
            if (c >= 2) {
              const int j = c & 1;
              if (ok) ok = mbar_wait_abort(&bar[kPLoFree + j], (lo_par >> j) & 1u, status, abort_flag);
              lo_par ^= 1u << j;
              tc_fence_after();
            }
          },
          [&](int c) {
            if (lane == 0) arrive_leader(kPChunk + c);
          });
      red_sum[par][row] = sum;
      // The next item, looked up while this one's wait is pending.
      Item nxt;
      const int itn = next_long(it + stride, stride, n_items, H, cu, nxt);
      soft_sync();
      const float total = __fadd_rn(red_sum[0][row], red_sum[1][row]);
      const bool w1 = ok && mbar_wait_abort(&bar[kPODone], n & 1, status, abort_flag);
      tc_fence_after();
      // O columns: [P V | P V_lo] of dh 0-31 (CTA 0's B), then of dh 32-63.
      uint32_t o[32], ob[32];
      tmem_ld32(tmem + kColO + lane_off + 64u * par, o);
      tmem_ld32(tmem + kColO + lane_off + 64u * par + 32u, ob);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j)
        o[j] = __float_as_uint(__fadd_rn(__uint_as_float(o[j]), __uint_as_float(ob[j])));
      {
        const float inv = __fdiv_rn(1.0f, total);
        const bool live = q0 + row < L;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 a = make_float4(__fmul_rn(__uint_as_float(o[j]), inv), __fmul_rn(__uint_as_float(o[j + 1]), inv),
                                       __fmul_rn(__uint_as_float(o[j + 2]), inv), __fmul_rn(__uint_as_float(o[j + 3]), inv));
          *reinterpret_cast<float4*>(slot + kOffKV + stage_off(row, par * 8 + (j >> 2))) = a;
          if (live)
            mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
        }
      }
      tc_fence_before();
      if (!soft_all(w1)) {
        ok = false;
        break;
      }
      {
        float* ob = out + static_cast<long>(cur.s0 + q0) * rs + cur.h * DH + col4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = lrow + i * 16;
          if (q0 + r < L)
            *reinterpret_cast<float4*>(ob + static_cast<long>(r) * rs) =
                *reinterpret_cast<const float4*>(slot + kOffKV + stage_off(r, col4 >> 2));
        }
      }
      fence_proxy_async_smem();  // generic writes in the slot precede its next TMA fill
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kPSlotFree + s]);
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
  }

  __syncwarp();
  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (all_ok && amax != nullptr) amax_publish(amax, mx_out);
  tc_fence_before();
  __syncthreads();
  // The pair retires together: CTA 1 arrives on CTA 0's barriers and CTA 0's
  // MMAs read CTA 1's shared memory and TMEM until the last item is done.
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
  if (wait_late) pdl_wait();
}

// ============================================================ long sequences
// Sequences of more than 256 tokens: items = (sequence, head, 128-row query
// tile), one CTA each on a persistent grid, keys in blocks of 128, one
// pass: S_j = Q K_j^T (3xTF32), P_j = 2^((S_j - m) log2 e) chunk by chunk
// into TMEM as in the short kernel, O += P_j V_j (3xTF32), row sums summed
// over the blocks, O / sum at the end.  The reference point m of a row is
// the max of its first block, kept while later blocks' maxima stay within
// 2^8 of P above it; a block whose max exceeds that moves m to the new max
// and rescales O and the row sum by 2^((m_old - m_new) log2 e) first (after
// the previous block's P.V is done).  The normalised result is the same
// function of S as with the global max (the reference's form), at the
// rounding level; rescaling, rare after the first block, is the only step
// the max-first form does not have.
// Two S buffers: S_{j+1} runs on the tensor cores while the softmax warps
// read or convert S_j: the MMAs go S_0, S_1, P.V_0, S_2, P.V_1, ...; P_lo
// has two 32-column slots, chunk c reusing slot c & 1 once the P.V that read
// it last is done.  Tiles flow through a ring of three 64 KB stages (raw |
// lo, the short kernel's slot layout) in the order the MMAs take them: K_0,
// K_1, V_0, K_2, V_1, ..., V_{n-1}; the prep warps form each tile's lo part
// and zero V rows past L.  A tile's load and lo take about two S
// computations, hence three stages.
// TMEM: S0 [0,128) S1 [128,256) O [256,384) P_lo [384,448) Q_lo [448,512).
constexpr uint32_t kLNst = 3;  // ring stages
constexpr uint32_t kLQ = 0, kLRing = 32768, kLStage = 65536;
constexpr uint32_t kLRed = kLRing + kLNst * kLStage;  // [2][128] floats: row max, then row sum
constexpr uint32_t kLBarOff = kLRed + 1024;
constexpr int kLSmemBytes = static_cast<int>(kLBarOff) + 256 + 1024;
// 227 KB per block on sm_100a, less the kernel's static shared memory (128 B).
static_assert(kLSmemBytes + 256 <= 232448, "long-kernel shared memory");
enum : int {
  kLFull = 0,     // [3] TMA tile landed in ring stage s
  kLReady = 3,    // [3] prep done with stage s (4 prep warps)
  kLFree = 6,     // [3] MMAs done with stage s
  kLQFull = 9,    // TMA Q landed
  kLQReady = 10,  // Q_lo in TMEM (4 prep warps)
  kLQFree = 11,   // the item's last S done: Q and Q_lo free
  kLSDone = 12,   // [2] S buffer b holds a finished S
  kLSFree = 14,   // [2] the softmax warps are done with S buffer b (8 warps)
  kLODone = 16,   // the item's P.V done
  kLLoFree = 17,  // [2] the P.V that read P_lo slot s is done
  kLChunk = 19,   // [4] P chunk c written (4 softmax warps)
  kLPVDone = 23,  // a key block's P.V done (once per block, all items)
  kLNumBars = 24
};
// Ring stage and phase parity of tile t.
__device__ __forceinline__ int ring_stage(uint32_t t) { return static_cast<int>(t % kLNst); }
__device__ __forceinline__ uint32_t ring_parity(uint32_t t) { return (t / kLNst) & 1u; }

struct QTile {
  int h, s0, L, q0;
};

// Item it = (b * H + h) * qtiles + qt; valid when L > 256 and q0 < L.
__device__ __forceinline__ bool decode_qtile(int it, int H, int qtiles, const int* __restrict__ cu,
                                             QTile& w) {
  const int per_seq = H * qtiles;
  const int b = it / per_seq;
  const int r = it - b * per_seq;
  w.h = r / qtiles;
  w.q0 = (r - w.h * qtiles) * QB;
  w.s0 = __ldg(cu + b);
  w.L = __ldg(cu + b + 1) - w.s0;
  return w.L > LMAX2 && w.q0 < w.L;
}

__device__ __forceinline__ int next_qtile(int it, int stride, int n_items, int H, int qtiles,
                                          const int* __restrict__ cu, QTile& w) {
  for (; it < n_items; it += stride)
    if (decode_qtile(it, H, qtiles, cu, w)) return it;
  return n_items;
}

// Pass-2 tile i of an item with nkb key blocks: K_0, then K_m and V_{m-1}
// alternately, V_{nkb-1} last.
__device__ __forceinline__ void pass2_tile(int i, int nkb, bool& is_v, int& j) {
  if (i == 0) {
    is_v = false;
    j = 0;
  } else if (i == 2 * nkb - 1) {
    is_v = true;
    j = nkb - 1;
  } else if (i & 1) {
    is_v = false;
    j = (i + 1) >> 1;
  } else {
    is_v = true;
    j = (i >> 1) - 1;
  }
}
__device__ __forceinline__ int pass2_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int pass2_v(int j, int nkb) { return j == nkb - 1 ? 2 * nkb - 1 : 2 * j + 2; }

__global__ void __maxnreg__(128)
    attention_tma_long_kernel(const __grid_constant__ CUtensorMap tmQ,
                              const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const int* __restrict__ cu,
                              int H, int qtiles, int n_items, float* __restrict__ out,
                              uint32_t* amax, uint32_t* status, int qk_bf16, int wait_late) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kLBarOff);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + kLNumBars);
  volatile uint32_t* abort_flag = tslot + 1;
  // wait_late: the previous kernel is another attention kernel of the same
  // call (disjoint sequences, same inputs), which passed its own wait before
  // this grid could launch -- q, k, v and cu are complete.  Waiting for it at
  // the end instead lets these CTAs fill its tail, and this grid still
  // completes after it, so the next kernel's wait covers both.
  if (!wait_late) pdl_wait();
  pdl_trigger();

  const int stride = gridDim.x;
  QTile first;
  const int it0 = next_qtile(blockIdx.x, stride, n_items, H, qtiles, cu, first);
  if (it0 >= n_items) {  // CTA-uniform, before any barrier
    if (wait_late) pdl_wait();
    return;
  }

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long rs = static_cast<long>(H) * DH;  // token row stride (floats)

  if (tid == 0) {
    for (int i = 0; i < static_cast<int>(kLNst); ++i) {
      mbar_init(&bar[kLFull + i], 1);
      mbar_init(&bar[kLReady + i], 4);
      mbar_init(&bar[kLFree + i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar[kLSDone + i], 1);
      mbar_init(&bar[kLSFree + i], 8);
      mbar_init(&bar[kLLoFree + i], 1);
    }
    mbar_init(&bar[kLQFull], 1);
    mbar_init(&bar[kLQReady], 4);
    mbar_init(&bar[kLQFree], 1);
    mbar_init(&bar[kLODone], 1);
    for (int c = 0; c < 4; ++c) mbar_init(&bar[kLChunk + c], 4);
    mbar_init(&bar[kLPVDone], 1);
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  bool ok = true;
  float mx_out = 0.0f;
  QTile cur = first;
  int it = it0;
  int n = 0;        // this CTA's item counter
  uint32_t tb = 0;  // ring index of the item's first tile (3 nkb tiles per item)

  if (warp == 0) {
    // ================================================== TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      while (ok) {
        const int nkb = (cur.L + QB - 1) / QB;
        if (n >= 1 && !(ok = mbar_wait_abort(&bar[kLQFree], (n - 1) & 1, status, abort_flag))) break;
        mbar_arrive_expect_tx(&bar[kLQFull], 2 * 16384);
        for (int blk = 0; blk < 2; ++blk)
          tma_load_2d(smem + kLQ + blk * 16384, &tmQ, &bar[kLQFull], cur.h * DH + 32 * blk,
                      cur.s0 + cur.q0);
        for (int i = 0; i < 2 * nkb; ++i) {
          const uint32_t t = tb + static_cast<uint32_t>(i);
          const int s = ring_stage(t);
          // The stage's previous tile, t - kLNst, must be consumed.
          if (t >= kLNst && !(ok = mbar_wait_abort(&bar[kLFree + s], ring_parity(t - kLNst), status, abort_flag)))
            break;
          bool is_v = false;
          int j = 0;
          pass2_tile(i, nkb, is_v, j);
          uint8_t* st = smem + kLRing + s * kLStage;
          mbar_arrive_expect_tx(&bar[kLFull + s], 2 * 16384);
          for (int blk = 0; blk < 2; ++blk)
            tma_load_2d(st + blk * 16384, is_v ? &tmV : &tmK, &bar[kLFull + s], cur.h * DH + 32 * blk,
                        cur.s0 + QB * j);
        }
        if (!ok) break;
        tb += 2u * static_cast<uint32_t>(nkb);
        QTile nxt;
        const int itn = next_qtile(it + stride, stride, n_items, H, qtiles, cu, nxt);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp == 1) {
    // ==================================================== MMA issuer
    if (lane == 0) {
      uint32_t cpar = 0;  // bit c: parity of the next completion of chunk barrier c
      uint32_t ns = 0;    // S computations issued (S buffer ns & 1)
      const uint32_t idS = idesc_tf32(QB, QB);
      const uint32_t idO = idesc_tf32_bmn(QB, DH);
      const uint32_t idO2 = idesc_tf32_bmn(QB, 2 * DH);
      const uint32_t q_s = smem_u32(smem + kLQ);

      // S = Q_raw K_raw^T + Q_raw K_lo^T + Q_lo K_raw^T for the K tile at
      // ring index t into the next S buffer; returns false on a failed wait.
      auto issue_s = [&](uint32_t t) -> bool {
        const int s = ring_stage(t);
        if (!mbar_wait_abort(&bar[kLReady + s], ring_parity(t), status, abort_flag)) return false;
        const uint32_t b = ns & 1;
        if (ns >= 2 && !mbar_wait_abort(&bar[kLSFree + b], ((ns >> 1) + 1) & 1, status, abort_flag))
          return false;
        ++ns;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + kLRing + s * kLStage), tS = tmem + 128u * b;
#pragma unroll
        for (int kk = 0; kk < DH / 8; ++kk) {
          const uint32_t o = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
          const uint64_t a_raw = sw128_kmajor_desc(q_s + o);
          mma_tf32(tS, a_raw, sw128_kmajor_desc(st + o), idS, kk > 0 ? 1u : 0u);
          if (!qk_bf16) {  // bf16-valued Q and K are exact in tf32: no lo terms
            mma_tf32(tS, a_raw, sw128_kmajor_desc(st + 32768u + o), idS, 1u);
            mma_tf32_ts(tS, tmem + kColQlo + 8u * kk, sw128_kmajor_desc(st + o), idS, 1u);
          }
        }
        mma_commit(&bar[kLSDone + b]);
        mma_commit(&bar[kLFree + s]);
        return true;
      };
      while (ok) {
        const int L = cur.L, nkb = (L + QB - 1) / QB;
        if (!(ok = mbar_wait_abort(&bar[kLQReady], n & 1, status, abort_flag))) break;
        // ---- S_0, S_1, P.V_0, S_2, P.V_1, ...
        const uint32_t t2 = tb;
        const uint32_t b0 = ns & 1;  // S buffer of the item's S_0
        if (!(ok = issue_s(t2))) break;
        if (nkb == 1) mma_commit(&bar[kLQFree]);
        for (int j = 0; j < nkb && ok; ++j) {
          if (j + 1 < nkb) {
            if (!(ok = issue_s(t2 + static_cast<uint32_t>(pass2_k(j + 1))))) break;
            if (j + 2 == nkb) mma_commit(&bar[kLQFree]);  // the item's last S
          }
          const uint32_t t = t2 + static_cast<uint32_t>(pass2_v(j, nkb));
          const int s = ring_stage(t);
          if (!(ok = mbar_wait_abort(&bar[kLReady + s], ring_parity(t), status, abort_flag))) break;
          const uint32_t st = smem_u32(smem + kLRing + s * kLStage);
          const uint32_t tS = tmem + 128u * ((b0 + static_cast<uint32_t>(j)) & 1u);
          const int nchunk = min(QB / KC, (L - QB * j + KC - 1) / KC);
          for (int c = 0; c < nchunk; ++c) {
            if (!(ok = mbar_wait_abort(&bar[kLChunk + c], (cpar >> c) & 1u, status, abort_flag))) break;
            cpar ^= 1u << c;
            tc_fence_after();
            // P_hi [V | V_lo] as one N = 128 MMA, then P_lo V at N = 64.
#pragma unroll
            for (int kk = 0; kk < KC / 8; ++kk) {
              const uint32_t vo = static_cast<uint32_t>(c * 4096 + kk * 1024);
              const uint64_t v_all = sw128b32_mnmajor_desc(st + vo, 16384);
              mma_tf32_ts(tmem + kColO, tS + 32u * c + 8u * kk, v_all, idO2, (j | c | kk) != 0 ? 1u : 0u);
              mma_tf32_ts(tmem + kColO, tmem + kColPlo + 32u * (c & 1) + 8u * kk, v_all, idO, 1u);
            }
            mma_commit(&bar[kLLoFree + (c & 1)]);
          }
          if (!ok) break;
          mma_commit(&bar[kLFree + s]);
          mma_commit(&bar[kLPVDone]);
        }
        if (!ok) break;
        mma_commit(&bar[kLODone]);
        tb += 2u * static_cast<uint32_t>(nkb);
        QTile nxt;
        const int itn = next_qtile(it + stride, stride, n_items, H, qtiles, cu, nxt);
        if (itn >= n_items) break;
        it = itn;
        cur = nxt;
        ++n;
      }
    }
  } else if (warp < kSoftWarp0) {
    // ================================================== prep warps
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int ptid = (warp - kPrepWarp0) * 32 + lane;  // 0..127
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    while (ok) {
      const int L = cur.L, nkb = (L + QB - 1) / QB;
      // Q_lo of this thread's row into TMEM once the previous item's last S
      // has read the previous Q_lo.
      if (!(ok = mbar_wait_abort(&bar[kLQFull], n & 1, status, abort_flag))) break;
      if (n >= 1 && !(ok = mbar_wait_abort(&bar[kLQFree], (n - 1) & 1, status, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        uint32_t lo[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 x = lds128(smem_u32(smem + kLQ + blk * 16384 + row * 128) +
                                  static_cast<uint32_t>((c4 ^ (row & 7)) << 4));
          const float4 l = tf32_lo4(x);
          lo[4 * c4] = __float_as_uint(l.x);
          lo[4 * c4 + 1] = __float_as_uint(l.y);
          lo[4 * c4 + 2] = __float_as_uint(l.z);
          lo[4 * c4 + 3] = __float_as_uint(l.w);
        }
        tmem_st32(tmem + kColQlo + 32u * blk + lane_off, lo);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kLQReady]);
      for (int i = 0; i < 2 * nkb; ++i) {
        const uint32_t t = tb + static_cast<uint32_t>(i);
        const int s = ring_stage(t);
        if (!(ok = mbar_wait_abort(&bar[kLFull + s], ring_parity(t), status, abort_flag))) break;
        bool is_v = false;
        int j = 0;
        pass2_tile(i, nkb, is_v, j);
        const uint32_t raw = smem_u32(smem + kLRing + s * kLStage), lo = raw + 32768u;
        if (!is_v) {
          tile_lo_32k(raw, lo, ptid);  // K_j
        } else {
          // V_j: lo, with keys (rows) past L zeroed in both parts.
          const int kvalid = L - QB * j;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float4 x[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              x[e] = lds128(raw + static_cast<uint32_t>((ptid + (h * 8 + e) * 128) * 16));
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const uint32_t o = static_cast<uint32_t>((ptid + (h * 8 + e) * 128) * 16);
              if (static_cast<int>((o & 16383u) >> 7) >= kvalid) {
                x[e] = make_float4(0.f, 0.f, 0.f, 0.f);
                sts128(raw + o, x[e]);
              }
              sts128(lo + o, tf32_lo4(x[e]));
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[kLReady + s]);
      }
      if (!ok) break;
      tb += 2u * static_cast<uint32_t>(nkb);
      QTile nxt;
      const int itn = next_qtile(it + stride, stride, n_items, H, qtiles, cu, nxt);
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
  } else {
    // ================================================ softmax warps
    // Named barriers are reached by all eight warps at the same points of
    // every item; a failed wait only ends an inner loop, and the AND-votes
    // end the item loop for all of them together.
    const int sw = warp - kSoftWarp0;  // 0..7
    const int quad = warp & 3, par = sw >> 2;
    const int row = quad * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    // One exchange array for the row max and then the row sum; a named
    // barrier after every read keeps each write behind all reads of the
    // previous value.
    float (*red)[QB] = reinterpret_cast<float (*)[QB]>(smem + kLRed);
    uint32_t ns = 0;       // S computations consumed (S buffer ns & 1)
    uint32_t lo_uses = 0;  // this warp's writes of P_lo slot par (chunks c with c & 1 == par)
    uint32_t gblk = 0;     // key blocks before this one, all items: kLPVDone completions
    bool good = ok;
    // Waits for S number ns; returns its TMEM address (this warp's lanes).
    auto next_s = [&](uint32_t& b) -> bool {
      b = ns & 1;
      const bool w = mbar_wait_abort(&bar[kLSDone + b], (ns >> 1) & 1, status, abort_flag);
      ++ns;
      tc_fence_after();
      return w;
    };
    auto release_s = [&](uint32_t b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kLSFree + b]);
    };
    while (true) {
      const int L = cur.L, nkb = (L + QB - 1) / QB;
      // ---- one pass over the key blocks: row max of the block, then the
      // reference point m (and, rarely, a rescale of O and the sum), then P
      // chunks and row sums.  The two warps of a row exchange their halves
      // of the block max through `red` at the same points (AND-votes).
      const float kLog2e = 1.4426950408889634f;
      float m = -INFINITY, sum = 0.0f;
      for (int j = 0; j < nkb; ++j) {
        uint32_t b = 0;
        const bool w = good && next_s(b);
        const int kv = L - QB * j, nch = min(QB / KC, (kv + KC - 1) / KC);
        const uint32_t tS = tmem + 128u * b + lane_off;
        red[par][row] = w ? s_row_max(tS, par, nch, kv) : -INFINITY;
        if (!soft_all(w)) {
          good = false;
          break;
        }
        const float mb = fmaxf(red[0][row], red[1][row]);
        soft_sync();
        float alpha = 1.0f;
        if (j == 0) {
          m = mb;
        } else if (__fmul_rn(__fsub_rn(mb, m), kLog2e) > 8.0f) {
          alpha = ex2_ftz(__fmul_rn(__fsub_rn(m, mb), kLog2e));
          m = mb;
        }
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
          // O holds P.V of blocks 0 .. j-1 against the old m: once the last
          // of them is done, scale this warp's rows of O (its 32 dh columns of
          // both halves) and their sums.  P.V of block j is issued only after
          // this warp's chunks below, which follow the store.
          if (good) good = mbar_wait_abort(&bar[kLPVDone], (gblk - 1) & 1, status, abort_flag);
          tc_fence_after();
          uint32_t o[32], ob[32];
          tmem_ld32(tmem + kColO + lane_off + 32u * par, o);
          tmem_ld32(tmem + kColO + 64u + lane_off + 32u * par, ob);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            o[jj] = __float_as_uint(__fmul_rn(__uint_as_float(o[jj]), alpha));
            ob[jj] = __float_as_uint(__fmul_rn(__uint_as_float(ob[jj]), alpha));
          }
          tmem_st32(tmem + kColO + lane_off + 32u * par, o);
          tmem_st32(tmem + kColO + 64u + lane_off + 32u * par, ob);
          tmem_st_wait();
          sum = __fmul_rn(sum, alpha);
        }
        ++gblk;
        sum = __fadd_rn(sum, p_chunks(tS, tmem + kColPlo + lane_off, 1u, par, nch, kv, m,
                                      [&](int) {
                                        if (lo_uses > 0 && good)
                                          good = mbar_wait_abort(&bar[kLLoFree + par], (lo_uses - 1) & 1,
                                                                 status, abort_flag);
                                        ++lo_uses;
                                        tc_fence_after();
                                      },
                                      [&](int c) {
                                        if (lane == 0) mbar_arrive(&bar[kLChunk + c]);
                                      }));
        release_s(b);
      }
      red[par][row] = sum;
      if (!soft_all(good)) break;
      const float total = __fadd_rn(red[0][row], red[1][row]);
      soft_sync();
      // ---- O / sum straight to the output rows of this tile
      good = mbar_wait_abort(&bar[kLODone], n & 1, status, abort_flag);
      if (good) {
        tc_fence_after();
        uint32_t o[32], ob[32];
        tmem_ld32(tmem + kColO + lane_off + 32u * par, o);
        tmem_ld32(tmem + kColO + 64u + lane_off + 32u * par, ob);
        tmem_ld_wait();
        tc_fence_before();
        const float inv = __fdiv_rn(1.0f, total);
        if (cur.q0 + row < L) {
          float* orow = out + static_cast<long>(cur.s0 + cur.q0 + row) * rs + cur.h * DH + 32 * par;
#pragma unroll
          for (int jj = 0; jj < 32; jj += 4) {
            float4 a;
            a.x = __fmul_rn(__fadd_rn(__uint_as_float(o[jj]), __uint_as_float(ob[jj])), inv);
            a.y = __fmul_rn(__fadd_rn(__uint_as_float(o[jj + 1]), __uint_as_float(ob[jj + 1])), inv);
            a.z = __fmul_rn(__fadd_rn(__uint_as_float(o[jj + 2]), __uint_as_float(ob[jj + 2])), inv);
            a.w = __fmul_rn(__fadd_rn(__uint_as_float(o[jj + 3]), __uint_as_float(ob[jj + 3])), inv);
            *reinterpret_cast<float4*>(orow + jj) = a;
            mx_out = fmaxf(mx_out, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
          }
        }
      }
      QTile nxt;
      const int itn = next_qtile(it + stride, stride, n_items, H, qtiles, cu, nxt);
      if (itn >= n_items) break;
      it = itn;
      cur = nxt;
      ++n;
    }
    ok = good;
  }

  __syncwarp();
  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (all_ok && amax != nullptr) amax_publish(amax, mx_out);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (wait_late) pdl_wait();
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// [T, H*64] fp32 with 128 x 32-float boxes; rows past T read as zero.
// Q and K use the 128-byte swizzle (K-major MMA operands), V the 128-byte
// swizzle with 32-byte atoms (MN-major operand).
bool make_tmap_rows(CUtensorMap* map, const float* base, long T, long cols,
                    CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || (cols % 4)) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 4)};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Every sequence of 1..128 tokens; others are skipped (callers run the
// longer ones elsewhere).  T = cu[B] (host-known), num_sms = grid bound.
cudaError_t launch_attention_tma(const float* q, const float* k, const float* v, const int* cu,
                                 int B, int H, long T, float* out, uint32_t* amax,
                                 uint32_t* status, int num_sms, bool qk_bf16, cudaStream_t s) {
  if (B <= 0 || H <= 0 || T <= 0) return cudaSuccess;
  CUtensorMap tmQ, tmK, tmV;
  const long cols = static_cast<long>(H) * DH;
  if (!make_tmap_rows(&tmQ, q, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmK, k, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmV, v, T, cols, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(attention_tma_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const long n_items = static_cast<long>(B) * H;
  if (n_items > (1L << 30)) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long>(n_items, std::max(1, num_sms)));
  return launch_pdl(attention_tma_kernel, dim3(grid), dim3(kThreads), kSSmemBytes, s, tmQ, tmK, tmV,
                    cu, H, static_cast<int>(n_items), out, amax, status, qk_bf16 ? 1 : 0);
}

// Every sequence of 129..256 tokens, one CTA pair per (sequence, head).
cudaError_t launch_attention_tma_pair(const float* q, const float* k, const float* v,
                                      const int* cu, int B, int H, long T, float* out,
                                      uint32_t* amax, uint32_t* status, int num_sms, bool qk_bf16,
                                      cudaStream_t s,
                                      bool wait_late) {
  if (B <= 0 || H <= 0 || T <= 0) return cudaSuccess;
  CUtensorMap tmQ, tmK, tmV;
  const long cols = static_cast<long>(H) * DH;
  if (!make_tmap_rows(&tmQ, q, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmK, k, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmV, v, T, cols, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(attention_tma_pair_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const long n_items = static_cast<long>(B) * H;
  if (n_items > (1L << 30)) return cudaErrorInvalidValue;
  const int pairs = static_cast<int>(std::max<long>(1, std::min<long>(n_items, std::max(1, num_sms / 2))));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1] = pdl_attribute();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, attention_tma_pair_kernel, tmQ, tmK, tmV, cu, H,
                            static_cast<int>(n_items), out, amax, status, qk_bf16 ? 1 : 0,
                            wait_late ? 1 : 0);
}

// Every sequence of more than 256 tokens: items = (sequence, head, 128-row
// query tile), qtiles = ceil(max_len / 128) tiles reserved per (sequence,
// head); one persistent CTA per SM at most.
cudaError_t launch_attention_tma_long(const float* q, const float* k, const float* v,
                                      const int* cu, int B, int H, long T, int max_len, float* out,
                                      uint32_t* amax, uint32_t* status, int num_sms, bool qk_bf16,
                                      cudaStream_t s,
                                      bool wait_late) {
  if (B <= 0 || H <= 0 || T <= 0 || max_len <= LMAX2) return cudaSuccess;
  CUtensorMap tmQ, tmK, tmV;
  const long cols = static_cast<long>(H) * DH;
  if (!make_tmap_rows(&tmQ, q, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmK, k, T, cols, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_rows(&tmV, v, T, cols, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B))
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(attention_tma_long_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kLSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  const int qtiles = (max_len + QB - 1) / QB;
  const long n_items = static_cast<long>(B) * H * qtiles;
  if (n_items > (1L << 30)) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long>(n_items, std::max(1, num_sms)));
  return launch_pdl(attention_tma_long_kernel, dim3(grid), dim3(kThreads), kLSmemBytes, s, tmQ, tmK,
                    tmV, cu, H, qtiles, static_cast<int>(n_items), out, amax, status,
                    qk_bf16 ? 1 : 0, wait_late ? 1 : 0);
}

}  // namespace esmb200

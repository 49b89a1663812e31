// W8A8 INT8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Replaces the reference's LinearVnni / LinearAmx integer core
// (gemm_int8.cpp:232-555, gemm_amx.cpp:146-309) and its FinalizeStore16
// dequant (gemm_int8.cpp:109-126).  The reference quantises activations to
// u8 with zero point 128 and subtracts 128*col_sum afterwards; the tensor
// cores take s8 x s8 directly, which yields the same int32 sum_k q*w.
//
// Structure (persistent, one CTA per SM, 320 threads):
//   warp 0      TMA producer: A [128 x 128] and W [BN x 128] int8 tiles,
//               128-byte swizzle, into a STAGES-deep shared-memory ring.
//   warp 1      TMEM owner + MMA issuer: 4 x (M=128, N=BN, K=32) MMAs per
//               stage into one of two TMEM accumulators (2*BN columns).
//   warps 2..9  epilogue, two warps per TMEM lane quadrant: tcgen05.ld 32
//               columns at a time (one output row per thread), dequant
//               fma(float(acc), ws[n]*as, bias[n]), then store / residual /
//               GELU / QKV-split+RoPE through TMA stores.
// The BN = 256 tiles run on CTA pairs (2-CTA clusters, tcgen05 cta_group::2):
// the pair computes a 256 x 256 tile with M = 256 MMAs issued by CTA 0, each
// CTA loading its own 128 rows of A and 128 rows of W, so a stage moves 32 KB
// into each SM instead of 48 KB for the same math.  Each CTA's epilogue
// drains its own 128 TMEM rows.
// The epilogue of tile i overlaps the mainloop of tile i+1.  Every barrier
// wait is bounded; a timeout sets a status bit and the CTA unwinds.
//
// The same kernel in its F32 mode is the 3xTF32 FP32 GEMM (launch_gemm_tf32x3,
// the reference's FP32 Linear, gemm_fp32.cpp:272-292, for the LM head): a
// stage holds 32 K-elements of A, W and their lo parts (x - tf32(x), formed
// by launch_tf32_lo), three kind::tf32 MMAs per 8 K-elements (A W + A W_lo +
// A_lo W; the tensor core reads the raw fp32 word as its tf32 hi part), and
// the epilogue adds the bias to the fp32 accumulator.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
// Epilogue warps per CTA (EW): 16 (four per TMEM lane quadrant) for the
// instruction-heavy GELU epilogue, 8 for the others.
constexpr int threads_for(int ew) { return 64 + 32 * ew; }  // + producer, MMA issuer
constexpr int kSmemLimit = 232448;                            // opt-in maximum per CTA

// F32: the tf32x3 mode -- fp32 operands, a stage holds 32 K-elements of A
// and W (raw) and of their lo parts, 128-byte rows each.
template <int BN, bool PAIR, int EW, int ROPE = 0, bool F32 = false>
struct Cfg {
  static constexpr int A_RAW = BM * BK;
  static constexpr int B_RAW = (PAIR ? BN / 2 : BN) * BK;  // this CTA's rows of W
  static constexpr int A_BYTES = (F32 ? 2 : 1) * A_RAW;     // [raw | lo] in F32 mode
  static constexpr int B_BYTES = (F32 ? 2 : 1) * B_RAW;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;

  static constexpr int TMEM_COLS = 2 * BN;
  // Epilogue staging for TMA stores: one [32 rows x 128 B] per warp, then the
  // tile's (w_scale * a_scale) and bias columns shared by the epilogue warps.
  static constexpr int STAGING_BYTES = EW * 4096;
  // (F32: the bias columns only)
  static constexpr int COLVEC_BYTES = (F32 ? 1 : 2) * BN * 4;
  // RoPE epilogue: the tile rows' cos / sin table entries 0..31 (128 rows x
  // 256 bytes), staged once per tile.
  static constexpr int ROPE_BYTES = ROPE ? BM * 256 : 0;
  // As many stages as the rest of shared memory holds (at most 8).  The
  // tiles start at the first 1024-byte boundary of the dynamic shared memory
  // (16-byte aligned: up to 1008 bytes of padding); the mbarriers (BAR_BYTES)
  // sit in that padding when it has room and after the tiles otherwise, so
  // 1024 bytes cover both.
  static constexpr int BAR_BYTES = 256;
  static constexpr int FIT = (kSmemLimit - 1024 - STAGING_BYTES - COLVEC_BYTES - ROPE_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = FIT < 8 ? FIT : 8;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + COLVEC_BYTES + ROPE_BYTES;
  static constexpr int SMEM = TILE_BYTES + 1024;
  static_assert(2 * STAGES * 8 + 4 * 8 + 4 <= BAR_BYTES, "mbarriers and the TMEM slot fit BAR_BYTES");
};

struct Params {
  int M, N, K;
  const float* w_scale;
  const float* a_scale;
  int per_token;
  const float* bias;
  EpiParams epi;
  uint32_t* status;
  int32_t* acc_out;
  int tma;  // epilogue stores through TMA (tensor maps tmC0..2 valid)
  int band;  // row slabs per tile band (0: all of them, row-slab-fastest order)
};

// Named barrier 1 across the EW epilogue warps only.
template <int EW>
__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, %0;" ::"n"(EW * 32) : "memory");
}
// The same barrier with an AND-vote: every epilogue warp gets the same answer,
// so a timeout leaves the loop in all of them together (none is left waiting
// at a later barrier).
template <int EW>
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "barrier.cta.red.and.pred po, 1, %2, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "n"(EW * 32)
      : "memory");
  return r != 0;
}

// Register cap: with EW = 16, 18 warps put five on one SM sub-partition (16K
// registers each) -> 96; with EW = 8, three -> 168.
template <int BN, int EPI, bool PAIR, int EW, bool F32 = false>
__global__ void __maxnreg__(EW == 16 ? 96 : 168)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC0,
                   const __grid_constant__ CUtensorMap tmC1,
                   const __grid_constant__ CUtensorMap tmC2,
                   const __grid_constant__ CUtensorMap tmAlo,
                   const __grid_constant__ CUtensorMap tmBlo, const Params p) {
  using C = Cfg<BN, PAIR, EW, EPI == kEpiQkvRope, F32>;
  constexpr int kEpiPerQuad = EW / 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;
  float* colvec = reinterpret_cast<float*>(staging + C::STAGING_BYTES);
  uint8_t* rope_cs = staging + C::STAGING_BYTES + C::COLVEC_BYTES;
  // The barriers: in the alignment padding when it holds them (the same
  // place in both CTAs of a pair: same kernel, same shared-memory layout).
  uint8_t* bar_region = (smem - smem_raw >= C::BAR_BYTES) ? smem_raw : smem + C::TILE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_region);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // one arrive per epilogue warp (of both CTAs of a pair: CTA 0's copy)
      mbar_init(&tempty[a], EW * (PAIR ? 2 : 1));
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (F32) {
      prefetch_tmap(&tmAlo);
      prefetch_tmap(&tmBlo);
    }
    if (p.tma) {
      prefetch_tmap(&tmC0);
      if (EPI == kEpiQkvRope) {
        prefetch_tmap(&tmC1);
        prefetch_tmap(&tmC2);
      }
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // CTA 0's barriers exist before CTA 1 signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Setup done; from here on the previous kernel's outputs are read (A, the
  // activation scale) and buffers it may still read are written (C).
  pdl_wait();
  pdl_trigger();

  // Tiles: m_units row slabs (128 rows, or 256 per pair) x n_blocks.  A pair
  // shares one tile index; CTA `rank` takes rows [128 rank, 128 rank + 128).
  // Tile order: bands of `band` row slabs, each band's tiles (row slab
  // fastest) before the next band's, so the tiles in flight share one band
  // of A -- which stays in L2 across the column blocks -- where A is too
  // large to stay in L2 whole; band = m_units is row-slab-fastest over all
  // of A.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int first_tile = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tile_stride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int m_units = PAIR ? (p.M + 2 * BM - 1) / (2 * BM) : (p.M + BM - 1) / BM;
  const int n_blocks = (p.N + BN - 1) / BN;
  const int num_tiles = m_units * n_blocks;
  const int kpb = F32 ? BK / 4 : BK;  // K elements per stage
  const int num_kb = (p.K + kpb - 1) / kpb;
  const int band = p.band > 0 && p.band < m_units ? p.band : m_units;
  auto tile_mu = [&](int tile) {
    const int b0 = (tile / (band * n_blocks)) * band;
    const int rows_b = min(band, m_units - b0);
    return b0 + (tile - b0 * n_blocks) % rows_b;
  };
  auto tile_nb = [&](int tile) {
    const int b0 = (tile / (band * n_blocks)) * band;
    const int rows_b = min(band, m_units - b0);
    return (tile - b0 * n_blocks) / rows_b;
  };
  auto tile_m_base = [&](int tile) {
    const int mu = tile_mu(tile);
    return PAIR ? mu * 2 * BM + static_cast<int>(rank) * BM : mu * BM;
  };

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_stride) {
        const int m_base = tile_m_base(tile);
        const int n_blk = tile_nb(tile);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
            ok = false;
            break;
          }
          const int kx = F32 ? kb * (BK / 4) : kb * BK;  // K coordinate in elements
          const int nrow = n_blk * BN + (PAIR ? static_cast<int>(rank) * (BN / 2) : 0);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if (PAIR) {
            // Both CTAs' bytes complete on CTA 0's full barrier, which CTA 0
            // arms for the pair.
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t bar0 = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(a_dst, &tmA, bar0, kx, m_base);
            tma_load_2d_pair(b_dst, &tmB, bar0, kx, nrow);
            if (F32) {
              tma_load_2d_pair(a_dst + C::A_RAW, &tmAlo, bar0, kx, m_base);
              tma_load_2d_pair(b_dst + C::B_RAW, &tmBlo, bar0, kx, nrow);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(a_dst, &tmA, &full[stage], kx, m_base);
            tma_load_2d(b_dst, &tmB, &full[stage], kx, nrow);
            if (F32) {
              tma_load_2d(a_dst + C::A_RAW, &tmAlo, &full[stage], kx, m_base);
              tma_load_2d(b_dst + C::B_RAW, &tmBlo, &full[stage], kx, nrow);
            }
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: wait until the consumer has released every issued stage so no
      // TMA write is still landing in shared memory when the CTA retires.
      for (int i = 0; i < C::STAGES && ok; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) break;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = F32 ? idesc_tf32(PAIR ? 2 * BM : BM, BN) : idesc_i8(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_stride) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            const uint64_t ad = sw128_kmajor_desc(a0 + k * 32), bd = sw128_kmajor_desc(b0 + k * 32);
            const uint32_t acc_in = (kb | k) != 0 ? 1u : 0u;
            if constexpr (F32) {
              // 3xTF32: A W + A W_lo + A_lo W (the tensor core reads an fp32
              // word as tf32 by dropping its low 13 bits, so raw = hi).
              const uint64_t alo = sw128_kmajor_desc(a0 + C::A_RAW + k * 32);
              const uint64_t blo = sw128_kmajor_desc(b0 + C::B_RAW + k * 32);
              if (PAIR) {
                mma_tf32_pair(d_tmem, ad, bd, idesc, acc_in);
                mma_tf32_pair(d_tmem, ad, blo, idesc, 1u);
                mma_tf32_pair(d_tmem, alo, bd, idesc, 1u);
              } else {
                mma_tf32(d_tmem, ad, bd, idesc, acc_in);
                mma_tf32(d_tmem, ad, blo, idesc, 1u);
                mma_tf32(d_tmem, alo, bd, idesc, 1u);
              }
            } else if (PAIR) {
              mma_i8_pair(d_tmem, ad, bd, idesc, acc_in);
            } else {
              mma_i8(d_tmem, ad, bd, idesc, acc_in);
            }
          }
          if (PAIR) {  // the stage is free in both CTAs
            mma_commit_pair(smem_u32(&empty[stage]));
            mma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            mma_commit(&empty[stage]);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (PAIR) {
          mma_commit_pair(smem_u32(&tfull[acc]));
          mma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
        } else {
          mma_commit(&tfull[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    // Warps 2..: TMEM lane quadrant warp % 4 (the hardware rule); the
    // kEpiPerQuad warps of a quadrant (index `sub`) take every kEpiPerQuad-th
    // column chunk.
    const int quad = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int etid = (warp - 2) * 32 + lane;  // index among epilogue threads
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    float amax = 0.0f;
    static_assert(BN <= EW * 32, "one vector column per epilogue thread");
    const bool has_col = p.acc_out == nullptr && etid < BN;
    // Per-tensor scale: ws[n]*as is the same for every row, so the rounded
    // product (the reference rounds it before the fma) is formed once per
    // column; the raw-accumulator mode carries no activation scale.
    const bool scaled = !F32 && p.acc_out == nullptr;
    const float as_col = (scaled && !p.per_token) ? __ldg(p.a_scale) : 1.0f;
    // The per-tile inputs of the epilogue -- this thread's w_scale / bias
    // column, its row's per-token scale, and (RoPE) its row's position and
    // cos / sin table entries -- are fetched one tile ahead (the position two
    // tiles ahead, as the table rows depend on it), so their global-memory
    // latency overlaps the current tile's work instead of preceding the
    // accumulator wait.
    auto fetch_cols = [&](int t, float& ws, float& b, float& as_row) {
      const long mm = static_cast<long>(tile_m_base(t)) + row_in_tile;
      as_row = (scaled && p.per_token && mm < p.M) ? __ldg(p.a_scale + mm) : 1.0f;
      ws = 0.0f;
      b = 0.0f;
      if (has_col) {  // tail columns read the last valid column
        const int n = min(tile_nb(t) * BN + etid, p.N - 1);
        if (!F32) ws = __ldg(p.w_scale + n);
        b = p.bias ? __ldg(p.bias + n) : 0.0f;
      }
    };
    constexpr bool kRope = EPI == kEpiQkvRope;
    // RoPE: the quadrant's 32 rows' cos (warp sub 0) or sin (sub 1) table
    // entries 0..31, 8 lanes per 128-byte row (coalesced): lane l holds
    // entry chunk l & 7 of rows (l >> 3) + 4 i.
    auto fetch_pos = [&](int t) {
      const long mm = static_cast<long>(tile_m_base(t)) + row_in_tile;
      return (kRope && p.tma && t < num_tiles && mm < p.M) ? __ldg(p.epi.pos + mm) : 0;
    };
    float4 rope_v[kRope ? 8 : 1];
    auto fetch_rope = [&](int pos_m) {
      if constexpr (kRope) {
        const float* tab = sub == 0 ? p.epi.cos_t : p.epi.sin_t;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int pr = __shfl_sync(0xffffffffu, pos_m, i * 4 + (lane >> 3));
          rope_v[i] = __ldg(reinterpret_cast<const float4*>(tab + static_cast<long>(pr) * 64) + (lane & 7));
        }
      }
    };
    float ws_nx = 0.0f, b_nx = 0.0f, as_nx = 1.0f;
    fetch_cols(first_tile, ws_nx, b_nx, as_nx);
    int pos_nx = 0;
    if constexpr (kRope) {
      if (p.tma) {
        fetch_rope(fetch_pos(first_tile));
        pos_nx = fetch_pos(first_tile + tile_stride);
      }
    }
    for (int tile = first_tile; tile < num_tiles; tile += tile_stride) {
      const int m_base = tile_m_base(tile);
      const int n_blk = tile_nb(tile);
      // This tile's RoPE rows into shared memory (row r's 16-byte chunk k at
      // position k ^ (r & 7), so the per-row reads are conflict-free); the
      // previous tile's readers are past the tile-end barrier, this tile's
      // read after the vectors-filled barrier.  Then the next tile's rows.
      if constexpr (kRope) {
        static_assert(EW / 4 == 2, "two epilogue warps per TMEM lane quadrant");
        if (p.tma) {
          uint8_t* qreg = rope_cs + quad * 32 * 256 + sub * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3), k = lane & 7;
            sts128(smem_u32(qreg + r * 256 + ((k ^ (r & 7)) << 4)), rope_v[i]);
          }
          fetch_rope(pos_nx);
          pos_nx = fetch_pos(tile + 2 * tile_stride);
        }
      }
      const long m = static_cast<long>(m_base) + row_in_tile;
      const bool row_ok = m < p.M;
      const float as = as_nx, ws_col = ws_nx, b_col = b_nx;
      if (tile + tile_stride < num_tiles) fetch_cols(tile + tile_stride, ws_nx, b_nx, as_nx);
      if (!epi_all<EW>(mbar_wait(&tfull[acc], acc_phase, p.status))) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);

      // This tile's w_scale / bias columns in shared memory for all epilogue
      // warps.
      float* wsv = colvec;
      float* bsv = F32 ? colvec : colvec + BN;
      if (has_col) {
        if (!F32) wsv[etid] = p.per_token ? ws_col : __fmul_rn(ws_col, as_col);
        bsv[etid] = b_col;
      }
      epi_barrier<EW>();  // vectors filled
      // Dequant of 32 accumulators at tile columns jc0.. (jc0 a multiple of
      // 4): fma(float(acc), ws[n]*as, bias[n]) (gemm_int8.cpp:109-126), the
      // column vectors read as float4.
      const uint32_t wsv_s = smem_u32(wsv), bsv_s = smem_u32(bsv);
      auto deq32 = [&](const uint32_t(&r)[32], int jc0, float* y) {
        if constexpr (F32) {  // fp32 accumulator + bias (gemm_fp32.cpp's Linear)
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 b = lds128(bsv_s + static_cast<uint32_t>((jc0 + 4 * j4) * 4));
            const float bs[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
              y[4 * j4 + u] = __fadd_rn(__uint_as_float(r[4 * j4 + u]), bs[u]);
          }
        } else {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const uint32_t o = static_cast<uint32_t>((jc0 + 4 * j4) * 4);
            const float4 w = lds128(wsv_s + o), b = lds128(bsv_s + o);
            unsigned long long w01 = f2_pack(w.x, w.y), w23 = f2_pack(w.z, w.w);
            if (p.per_token) {
              const unsigned long long as2 = f2_pack(as, as);
              w01 = f2_mul(w01, as2);
              w23 = f2_mul(w23, as2);
            }
            const int* ri = reinterpret_cast<const int*>(r) + 4 * j4;
            // fma(float(acc), scale, bias) two columns per instruction
            f2_unpack(f2_fma(f2_pack(__int2float_rn(ri[0]), __int2float_rn(ri[1])), w01,
                             f2_pack(b.x, b.y)),
                      y[4 * j4], y[4 * j4 + 1]);
            f2_unpack(f2_fma(f2_pack(__int2float_rn(ri[2]), __int2float_rn(ri[3])), w23,
                             f2_pack(b.z, b.w)),
                      y[4 * j4 + 2], y[4 * j4 + 3]);
          }
        }
      };
      // This warp's staging buffer and the top row of its 32-row slab.
      uint8_t* stg_one = staging + (warp - 2) * 4096;
      auto next_stg = [&]() {
        if (lane == 0) bulk_wait_read<0>();  // the buffer's last store has read it
        __syncwarp();
        return stg_one;
      };
      const int y0 = m_base + quad * 32;
      // Stage y[0..32) of this thread's row (lane) with the 128-byte swizzle
      // the tensor map expects.
      auto stage32 = [&](uint8_t* buf, const float* y) {
        const uint32_t b = smem_u32(buf) + static_cast<uint32_t>(lane * 128);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          sts128(b + static_cast<uint32_t>((j ^ (lane & 7)) * 16),
                 make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]));
      };

      // One 32-column chunk of the plain epilogues (store / residual / GELU /
      // raw int32), from accumulators already in registers.
      auto epi_chunk = [&](int c, const uint32_t(&r)[32]) {
        const int n0 = n_blk * BN + c * 32;
        if (n0 >= p.N) return;  // warp-uniform
        if (p.acc_out != nullptr) {
          if (row_ok)
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) p.acc_out[m * p.N + n0 + j] = static_cast<int32_t>(r[j]);
          return;
        }
        float y[32];
        deq32(r, c * 32, y);
        if (!p.tma) {
          if (row_ok) amax = fmaxf(amax, epi_row_run<32>(p.epi, m, n0, p.N, y));
          return;
        }
        if (p.epi.kind == kEpiGelu) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) gelu_erf2(y[j], y[j + 1]);
        }
        if (row_ok && p.epi.amax != nullptr) {
          if (n0 + 32 <= p.N) {  // warp-uniform: the whole chunk is in range
#pragma unroll
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(y[j]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) amax = fmaxf(amax, fabsf(y[j]));
          }
        }
        uint8_t* stg = next_stg();
        stage32(stg, y);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // hidden += proj (fp32 add in the memory system: h + y rounded once)
          if (p.epi.kind == kEpiResidual) tma_reduce_add_2d(&tmC0, stg, n0, y0);
          else tma_store_2d(&tmC0, stg, n0, y0);
          bulk_commit();
        }
      };

      if (EPI == kEpiQkvRope) {
#pragma unroll 1
        for (int c = sub; c < BN / 64; c += kEpiPerQuad) {
          uint32_t lo[32], hi[32];
          tmem_ld32(t_row + c * 64, lo);
          tmem_ld32(t_row + c * 64 + 32, hi);
          tmem_ld_wait();
          const int n_base = n_blk * BN + c * 64;
          if (n_base < p.N) {  // warp-uniform
            float y[64];
            deq32(lo, c * 64, y);
            deq32(hi, c * 64 + 32, y + 32);
            if (p.tma) {
              const int which = n_base / p.epi.d;
              const int col = n_base - which * p.epi.d;
              epi_qkv_rope_values(p.epi, smem_u32(rope_cs + row_in_tile * 256), lane & 7, which, y);
              const CUtensorMap* mp = which == 0 ? &tmC0 : (which == 1 ? &tmC1 : &tmC2);
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                uint8_t* stg = next_stg();
                stage32(stg, y + 32 * half);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  tma_store_2d(mp, stg, col + 32 * half, y0);
                  bulk_commit();
                }
              }
            } else if (row_ok) {
              epi_qkv_rope_head(p.epi, m, n_base, y);
            }
          }
        }
      } else {
        // This warp's 32-column chunks: sub, sub + kEpiPerQuad, ...
#pragma unroll 1
        for (int c = sub; c < BN / 32; c += kEpiPerQuad) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_ld_wait();
          epi_chunk(c, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        else mbar_arrive(&tempty[acc]);
      }
      epi_barrier<EW>();  // every epilogue warp is done with this tile's vectors
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.epi.amax != nullptr) amax_publish_warp(p.epi.amax, amax);
    if (p.tma && lane == 0) bulk_wait<0>();  // stores done before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  // A pair retires together: CTA 1's epilogue arrives on CTA 0's barriers and
  // CTA 0's MMAs read CTA 1's shared memory until the last tile is done.
  if (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
  }
  return fn;
}

// 2-D int8 tensor [rows, cols] with row stride `ld` bytes; box = [box_rows,
// 128 bytes], 128-byte swizzle, out-of-range elements read as zero.
bool make_tmap_i8(CUtensorMap* map, const int8_t* base, int rows, int cols, long ld,
                  int box_rows) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D fp32 tensor [rows, cols] with row stride `ld` floats; box = 32 columns
// x box_rows (128-byte rows, 128-byte swizzle): 32 x 32 for the epilogue's
// TMA stores, BM or BN rows for the tf32x3 operand loads.
bool make_tmap_f32(CUtensorMap* map, const float* base, long rows, long cols, long ld,
                   int box_rows = 32) {
  auto fn = get_encode_fn();
  if (fn == nullptr || base == nullptr || (ld & 3) || (reinterpret_cast<uintptr_t>(base) & 15))
    return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI, bool PAIR, int EW>
cudaError_t launch_bn(const GemmI8Args& a, cudaStream_t s) {
  using C = Cfg<BN, PAIR, EW, EPI == kEpiQkvRope>;
  constexpr int kThreads = threads_for(EW);
  CUtensorMap tmA, tmB, tmC[3];
  if (!make_tmap_i8(&tmA, a.A, a.M, a.K, a.lda, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_i8(&tmB, a.W, a.N, a.K, a.ldw, PAIR ? BN / 2 : BN)) return cudaErrorInvalidValue;
  std::memset(tmC, 0, sizeof(tmC));
  bool tma = false;
  if (a.acc_out == nullptr) {
    if (EPI == kEpiQkvRope) {
      tma = (a.epi.d % 32 == 0) && make_tmap_f32(&tmC[0], a.epi.q, a.M, a.epi.d, a.epi.d) &&
            make_tmap_f32(&tmC[1], a.epi.k, a.M, a.epi.d, a.epi.d) &&
            make_tmap_f32(&tmC[2], a.epi.v, a.M, a.epi.d, a.epi.d);
    } else {
      tma = make_tmap_f32(&tmC[0], a.epi.C, a.M, a.N, a.epi.ldc);
    }
  }
  // The opt-in shared-memory size is a per-device function attribute.
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, EPI, PAIR, EW, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  Params p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.w_scale = a.w_scale;
  p.a_scale = a.a_scale;
  p.per_token = a.per_token;
  p.bias = a.bias;
  p.epi = a.epi;
  p.status = a.status;
  p.acc_out = a.acc_out;
  p.tma = tma ? 1 : 0;
  // Where A is too large to stay in L2 across the column blocks (long K),
  // bands of row slabs just wide enough for the tiles in flight.
  p.band = 0;
  if (static_cast<long>(a.M) * a.K > (32l << 20)) {
    const int nb = (a.N + BN - 1) / BN;
    const int in_flight = PAIR ? a.num_sms / 2 : a.num_sms;
    p.band = std::max(1, (in_flight + nb - 1) / nb);
  }
  if constexpr (!PAIR) {
    const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    const int grid = tiles < a.num_sms ? tiles : a.num_sms;
    return launch_pdl(gemm_i8_kernel<BN, EPI, false, EW, false>, dim3(grid), dim3(kThreads),
                      C::SMEM, s, tmA, tmB, tmC[0], tmC[1], tmC[2], tmC[1], tmC[2], p);
  } else {
  // CTA pairs: one 2-CTA cluster per pair tile, at most num_sms / 2 pairs.
  const int tiles = ((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + BN - 1) / BN);
  const int pairs = std::max(1, std::min(tiles, a.num_sms / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1] = pdl_attribute();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN, EPI, true, EW, false>, tmA, tmB, tmC[0],
                            tmC[1], tmC[2], tmC[1], tmC[2], p);
  }
}

// The tf32x3 mode (fp32 operands with their lo parts): BN = 256 on CTA pairs
// or BN = 128 on single CTAs, 8 epilogue warps, 3 stages of 64 KB.
template <int BN, bool PAIR>
cudaError_t launch_f32(const GemmTf32Args& a, cudaStream_t s) {
  constexpr int EW = 8;
  using C = Cfg<BN, PAIR, EW, 0, true>;
  static_assert(C::STAGES >= 2, "the tf32x3 ring needs two stages");
  constexpr int kThreads = threads_for(EW);
  constexpr int brow = PAIR ? BN / 2 : BN;
  CUtensorMap tmA, tmAlo, tmB, tmBlo, tmC[3];
  if (!make_tmap_f32(&tmA, a.A, a.M, a.K, a.lda, BM) ||
      !make_tmap_f32(&tmAlo, a.A_lo, a.M, a.K, a.lda, BM) ||
      !make_tmap_f32(&tmB, a.W, a.N, a.K, a.ldw, brow) ||
      !make_tmap_f32(&tmBlo, a.W_lo, a.N, a.K, a.ldw, brow))
    return cudaErrorInvalidValue;
  std::memset(tmC, 0, sizeof(tmC));
  const bool tma = make_tmap_f32(&tmC[0], a.epi.C, a.M, a.N, a.epi.ldc);
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if ((attr_set.load() & bit) == 0) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, kEpiStore, PAIR, EW, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit);
  }
  Params p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.w_scale = nullptr;
  p.a_scale = nullptr;
  p.per_token = 0;
  p.bias = a.bias;
  p.epi = a.epi;
  p.status = a.status;
  p.acc_out = nullptr;
  p.tma = tma ? 1 : 0;
  p.band = 0;
  if constexpr (!PAIR) {
    const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
    const int grid = tiles < a.num_sms ? tiles : a.num_sms;
    return launch_pdl(gemm_i8_kernel<BN, kEpiStore, false, EW, true>, dim3(grid), dim3(kThreads),
                      C::SMEM, s, tmA, tmB, tmC[0], tmC[1], tmC[2], tmAlo, tmBlo, p);
  } else {
    const int tiles = ((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + BN - 1) / BN);
    const int pairs = std::max(1, std::min(tiles, a.num_sms / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1] = pdl_attribute();
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gemm_i8_kernel<BN, kEpiStore, true, EW, true>, tmA, tmB,
                              tmC[0], tmC[1], tmC[2], tmAlo, tmBlo, p);
  }
}

}  // namespace

cudaError_t launch_gemm_i8(const GemmI8Args& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  if (a.K <= 0 || (a.K & 15) || (a.lda & 15) || (a.ldw & 15) ||
      (reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.W) & 15) ||
      a.status == nullptr)
    return cudaErrorInvalidValue;
  if (a.acc_out == nullptr && (a.a_scale == nullptr || a.w_scale == nullptr))
    return cudaErrorInvalidValue;  // dequant needs both scales
  const int epi = a.acc_out ? kEpiStore : a.epi.kind;
  if (epi == kEpiQkvRope) {
    // One tile never straddles q|k|v and holds whole 64-wide heads.
    if (a.epi.d % 256 == 0) return launch_bn<256, kEpiQkvRope, false, 8>(a, s);
    if (a.epi.d % 64 == 0) return launch_bn<64, kEpiQkvRope, false, 8>(a, s);
    return cudaErrorInvalidValue;
  }
  // Wide tiles when N is large, narrower ones to fill the SMs otherwise.
  // CTA pairs where the mainloop dominates (long K): there the operand feed,
  // not the epilogue, sets the pace, and pairs cut it by a third.
  const long tiles256 = ((a.M + BM - 1) / BM) * static_cast<long>((a.N + 255) / 256);
  const bool wide = a.N >= 256 && tiles256 >= a.num_sms;
  // The epilogue kind is a runtime field; the heavy GELU epilogue gets 16 warps.
  const bool gelu = a.acc_out == nullptr && a.epi.kind == kEpiGelu;
  if (wide && a.K >= 2560) return launch_bn<256, kEpiStore, true, 8>(a, s);
  if (wide) return gelu ? launch_bn<256, kEpiStore, false, 16>(a, s)
                        : launch_bn<256, kEpiStore, false, 8>(a, s);
  return gelu ? launch_bn<128, kEpiStore, false, 16>(a, s) : launch_bn<128, kEpiStore, false, 8>(a, s);
}

cudaError_t launch_gemm_tf32x3(const GemmTf32Args& a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0) return cudaSuccess;
  if (a.K <= 0 || (a.K & 3) || (a.lda & 3) || (a.ldw & 3) || a.A_lo == nullptr ||
      a.W_lo == nullptr || a.status == nullptr || a.epi.kind == kEpiQkvRope ||
      ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.A_lo) |
        reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.W_lo)) & 15))
    return cudaErrorNotSupported;
  // CTA pairs (M = 256, N = 256) when there are tiles for every pair: each
  // CTA then streams 64 KB per 32 K-elements for 12 full-rate MMAs.
  const long pair_tiles = static_cast<long>((a.M + 255) / 256) * ((a.N + 255) / 256);
  if (a.N >= 256 && pair_tiles >= a.num_sms / 2) return launch_f32<256, true>(a, s);
  return launch_f32<128, false>(a, s);
}

}  // namespace esmb200

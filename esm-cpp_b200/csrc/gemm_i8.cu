// W8A8 INT8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Replaces the reference's LinearVnni / LinearAmx integer core
// (gemm_int8.cpp:232-555, gemm_amx.cpp:146-309) and its FinalizeStore16
// dequant (gemm_int8.cpp:109-126).  The reference quantises activations to
// u8 with zero point 128 and subtracts 128*col_sum afterwards; the tensor
// cores take s8 x s8 directly, which yields the same int32 sum_k q*w.
//
// Structure (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: A [BM x 128] and W [BN x 128] int8 tiles,
//               128-byte swizzle, into a STAGES-deep shared-memory ring.
//   warp 1      TMEM owner + MMA issuer: 4 x (M=128, N=BN, K=32) MMAs per
//               stage into one of two TMEM accumulators (2*BN columns).
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (one output row
//               per thread), dequant fma(float(acc), ws[n]*as, bias[n]),
//               then store / residual / GELU / QKV-split+RoPE.
// The epilogue of tile i overlaps the mainloop of tile i+1.  Every barrier
// wait is bounded; a timeout sets a status bit and the CTA unwinds.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>

#include "common.cuh"
#include "epilogue.cuh"
#include "kernels.cuh"

namespace esmb200 {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int kThreads = 320;    // producer, MMA issuer, 8 epilogue warps
constexpr int kEpiWarps = 8;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 3 : (BN == 128 ? 5 : 7);
  static constexpr int TMEM_COLS = 2 * BN;
  // Epilogue staging for TMA stores: 8 warps x [32 rows x 128 B], then the
  // tile's (w_scale * a_scale) and bias columns shared by the epilogue warps.
  static constexpr int STAGING_BYTES = kEpiWarps * 4096;
  static constexpr int COLVEC_BYTES = 2 * BN * 4;
  static constexpr int SMEM =
      STAGES * STAGE_BYTES + STAGING_BYTES + COLVEC_BYTES + 1024 /*align*/ + 256 /*barriers*/;
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
};

// Named barrier 1 across the kEpiWarps epilogue warps only.
__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}
// The same barrier with an AND-vote: every epilogue warp gets the same answer,
// so a timeout leaves the loop in all of them together (none is left waiting
// at a later barrier).
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "barrier.cta.red.and.pred po, 1, %2, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "n"(kEpiWarps * 32)
      : "memory");
  return r != 0;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC0,
                   const __grid_constant__ CUtensorMap tmC1,
                   const __grid_constant__ CUtensorMap tmC2, const Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* staging = smem + C::STAGES * C::STAGE_BYTES;
  float* colvec = reinterpret_cast<float*>(staging + C::STAGING_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::STAGING_BYTES + C::COLVEC_BYTES);
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
      mbar_init(&tempty[a], kEpiWarps);  // one arrive per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.tma) {
      prefetch_tmap(&tmC0);
      if (EPI == kEpiQkvRope) {
        prefetch_tmap(&tmC1);
        prefetch_tmap(&tmC2);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int m_blocks = (p.M + BM - 1) / BM;
  const int n_blocks = (p.N + BN - 1) / BN;
  const int num_tiles = m_blocks * n_blocks;
  const int num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile % m_blocks;
        const int n_blk = tile / m_blocks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, m_blk * BM);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, n_blk * BN);
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
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
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
            mma_i8(d_tmem, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32), idesc,
                   (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    // Warps 2..9: TMEM lane quadrant warp % 4 (the hardware rule), and the
    // column half `half`: the two warps of a quadrant take alternate chunks.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int etid = (warp - 2) * 32 + lane;  // 0..255 among epilogue threads
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    float amax = 0.0f;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile % m_blocks;
      const int n_blk = tile / m_blocks;
      if (!epi_all(mbar_wait(&tfull[acc], acc_phase, p.status))) break;
      tc_fence_after();
      const long m = static_cast<long>(m_blk) * BM + row_in_tile;
      const bool row_ok = m < p.M;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      float as = 1.0f;  // the raw-accumulator mode carries no activation scale
      if (row_ok && p.acc_out == nullptr) as = p.per_token ? __ldg(p.a_scale + m) : __ldg(p.a_scale);

      // This tile's w_scale / bias columns, copied once into shared memory by
      // the epilogue warps (tail columns read the last valid column).
      float* wsv = colvec;
      float* bsv = colvec + BN;
      // Per-tensor scale: ws[n]*as is the same for every row, so the rounded
      // product (the reference rounds it before the fma) is formed once.
      const float as_col = p.per_token ? 1.0f : (p.acc_out ? 1.0f : __ldg(p.a_scale));
      if (p.acc_out == nullptr) {
        for (int j = etid; j < BN; j += kEpiWarps * 32) {
          const int n = min(n_blk * BN + j, p.N - 1);
          wsv[j] = p.per_token ? __ldg(p.w_scale + n) : __fmul_rn(__ldg(p.w_scale + n), as_col);
          bsv[j] = p.bias ? __ldg(p.bias + n) : 0.0f;
        }
      }
      epi_barrier();  // vectors filled
      // Dequant of one accumulator at tile column jc: fma(float(acc),
      // ws[n]*as, bias[n]) (gemm_int8.cpp:109-126).
      auto deq = [&](uint32_t a, int jc) {
        const float sc = p.per_token ? __fmul_rn(wsv[jc], as) : wsv[jc];
        return __fmaf_rn(__int2float_rn(static_cast<int>(a)), sc, bsv[jc]);
      };
      // This warp's staging buffer and the top row of its 32-row slab.
      uint8_t* stg = staging + (warp - 2) * 4096;
      const int y0 = m_blk * BM + quad * 32;
      // Stage y[0..32) of this thread's row (lane) with the 128-byte swizzle
      // the tensor map expects.
      auto stage32 = [&](uint8_t* buf, const float* y) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(buf + lane * 128 + ((j ^ (lane & 7)) * 16)) =
              make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
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
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = deq(r[j], c * 32 + j);
        if (!p.tma) {
          if (row_ok) amax = fmaxf(amax, epi_row_run<32>(p.epi, m, n0, p.N, y));
          return;
        }
        if (p.epi.kind == kEpiGelu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) y[j] = gelu_erf(y[j]);
        }
        if (row_ok && p.epi.amax != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) amax = fmaxf(amax, fabsf(y[j]));
        }
        if (lane == 0) bulk_wait_read<0>();  // the buffer's last store has read it
        __syncwarp();
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
        for (int c = half; c < BN / 64; c += 2) {
          uint32_t lo[32], hi[32];
          tmem_ld32(t_row + c * 64, lo);
          tmem_ld32(t_row + c * 64 + 32, hi);
          tmem_ld_wait();
          const int n_base = n_blk * BN + c * 64;
          if (n_base < p.N) {  // warp-uniform
            float y[64];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              y[j] = deq(lo[j], c * 64 + j);
              y[32 + j] = deq(hi[j], c * 64 + 32 + j);
            }
            if (p.tma) {
              const int which = n_base / p.epi.d;
              const int col = n_base - which * p.epi.d;
              epi_qkv_rope_values(p.epi, row_ok ? m : 0, which, y);
              const CUtensorMap* mp = which == 0 ? &tmC0 : (which == 1 ? &tmC1 : &tmC2);
#pragma unroll
              for (int half = 0; half < 2; ++half) {
                if (lane == 0) bulk_wait_read<0>();  // the buffer's last store has read it
                __syncwarp();
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
        // This warp's chunks are half, half+2, ...; the TMEM load of the next
        // one runs while the previous one is dequantised and stored.
        constexpr int NC = BN / 64;  // chunks per warp (>= 1)
        uint32_t ra[32], rb[32];
        tmem_ld32(t_row + half * 32, ra);
        tmem_ld_wait();
#pragma unroll 1
        for (int i = 0; i < NC; i += 2) {
          const int c0 = half + 2 * i;
          if (i + 1 < NC) tmem_ld32(t_row + (c0 + 2) * 32, rb);
          epi_chunk(c0, ra);
          tmem_ld_wait();
          if (i + 1 < NC) {
            if (i + 2 < NC) tmem_ld32(t_row + (c0 + 4) * 32, ra);
            epi_chunk(c0 + 2, rb);
            tmem_ld_wait();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      epi_barrier();  // every epilogue warp is done with this tile's vectors
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.epi.amax != nullptr) amax_publish_warp(p.epi.amax, amax);
    if (p.tma && lane == 0) bulk_wait<0>();  // stores done before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// 2-D fp32 tensor [rows, cols] with row stride `ld` floats; box = 32 x 32
// (128-byte rows, 128-byte swizzle) for the epilogue's TMA stores.
bool make_tmap_f32(CUtensorMap* map, const float* base, long rows, long cols, long ld) {
  auto fn = get_encode_fn();
  if (fn == nullptr || base == nullptr || (ld & 3) || (reinterpret_cast<uintptr_t>(base) & 15))
    return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
cudaError_t launch_bn(const GemmI8Args& a, cudaStream_t s) {
  using C = Cfg<BN>;
  CUtensorMap tmA, tmB, tmC[3];
  if (!make_tmap_i8(&tmA, a.A, a.M, a.K, a.lda, BM)) return cudaErrorInvalidValue;
  if (!make_tmap_i8(&tmB, a.W, a.N, a.K, a.ldw, BN)) return cudaErrorInvalidValue;
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
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<BN, EPI>,
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
  const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN);
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  gemm_i8_kernel<BN, EPI><<<grid, kThreads, C::SMEM, s>>>(tmA, tmB, tmC[0], tmC[1], tmC[2], p);
  return cudaGetLastError();
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
    if (a.epi.d % 256 == 0) return launch_bn<256, kEpiQkvRope>(a, s);
    if (a.epi.d % 64 == 0) return launch_bn<64, kEpiQkvRope>(a, s);
    return cudaErrorInvalidValue;
  }
  // Wide tiles when N is large, narrower ones to fill the SMs otherwise.
  const long tiles256 = ((a.M + BM - 1) / BM) * static_cast<long>((a.N + 255) / 256);
  const bool wide = a.N >= 256 && tiles256 >= a.num_sms;
  if (wide) return launch_bn<256, kEpiStore>(a, s);  // epilogue kind is a runtime field
  return launch_bn<128, kEpiStore>(a, s);
}

}  // namespace esmb200

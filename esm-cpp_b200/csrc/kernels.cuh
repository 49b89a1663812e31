// Internal launcher API of the sm_100a kernels.  The C-ABI layer (capi.cu)
// and nothing else calls these; every pointer is a device pointer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace esmb200 {

// Launch attribute of the forward's kernels: programmatic stream
// serialisation (the kernel calls pdl_wait() before touching global memory,
// common.cuh), so its launch and setup overlap the previous kernel's tail.
inline cudaLaunchAttribute pdl_attribute() {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}

// kernel<<<grid, block, smem, s>>>(args...) with the PDL attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1] = {pdl_attribute()};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// A per-tensor absmax lives in kAmaxSlots uint32 slots (float bits): each
// producer block folds its maximum into slot (blockIdx.x % kAmaxSlots) and the
// consumer takes the max over the slots.  Spreading the atomics over 64
// addresses keeps thousands of blocks from serialising on one L2 line.
constexpr int kAmaxSlots = 64;

// Epilogue applied to a finished fp32 output tile (after dequant for the
// INT8 GEMM, after bias for the FP32 GEMM).
enum EpiKind : int {
  kEpiStore = 0,    // C[m,n] = y
  kEpiResidual = 1, // C[m,n] = C[m,n] + y           (hidden += proj)
  kEpiGelu = 2,     // C[m,n] = gelu(y)
  kEpiQkvRope = 3,  // y -> q|k|v split, q *= q_scale, RoPE(q,k) at pos[m]
};

struct EpiParams {
  int kind = kEpiStore;
  float* C = nullptr;
  long ldc = 0;
  // When non-null, max|stored value| over the tensor is folded into the
  // kAmaxSlots slots at amax.  Feeds the next GEMM's per-tensor scale.
  uint32_t* amax = nullptr;
  // kEpiQkvRope: the output columns [0,d) | [d,2d) | [2d,3d) go to q | k | v,
  // each [M, d] with row stride d; head_dim must be 64.
  float* q = nullptr;
  float* k = nullptr;
  float* v = nullptr;
  int d = 0;
  const int* pos = nullptr;      // [M] position of each token in its sequence
  const float* cos_t = nullptr;  // [max_len, 64]
  const float* sin_t = nullptr;
  float q_scale = 1.0f;
  // kEpiQkvRope: q and k stored rounded to bf16 (round to nearest even), the
  // opt-in BF16 attention of the reference (ESM_AMX_ATTENTION).
  int qk_bf16 = 0;
};

// ---------------------------------------------------------------- INT8 GEMM
// C = epilogue( fma(float(A_q8 . W_q8^T), w_scale[n] * a_scale, bias[n]) )
// A: [M, K] int8 row stride lda (bytes); W: [N, K] int8 row stride ldw.
// K, lda, ldw must be multiples of 16 and the pointers 16-byte aligned.
// a_scale: one float (per_token == 0) or M floats (per_token == 1).
struct GemmI8Args {
  const int8_t* A = nullptr;
  long lda = 0;
  const int8_t* W = nullptr;
  long ldw = 0;
  int M = 0, N = 0, K = 0;
  const float* w_scale = nullptr;
  const float* a_scale = nullptr;
  int per_token = 0;
  const float* bias = nullptr;
  EpiParams epi;
  uint32_t* status = nullptr;
  int num_sms = 148;
  // Debug/test: write the raw int32 accumulators [M, N] here instead of
  // running the epilogue.
  int32_t* acc_out = nullptr;
};
cudaError_t launch_gemm_i8(const GemmI8Args& a, cudaStream_t s);

// ---------------------------------------------------------------- FP32 GEMM
// C = epilogue( A[M,K] . W[N,K]^T + bias ), FP32 SIMT.
struct GemmF32Args {
  const float* A = nullptr;
  long lda = 0;
  const float* W = nullptr;
  long ldw = 0;
  int M = 0, N = 0, K = 0;
  const float* bias = nullptr;
  EpiParams epi;
};
cudaError_t launch_gemm_f32(const GemmF32Args& a, cudaStream_t s);

// The same product on the tensor cores, 3xTF32 (tcgen05 kind::tf32):
// C = epilogue( A W^T + A W_lo^T + A_lo W^T + bias ), where x_lo = x - tf32(x)
// (launch_tf32_lo) is given for both operands.  FP32-accurate to about 2^-21
// relative per product.  K, lda, ldw multiples of 4, operands 16-byte
// aligned; cudaErrorNotSupported otherwise (and for the QKV epilogue).
struct GemmTf32Args {
  const float* A = nullptr;
  const float* A_lo = nullptr;
  long lda = 0;
  const float* W = nullptr;
  const float* W_lo = nullptr;
  long ldw = 0;
  int M = 0, N = 0, K = 0;
  const float* bias = nullptr;
  EpiParams epi;
  uint32_t* status = nullptr;
  int num_sms = 148;
};
cudaError_t launch_gemm_tf32x3(const GemmTf32Args& a, cudaStream_t s);
// lo[i] = x[i] - (x[i] with its low 13 mantissa bits cleared), i < n.
cudaError_t launch_tf32_lo(const float* x, float* lo, long n, cudaStream_t s);

// ------------------------------------------------------------ quantisation
// Per-tensor: scale = amax>0 ? amax/127 : 1 (amax = max over the kAmaxSlots
// slots at amax_bits);
// q = clamp(rne(x * (1/scale)), +-127); writes *scale_out; pads columns
// [K, ldq) of each row with zeros.
cudaError_t launch_quantize_per_tensor(const float* x, long ldx, int M, int K,
                                       const uint32_t* amax_bits, int8_t* q, long ldq,
                                       float* scale_out, cudaStream_t s);
// Per-token: one scale per row computed from that row's absmax.
cudaError_t launch_quantize_per_token(const float* x, long ldx, int M, int K, int8_t* q,
                                      long ldq, float* row_scales, cudaStream_t s);
cudaError_t launch_absmax(const float* x, long n, uint32_t* amax_bits, cudaStream_t s);
// quant::Quantize of weights W [N, K] (dense rows) -> q [N, K] int8 in rows
// of stride ldq >= K bytes (bytes past K untouched) and per-row scales [N].
cudaError_t launch_quantize_weights(const float* W, int N, int K, int8_t* q, long ldq,
                                    float* scale, cudaStream_t s);
// x = float(half(x)) in place (round to nearest even); optional absmax of the
// rounded values into amax_bits.
cudaError_t launch_round_fp16(float* x, long n, uint32_t* amax_bits, cudaStream_t s);

// --------------------------------------------------------------- LayerNorm
// out = LN(x) with the reference's rounding (double sums, float normalise).
// Optional absmax of out into *amax.  When q != nullptr the row is also (or
// only, if out == nullptr) quantised per token into q / row_scales.
cudaError_t launch_layernorm(const float* x, const float* g, const float* b, float eps,
                             float* out, int rows, int d, uint32_t* amax, int8_t* q,
                             long ldq, float* row_scales, cudaStream_t s);

// LayerNorm fused with the per-tensor int8 quantisation of its output; the
// fp32 output is never written.  Phase 1 computes every row's statistics
// (into stats [rows]) and the absmax of y (into the kAmaxSlots slots of
// amax, zeroed by the caller); after a grid-wide barrier (cooperative launch;
// *counter must be zero, one counter per launch) phase 2 recomputes y with
// the same arithmetic and writes q [rows x ldq] (columns >= d zeroed) and
// *scale_out = max(absmax/127, or 1 if 0).  Returns cudaErrorNotSupported for
// widths other than d = 128 k (k <= 16) or unaligned buffers; callers then
// use launch_layernorm + launch_quantize_per_tensor.
cudaError_t launch_layernorm_quant(const float* x, const float* g, const float* b, float eps,
                                   int rows, int d, uint32_t* amax, float2* stats,
                                   uint32_t* counter, int8_t* q, long ldq, float* scale_out,
                                   uint32_t* status, cudaStream_t s);

// --------------------------------------------------------------- attention
// Packed-varlen attention, q pre-scaled and RoPE'd; q,k,v,out [T, H, dh].
// T = cu[B], min_len / max_len = shortest / longest sequence (host-known).
// Optional absmax of out into *amax.  head_dim 64 runs on the tensor cores
// (needs the status word): one CTA per (sequence, head) for L <= 128, a CTA
// pair for 128 < L <= 256, one CTA per (sequence, head, 128-row query tile)
// above; other head dims on FP32 SIMT.  qk_bf16: q and k hold bf16 values
// (launch_round_bf16), so S needs no lo terms on the tensor cores.
cudaError_t launch_attention_varlen(const float* q, const float* k, const float* v,
                                    const int* cu, int B, int H, int dh, long T, int min_len,
                                    int max_len, float* out, uint32_t* amax, uint32_t* status,
                                    int num_sms, cudaStream_t s, bool qk_bf16 = false);

// ------------------------------------------------------------- elementwise
cudaError_t launch_gelu(const float* x, float* out, long n, cudaStream_t s);
cudaError_t launch_residual_add(float* y, const float* x, long n, cudaStream_t s);
cudaError_t launch_scale(float* x, long n, float scale, cudaStream_t s);
cudaError_t launch_rope_varlen(float* x, const float* cos_t, const float* sin_t,
                               const int* cu, int B, int H, int dh, cudaStream_t s);
// qkv [T, 3d] -> q, k, v [T, d]; q *= q_scale; RoPE on q and k.
cudaError_t launch_split_qkv_rope(const float* qkv, float* q, float* k, float* v, int T,
                                  int d, int H, int dh, const int* pos, const float* cos_t,
                                  const float* sin_t, float q_scale, cudaStream_t s,
                                  bool qk_bf16 = false);
// y = float(bf16(x)), round to nearest even (y may equal x).
cudaError_t launch_round_bf16(const float* x, float* y, long n, cudaStream_t s);
// Token -> position inside its sequence, from cu_seqlens.
cudaError_t launch_positions(const int* cu, int B, int* pos, cudaStream_t s);
// out [R, d] = x[rows[r]] (rows must index rows of x).
cudaError_t launch_gather_rows(const float* x, const int* rows, int R, int d, float* out,
                               cudaStream_t s);
// In-place log-softmax of each row of x [R, V].
cudaError_t launch_log_softmax_rows(float* x, int R, int V, cudaStream_t s);
// model.cpp:737-778 Embed.
cudaError_t launch_embed(const float* embed_w, int d, const int* ids, const int* masks,
                         const int* cu, int B, int mask_id, float* out, cudaStream_t s);

// ---------------------------------------------- reference-rounding mode
// The reference's default x86 kernels bit for bit (refmath.cu).
// LayerNormAvx512: d % 16 == 0; amax (nullable) gets max|y|.
cudaError_t launch_layernorm_avx(const float* x, const float* g, const float* b, float eps,
                                 float* out, int rows, int d, uint32_t* amax, cudaStream_t s);
// GeluAvx512 over n values (in place allowed); amax (nullable) gets max|y|.
cudaError_t launch_gelu_avx(const float* x, float* y, long n, uint32_t* amax, cudaStream_t s);
// AttentionVarlenAvx512, q/k/v/out [T, H, dh], dh in {16, 32, 64}; max_len
// = the longest sequence; amax (nullable) gets max|out|.
cudaError_t launch_attention_avx(const float* q, const float* k, const float* v, const int* cu,
                                 int B, int H, int dh, int T, int max_len, float* out,
                                 uint32_t* amax, cudaStream_t s);

// ---------------------------------------------- on-device weight preparation
// (prep.cu) The SmoothQuant migration's element steps on FP32 weights.
// out[k] = max_n |W[n, k]| as float bits (out is zeroed first).
cudaError_t launch_col_absmax(const float* W, int N, int K, uint32_t* out, cudaStream_t s);
// W[n, k] *= scales[k].
cudaError_t launch_mul_cols(float* W, long N, int K, const float* scales, cudaStream_t s);
// W[n, k] /= scales[n] and bias[n] /= scales[n] (bias nullable).
cudaError_t launch_div_rows(float* W, long N, int K, float* bias, const float* scales,
                            cudaStream_t s);
// x[i] /= scales[i], y[i] /= scales[i].
cudaError_t launch_div_vec2(float* x, float* y, int n, const float* scales, cudaStream_t s);

}  // namespace esmb200

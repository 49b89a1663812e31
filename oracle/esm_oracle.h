/* CPU restatement of the reference esm.cpp hot path (packed-varlen ESM-2
 * encoder, W8A8 per-tensor SmoothQuant INT8) -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker.  The product path
 * (esm-cpp_b200/) never calls it.
 *
 * Parity is pinned: tests/test_oracle_pins.py checks every function here
 * against the reference compiled from its own sources (oracle/_ref/) and
 * against the known-answer values of the reference's own unit tests.
 */
#ifndef ESM_ORACLE_H
#define ESM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* pack.cpp:149-177 */
void orc_quantize_weights(const float* W, int N, int K, int8_t* q, float* scales);
/* gemm_int8.cpp:391-508 (absmax pass) */
float orc_absmax(const float* x, size_t n);
/* gemm_int8.cpp:479 (amax>0 ? amax/127 : 1) */
float orc_act_scale(float amax);
/* gemm_int8.cpp:415-426 vector path: clamp(rne(x*(1/s)),+-127), s8 form */
void orc_quantize_act(const float* x, size_t n, float scale, int8_t* q);
/* Per-token mode: one scale per row, each row quantised as above. */
void orc_quantize_act_per_token(const float* x, int M, int K, int8_t* q, float* row_scales);
/* Exact int32 dot over int8 operands: acc[m,n] = sum_k q[m,k]*w[n,k]. */
void orc_gemm_i8_s32(const int8_t* q, const int8_t* w, int32_t* acc, int M, int N, int K);
/* gemm_int8.cpp:109-126: C = fma(float(acc), ws[n]*as, bias[n]).
 * row_scales != NULL selects per-token scales (as = row_scales[m]). */
void orc_dequant(const int32_t* acc, const float* ws, float act_scale,
                 const float* row_scales, const float* bias, float* C, int M, int N);
/* gemm_fp32.cpp:33-46 (LinearRef). */
void orc_linear_f32(const float* A, const float* W, const float* bias, float* C,
                    int M, int N, int K);
/* layernorm.cpp:23-43 (LayerNormRef, double accumulation). */
void orc_layernorm(const float* x, const float* g, const float* b, float eps,
                   float* out, int rows, int d);
/* gelu.cpp:30-35 (GeluRef, erf form). */
void orc_gelu(const float* x, float* out, size_t n);
/* residual.cpp:23-29. */
void orc_residual_add(float* y, const float* x, size_t n);
void orc_scale(float* x, size_t n, float s);
/* rope_tables.cpp:14-29. */
void orc_rope_build_tables(int L, int dh, float* cos_t, float* sin_t);
/* rope.cpp:47-70 (fused=0, the Ref form) and rope.cpp:90-152 (fused=1, the
 * AVX-512 form: lo' = fma(-hi, s, lo*c), hi' = fma(hi, c, lo*s)). */
void orc_rope_apply_varlen(float* x, const float* cos_t, const float* sin_t,
                           const int* cu, int B, int H, int dh, int fused);
/* attention.cpp:99-144 (AttentionVarlenRef: FP32 dots, exp, double sum). */
void orc_attention_varlen(const float* q, const float* k, const float* v,
                          const int* cu, int B, int H, int dh, float* out);
/* model.cpp:737-778 (Embed with per-sequence token-dropout rescale). */
void orc_embed(const float* embed_w, int d, const int* ids, const int* masks,
               const int* cu, int B, int mask_id, float* out);
/* scheduler.cpp:13-75 (PlanBatches): writes caller indices in plan order and
 * the size of every group; returns the group count. */
int orc_plan_batches(const int* lengths, int n, float threshold, int max_batch,
                     int* order_out, int* group_sizes_out);

/* The reference's default x86 kernels, bit for bit (esm_oracle_avx.c). */
/* layernorm.cpp:59-149 LayerNormAvx512, d % 16 == 0 */
void orc_layernorm_avx(const float* x, const float* g, const float* b, float eps, float* out,
                       int rows, int d);
/* gelu.cpp:48-148 GeluAvx512 */
void orc_gelu_avx(const float* x, float* out, size_t n);
/* the C library's expf (used by AttentionVarlenAvx512 past whole 16-key blocks) */
float orc_expf_libc(float x);
/* attention.cpp:230-437, 770-811 AttentionVarlenAvx512, head_dim % 16 == 0,
 * scratch of max_len floats */
void orc_attention_avx(const float* q, const float* k, const float* v, const int* cu, int B,
                       int H, int dh, float* out, float* scratch);

#ifdef __cplusplus
}
#endif
#endif

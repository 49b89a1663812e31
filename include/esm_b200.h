/* esm_b200: B200-native (sm_100a) packed-varlen ESM-2 encoder forward,
 * W8A8 SmoothQuant INT8 -- the C-ABI drop-in boundary.
 *
 * Two layers of entry points, both plain C (no C++ or torch types):
 *
 *  1. Kernel facade (device pointers, enqueued on the context's stream).
 *     One function per function of the reference's kernel facade
 *     include/esm_cpp/kernels.h, same argument order and meaning, plus a
 *     context and an int status.  The reference's versions take host
 *     pointers; these take device pointers, because the device-resident
 *     forward never round-trips activations through the host.
 *
 *  2. Model (host buffers in, host buffers out).  Mirrors esm::Model's
 *     ForwardPacked / ForwardScheduled (include/esm_cpp/model.h:136-159)
 *     on a per-device weight replica; the host side keeps the reference's
 *     BatchView validation and PlanBatches packing.
 *
 * Every function returns an esmcu_status; esmcu_last_error() gives the
 * message of the calling thread's last failure.  No C++ exception crosses
 * this boundary.  A context serves one host thread at a time, like
 * esm::Model (model.h:179-181: one forward in flight per instance).
 */
#ifndef ESM_B200_H
#define ESM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The first seven values mirror esm::StatusCode (include/esm_cpp/status.h:9-17). */
typedef enum {
  ESMCU_OK = 0,
  ESMCU_ERR_INVALID_ARGUMENT = 1,
  ESMCU_ERR_OUT_OF_RANGE = 2,
  ESMCU_ERR_NOT_FOUND = 3,
  ESMCU_ERR_IO = 4,
  ESMCU_ERR_SHAPE_MISMATCH = 5,
  ESMCU_ERR_INTERNAL = 6,
  ESMCU_ERR_CUDA = 7,    /* a CUDA runtime call failed */
  ESMCU_ERR_TIMEOUT = 8, /* a device-side bounded wait ran out */
  ESMCU_ERR_NO_DEVICE = 9
} esmcu_status;

/* Activation quantisation of the W8A8 GEMMs. */
typedef enum {
  /* Reference semantics: one dynamic scale max|A|/127 over the whole packed
   * operand (gemm_int8.cpp:391-508).  Bit-exact int8/int32 parity mode. */
  ESMCU_ACT_PER_TENSOR = 0,
  /* One scale per token row (QuantizeActivationSymmetricRef per row,
   * pack.cpp:134-147). */
  ESMCU_ACT_PER_TOKEN = 1
} esmcu_act_quant;

typedef struct esmcu_context esmcu_context;
typedef struct esmcu_model esmcu_model;

const char* esmcu_last_error(void);
const char* esmcu_version(void);
int esmcu_device_count(int* count);

/* ---- context ----------------------------------------------------------- */
int esmcu_open(int device, esmcu_context** out);
int esmcu_close(esmcu_context* ctx);
/* Use an existing cudaStream_t (passed as void*); NULL = the context's own. */
int esmcu_set_stream(esmcu_context* ctx, void* cuda_stream);
void* esmcu_get_stream(esmcu_context* ctx);
/* Waits for the stream and reports device-side failures (timeouts). */
int esmcu_synchronize(esmcu_context* ctx);
/* Arithmetic of the LayerNorm, GELU and attention kernels (facade calls and
 * the forwards of models on this context).
 *   ESMCU_MATH_DEFAULT  the tensor-core / fused kernels, within the FP32
 *                       class of the reference's scalar twins.
 *   ESMCU_MATH_AVX512   the reference's default x86 kernels bit for bit:
 *                       LayerNormAvx512 (layernorm.cpp:59-149), GeluAvx512
 *                       (gelu.cpp:48-148) and AttentionVarlenAvx512
 *                       (attention.cpp:230-437, 770-811) as its release build
 *                       rounds them; with the INT8 GEMMs already exact, a W8A8
 *                       forward then reproduces the reference's default path
 *                       layer by layer.  SIMT kernels, several times slower;
 *                       needs hidden and head dims that are multiples of 16
 *                       (head_dim 16, 32 or 64); the FP32 attention form
 *                       (ESM_AMX_ATTENTION is not applied in this mode). */
typedef enum { ESMCU_MATH_DEFAULT = 0, ESMCU_MATH_AVX512 = 1 } esmcu_math_mode;
int esmcu_set_math_mode(esmcu_context* ctx, int mode);
int esmcu_get_math_mode(const esmcu_context* ctx, int* mode);
/* Failure-detection self-test; no counterpart in the reference, which has no
 * device waits.  Runs one small kernel whose mbarrier waits can never
 * complete (one of two expected arrivals is made) and must give up after
 * limit_us microseconds (0 < limit_us <= 1e6) through the same bounded-wait
 * code every kernel here uses.  Returns ESMCU_ERR_TIMEOUT when they did, with
 * *waiters_released = the number of waiting threads that gave up (4), and
 * leaves the context usable. */
int esmcu_bounded_wait_selftest(esmcu_context* ctx, int limit_us, int* waiters_released);
/* Device memory helpers for C callers without another allocator. */
int esmcu_malloc(esmcu_context* ctx, size_t bytes, void** dptr);
int esmcu_free(esmcu_context* ctx, void* dptr);
int esmcu_memcpy_h2d(esmcu_context* ctx, void* dst, const void* src, size_t bytes);
int esmcu_memcpy_d2h(esmcu_context* ctx, void* dst, const void* src, size_t bytes);

/* ---- kernel facade (device pointers) ------------------------------------
 * Each replaces the esm::kernels function named in its comment. */

/* kernels.h:19-20 Linear: C[M,N] = A[M,K] . W[N,K]^T + bias (bias nullable).
 * FP32-accurate: 3xTF32 on the tensor cores when K % 4 == 0 and A, W are
 * 16-byte aligned (the lo parts of A and W, 4*(M+N)*K bytes, go to the
 * context's scratch, which grows on demand), FP32 SIMT otherwise. */
int esmcu_linear(esmcu_context* ctx, const float* A, const float* W, const float* bias,
                 float* C, int M, int N, int K);

/* kernels.h:56-57 LinearInt8 (W8A8): W is QuantizedTensor::packed [N,K]
 * int8 with per_channel_scales w_scales [N] (quant.h:17-23).  Activations are
 * quantised on the device per esmcu_act_quant, accumulated in int32 and
 * dequantised as fma(float(acc), w_scales[n]*a_scale, bias[n])
 * (gemm_int8.cpp:109-126). */
int esmcu_linear_int8(esmcu_context* ctx, const float* A, const int8_t* W,
                      const float* w_scales, const float* bias, float* C, int M, int N, int K,
                      int act_quant);

/* No counterpart in the reference.  esmcu_linear_int8 without any device
 * allocation, for callers that cannot let the library call cudaMalloc (a
 * process whose HBM is all handed to its own pool, or one that cannot take
 * the synchronisation an allocation implies).  Same arguments, checks and
 * results; its scratch is one fixed 16 MiB array per device, built into the
 * library, so 256 + 4*M (to 256) + M*ldq bytes, plus N*ldq when K % 16 != 0
 * or W is not 16-byte aligned, must fit, ldq = K rounded up to 16, else
 * ESMCU_ERR_OUT_OF_RANGE.  All calls on a device share that array: calls
 * that overlap on the GPU race.  esmcu_open loads the array onto its device
 * (the driver commits the 16 MiB then), so the first call allocates
 * nothing; open the context before handing HBM to a pool. */
int esmcu_linear_int8_noalloc(esmcu_context* ctx, const float* A, const int8_t* W,
                              const float* w_scales, const float* bias, float* C, int M, int N,
                              int K, int act_quant);

/* The two halves of LinearInt8, exposed for the bit-exact parity gates.
 * esmcu_quantize_activations: QuantizeActPrefixAvx512 (gemm_int8.cpp:391-508)
 * in its symmetric s8 form q = clamp(rne(A*(1/s)), +-127), q_out [M, ldq]
 * (ldq >= K, a multiple of 16; columns [K, ldq) are zeroed); scales_out gets
 * 1 (per tensor) or M (per token) floats.
 * esmcu_gemm_int8_s32: acc[M,N] = sum_k q[m,k]*W[n,k] in int32 on the
 * tensor cores (K, ldq, ldw multiples of 16). */
int esmcu_quantize_activations(esmcu_context* ctx, const float* A, int M, int K, int8_t* q_out,
                               int ldq, float* scales_out, int act_quant);
int esmcu_gemm_int8_s32(esmcu_context* ctx, const int8_t* q, int ldq, const int8_t* W, int ldw,
                        int32_t* acc, int M, int N, int K);
/* quant::Quantize (quant.h:17-56; pack.cpp:149-177) on the device: W [N, K]
 * fp32 (dense rows) -> q [N, K] int8 and per-output-channel scales [N],
 * scale = max|row| / 127, q = clamp(rne(w * (1/scale)), +-127), an all-zero
 * row scale 0; bit-identical to the reference.  Asynchronous on the context
 * stream, device pointers. */
int esmcu_quantize_weights(esmcu_context* ctx, const float* W, int N, int K, int8_t* q,
                           float* scales);

/* kernels.h:32-33 LayerNorm over rows of width d. */
int esmcu_layernorm(esmcu_context* ctx, const float* x, const float* gamma, const float* beta,
                    float eps, float* out, int num_rows, int d);
/* kernels.h:35 Gelu (exact erf form). */
int esmcu_gelu(esmcu_context* ctx, const float* x, float* out, size_t n);
/* kernels.h:24 ResidualAddInplace: y += x. */
int esmcu_residual_add_inplace(esmcu_context* ctx, float* y, const float* x, size_t n);
/* kernels.h:29 ScaleInplace: x *= scale. */
int esmcu_scale_inplace(esmcu_context* ctx, float* x, size_t n, float scale);
/* kernels.h:73 RopeBuildTables: pure host function, host buffers
 * cos/sin [seq_len, head_dim] (rope_tables.cpp:14-29). */
int esmcu_rope_build_tables(int seq_len, int head_dim, float* cos_out, float* sin_out);
/* kernels.h:90-92 RopeApplyVarlen: x [T, H, dh] in place, positions restart
 * at every cu_seqlens boundary. */
int esmcu_rope_apply_varlen(esmcu_context* ctx, float* x, const float* cos_t,
                            const float* sin_t, const int* cu_seqlens, int batch_size,
                            int num_heads, int head_dim);
/* kernels.h:119-121 AttentionVarlen: q (pre-scaled, RoPE'd), k, v, out
 * [T, H, dh]; per-sequence softmax attention over cu_seqlens.  With
 * ESM_AMX_ATTENTION=on and head_dim % 32 == 0, q and k are rounded to bf16
 * first, in scratch (attention.cpp:686-700); the inputs are not modified. */
int esmcu_attention_varlen(esmcu_context* ctx, const float* q, const float* k, const float* v,
                           const int* cu_seqlens, int batch_size, int num_heads, int head_dim,
                           float* out);

/* ---- host-side packing (scheduler.h:29-30, batch.h:28-31) ---------------- */
/* PlanBatches: writes every caller index once, group after group, into
 * order_out[n] and each group's size into group_sizes_out; returns the
 * group count (>= 0) or -1. */
int esmcu_plan_batches(const int* lengths, int n, float imbalance_threshold,
                       int max_batch_size, int* order_out, int* group_sizes_out);
/* BatchView validation: ESMCU_OK or ESMCU_ERR_INVALID_ARGUMENT with the
 * reference's message. n_masks is 0 (all tokens real) or T. */
int esmcu_batch_view_check(int T, int n_masks, const int* cu_seqlens, int n_cu,
                           int batch_size);

/* ---- model --------------------------------------------------------------- */
typedef struct {
  int num_layers;
  int hidden_size;
  int num_heads;
  int head_dim;
  int intermediate_size;
  int vocab_size;
  float layer_norm_eps;
  int mask_token_id;
  int weights_quantized; /* 1: W8A8 Linears (Q8_ESM weights); 0: FP32 */
  int act_quant;         /* esmcu_act_quant */
} esmcu_config;

/* Host pointers to one encoder layer (LayerWeights, model.h:50-85).  FP32
 * Linear weights [out, in] for an unquantised model; int8 [out, in] plus
 * per-output-channel scales for a quantised one.  Biases and LN are FP32. */
typedef struct {
  const float *attn_ln_w, *attn_ln_b;
  const float *q_w, *k_w, *v_w, *out_w, *fc1_w, *fc2_w;
  const int8_t *q_wq, *k_wq, *v_wq, *out_wq, *fc1_wq, *fc2_wq;
  const float *q_ws, *k_ws, *v_ws, *out_ws, *fc1_ws, *fc2_ws;
  const float *q_b, *k_b, *v_b, *out_b, *fc1_b, *fc2_b;
  const float *ffn_ln_w, *ffn_ln_b;
} esmcu_layer_weights;

/* Caller-owned host buffers to read one layer back into
 * (esmcu_model_get_layer): the same fields as esmcu_layer_weights; null
 * fields are skipped. */
typedef struct {
  float *attn_ln_w, *attn_ln_b;
  float *q_w, *k_w, *v_w, *out_w, *fc1_w, *fc2_w;
  int8_t *q_wq, *k_wq, *v_wq, *out_wq, *fc1_wq, *fc2_wq;
  float *q_ws, *k_ws, *v_ws, *out_ws, *fc1_ws, *fc2_ws;
  float *q_b, *k_b, *v_b, *out_b, *fc1_b, *fc2_b;
  float *ffn_ln_w, *ffn_ln_b;
} esmcu_layer_buffers;

/* Allocates the per-device replica on ctx's device. */
int esmcu_model_create(esmcu_context* ctx, const esmcu_config* cfg, esmcu_model** out);
int esmcu_model_destroy(esmcu_model* m);
int esmcu_model_config(const esmcu_model* m, esmcu_config* out);
/* Uploads (copies) weights; the host buffers may be freed afterwards. */
int esmcu_model_set_embeddings(esmcu_model* m, const float* embed /* [V, d] */);
int esmcu_model_set_layer(esmcu_model* m, int layer, const esmcu_layer_weights* w);
int esmcu_model_set_head(esmcu_model* m, const float* final_ln_w, const float* final_ln_b,
                         const float* lm_dense_w, const float* lm_dense_b,
                         const float* lm_ln_w, const float* lm_ln_b,
                         const float* lm_decoder_bias);
/* lm_head.dense as INT8 (Config::lm_head_dense_quantized, model.h:43-47;
 * set by QuantizeWeights under ESM_QUANTIZE_LM_HEAD, model.cpp:1487-1492):
 * per-channel int8 [d, d] (row-major, rows of d bytes) and scales [d]; the
 * forward then runs LinearInt8 for it (model.cpp:1209-1211) with the
 * model's activation quantisation.  NULL lm_dense_wq restores the FP32
 * dense set by esmcu_model_set_head. */
int esmcu_model_set_head_int8(esmcu_model* m, const int8_t* lm_dense_wq, const float* lm_dense_ws);
/* Config::first_block_fc1_fp16 (model.h:38-41; GGUF key
 * esm.first_block_fc1_fp16): nonzero rounds layer 0's fc1 input to fp16
 * precision, round to nearest even, before its Linear (model.cpp:1031-1033). */
int esmcu_model_set_first_block_fc1_fp16(esmcu_model* m, int enabled);
/* Model::ForwardPacked (model.cpp:1093-1255): host ids [T], masks [T] or
 * NULL, cu_seqlens [B+1] -> host logits [T, V] in packed order.  T == 0
 * writes nothing. */
int esmcu_model_forward_packed(esmcu_model* m, const int32_t* ids, const int32_t* masks, int T,
                               const int32_t* cu_seqlens, int batch_size, float* logits);

/* Model::ForwardWithHiddenStates (model.h:185-191) on a packed batch, the
 * hidden_packed_out of ForwardPackedInto (model.cpp:1142-1189): host
 * hidden_out [num_layers + 1, T, hidden_size] receives the embedding output,
 * each layer's output and, last, the final LayerNorm's output (in place of
 * the last layer's); logits [T, V] as esmcu_model_forward_packed, or NULL. */
int esmcu_model_forward_hidden_states(esmcu_model* m, const int32_t* ids, const int32_t* masks,
                                      int T, const int32_t* cu, int B, float* logits,
                                      float* hidden_out);
/* Model::ForwardScheduled (model.cpp:1298-1421): n sequences concatenated in
 * ids_concat with lengths lens[n] (masks_concat NULL = all real) -> logits
 * concatenated in caller order [sum(lens), V]. */
int esmcu_model_forward_scheduled(esmcu_model* m, const int32_t* ids_concat,
                                  const int32_t* lens, const int32_t* masks_concat, int n,
                                  float imbalance_threshold, int max_batch_size, float* logits);
/* The masked-marginal head of score_assay (python/esm_cpp/eval/proteingym.py:
 * 75-98): the scheduled forward of n sequences (as esmcu_model_forward_scheduled)
 * with the LM head run only on row rows[i] of sequence i (0 <= rows[i] <
 * lens[i], else ESMCU_ERR_OUT_OF_RANGE); log_probs [n, V] receives the
 * log-softmax of those rows, (x - max) - log(sum(exp(x - max))). */
int esmcu_model_masked_marginals(esmcu_model* m, const int32_t* ids_concat, const int32_t* lens,
                                 const int32_t* masks_concat, const int32_t* rows, int n,
                                 float imbalance_threshold, int max_batch_size, float* log_probs);
/* The same forward on device buffers, asynchronous on the context stream:
 * d_ids [T] (and d_masks [T] or NULL) already on the device, host cu_seqlens
 * [B+1] (validated on the host), d_logits [T, V] on the device.  Call
 * esmcu_synchronize to wait and collect device-side failures. */
int esmcu_model_forward_packed_device(esmcu_model* m, const int32_t* d_ids,
                                      const int32_t* d_masks, int T, const int32_t* cu_seqlens,
                                      int batch_size, float* d_logits);
/* ForwardScheduled over several per-device replicas (one host thread each):
 * groups from PlanBatches go to devices by longest-processing-time on the
 * cost sum(24*d^2*L + 4*d*L^2); logits come back in caller order. */
int esmcu_forward_scheduled_multi(esmcu_model** models, int n_models, const int32_t* ids_concat,
                                  const int32_t* lens, const int32_t* masks_concat, int n,
                                  float imbalance_threshold, int max_batch_size, float* logits);
/* ---- calibration (ActivationObserver, observer.h:14-44) ----------------
 * esmcu_observer is the reference's per-site reservoir observer: each site
 * keeps at most 65536 |values| by Algorithm R with its own std::mt19937
 * seeded 0xc1b1ce (observer.cpp:8-31), so the same values observed in the
 * same order keep the same sample as the reference; percentiles index the
 * sorted sample as observer.cpp:33-51 does.  Sites are listed in the order
 * they were first observed. */
typedef struct esmcu_observer esmcu_observer;
int esmcu_observer_create(esmcu_observer** out);
int esmcu_observer_destroy(esmcu_observer* obs);
/* ActivationObserver::Clear (observer.cpp:53). */
int esmcu_observer_clear(esmcu_observer* obs);
/* ActivationObserver::Observe (observer.cpp:8-31) on n host values. */
int esmcu_observer_observe(esmcu_observer* obs, const char* site_key, const float* values,
                           size_t n);
int esmcu_observer_num_sites(const esmcu_observer* obs);
/* Site i: its key (valid until the observer changes), its pctile-th
 * percentile and how many values it has seen (each nullable). */
int esmcu_observer_site(esmcu_observer* obs, int i, float pctile, const char** key,
                        float* value, size_t* total_seen);
/* ActivationObserver::Percentile (observer.cpp:33-51) of one site;
 * ESMCU_ERR_NOT_FOUND when the site was never observed. */
int esmcu_observer_percentile(esmcu_observer* obs, const char* site_key, float pctile,
                              float* value);
/* Model::ForwardWithObserver (model.cpp:1084-1090) on a packed batch of an
 * unquantised model: the four Linear inputs of layer i are observed under
 * "layer<i>.attn_ln_output", ".attn_out", ".ffn_ln_output", ".inter_gelu"
 * (model.cpp:952-1050), in packed row-major order -- the same stream of
 * values as one reference call per sequence, in sequence order.  logits
 * (host, [T, V]) is nullable. */
int esmcu_model_forward_observed(esmcu_model* m, esmcu_observer* obs, const int32_t* ids, int T,
                                 const int32_t* cu_seqlens, int batch_size, float* logits);
/* esmcu_model_forward_observed with a fresh observer, then the pctile-th
 * percentile of each site into stats_out[num_layers * 4] (layer-major, sites
 * in the order above). */
int esmcu_model_observe_packed(esmcu_model* m, const int32_t* ids, int T,
                               const int32_t* cu_seqlens, int batch_size, float pctile,
                               float* stats_out);

/* ---- on-device weight preparation --------------------------------------
 * Model::ApplySmoothQuant (model.cpp:1462-1468 -> MigrateSmoothQuant,
 * smoothquant.cpp:100-185) on the model's FP32 weights in HBM, with
 * stats[num_layers * 4] as esmcu_model_observe_packed returns them (the
 * inter_gelu entries are unused: fc2 is not migrated).  The per-channel
 * column maxima, the LayerNorm / V / weight rescales run on the device; the
 * scales s = clamp(P_X^a / P_W^(1-a), 1e-3, 1e3) are formed on the host with
 * the reference's float arithmetic; the migrated weights are the
 * reference's bit for bit. */
int esmcu_model_apply_smoothquant(esmcu_model* m, const float* stats, float alpha);
/* Model::QuantizeWeights (model.cpp:1470-1494) on the device: every encoder
 * Linear (and lm_head.dense when quantize_lm_head, the ESM_QUANTIZE_LM_HEAD
 * case) becomes per-output-channel int8 by quant::Quantize (pack.cpp:149-177)
 * in place; the FP32 copies are freed.  No-op on a quantised model. */
int esmcu_model_quantize_weights(esmcu_model* m, int quantize_lm_head);
/* Reads layer `layer` back into the host buffers of `out` (FP32 weights of
 * an unquantised model, int8 rows [out, in] and scales of a quantised one;
 * LN and biases always).  ESMCU_ERR_INVALID_ARGUMENT for a requested tensor
 * the model does not hold. */
int esmcu_model_get_layer(esmcu_model* m, int layer, const esmcu_layer_buffers* out);
/* The INT8 lm_head.dense (ESMCU_ERR_NOT_FOUND when the head is FP32). */
int esmcu_model_get_head_int8(esmcu_model* m, int8_t* lm_dense_wq, float* lm_dense_ws);
/* Section times (ms, CUDA events on the model's stream, names as the
 * reference's ESM_PROFILE sections) when profiling is on (ESM_PROFILE=1 or
 * esmcu_model_set_profiling).  esmcu_model_profile sums every forward since
 * profiling was (re)enabled, or since the last host-buffer forward, and
 * writes up to n {name, ms} entries; returns the count. */
int esmcu_model_set_profiling(esmcu_model* m, int enabled);
int esmcu_model_profile(esmcu_model* m, const char** names, float* ms, int n);
/* Kernel launches issued by the last forward (the product's own kernels). */
int esmcu_model_last_launch_count(const esmcu_model* m);

#ifdef __cplusplus
}
#endif
#endif /* ESM_B200_H */

// Device-resident ESM-2 model: one weight replica per device, the packed
// varlen forward, the scheduled forward and the multi-device dispatcher.
//
// Mirrors the reference's model.cpp:
//   ForwardPackedInto (model.cpp:1093-1255): embed -> N x TransformerBlock ->
//     final LN -> LM head (dense, GELU, LN, tied decoder) -> packed logits.
//   TransformerBlock (model.cpp:932-1066): pre-LN attention block and FFN
//     block, INT8 Linears when the model is quantised, FP32 otherwise.
//   ForwardScheduled (model.cpp:1298-1421): PlanBatches, pack each group,
//     ForwardPacked, scatter outputs back to caller order.
//
// The W8A8 layer on the device (per-tensor activation scales):
//   LN1(+absmax) -> quantise -> QKV GEMM (dequant, Q scale, RoPE fused in the
//   epilogue) -> attention(+absmax) -> quantise -> out GEMM (+residual fused)
//   -> LN2(+absmax) -> quantise -> fc1 GEMM (+GELU, +absmax fused) ->
//   quantise -> fc2 GEMM (+residual fused).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../kernels.cuh"
#include "context.h"
#include "esm_b200.h"
#include "observer.h"
#include "scheduler.h"

using namespace esmb200;

namespace {

struct DevLayer {
  float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
  int8_t *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr;
  float *sqkv = nullptr, *so = nullptr, *s1 = nullptr, *s2 = nullptr;
  float *fqkv = nullptr, *fo = nullptr, *f1 = nullptr, *f2 = nullptr;
  float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
  bool set = false;
};

// Byte offsets of the per-forward buffers inside the arena.
struct Arena {
  size_t ids, masks, cu, pos, hidden, ln, q8, ascale, q, k, v, attn, inter, qkv, logits, amax;
  size_t rows;  // packed row indices scored by the masked-marginal head
  size_t lnstat;  // per-row LayerNorm statistics of the fused LN + quantise kernel
  size_t total;
  int min_len = 0;  // shortest sequence of the batch (kernel choice)
};

}  // namespace

struct esmcu_model {
  esmcu_context* ctx = nullptr;
  esmcu_config cfg{};
  long ldk_d = 0, ldk_ffn = 0;  // int8 row strides (multiples of 16)
  std::vector<DevLayer> layers;
  float *embed = nullptr, *final_ln_w = nullptr, *final_ln_b = nullptr;
  float *lm_w = nullptr, *lm_b = nullptr, *lm_ln_w = nullptr, *lm_ln_b = nullptr,
        *lm_bias = nullptr;
  float* lm_w_lo = nullptr;   // lm_w - tf32(lm_w), for the 3xTF32 dense GEMM
  // INT8 lm_head.dense (ESM_QUANTIZE_LM_HEAD, model.cpp:1209-1211), rows of
  // stride ldk_d, with its per-channel scales; null = the FP32 head.
  int8_t* lm_wq = nullptr;
  float* lm_ws = nullptr;
  // Config::first_block_fc1_fp16 (model.h:38-41): layer 0's fc1 input is
  // rounded to fp16 precision (model.cpp:1031-1033).
  bool fc1_fp16 = false;
  float* embed_lo = nullptr;  // the same for the tied decoder (embed^T)
  // Device staging of the hidden states for ForwardWithHiddenStates.
  float* hs_dev = nullptr;
  size_t hs_bytes = 0;
  bool embed_set = false, head_set = false;
  float *cos_t = nullptr, *sin_t = nullptr;
  int rope_len = 0;
  std::vector<void*> owned;
  char* arena = nullptr;
  size_t arena_bytes = 0;
  // Pinned host staging for the host-buffer entry points: inputs are copied
  // here and sent with one async H2D each; logits come back the same way.
  char* pinned = nullptr;
  size_t pinned_bytes = 0;
  // Pinned ring for the cu_seqlens of esmcu_model_forward_packed_device, so
  // consecutive device-resident forwards enqueue without a host wait: each
  // call copies its cu into the next free stretch and sends it with an async
  // H2D.  When the ring wraps, an event recorded behind the lap's copies is
  // waited on before the stretches are written again (one wait per lap).
  char* cu_ring = nullptr;
  size_t cu_ring_off = 0;
  cudaEvent_t cu_ring_lap = nullptr;
  // profiling
  bool profiling = false;
  using EventPair = std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>;
  std::vector<EventPair> pending;  // recorded, not yet read
  std::vector<cudaEvent_t> event_pool;  // reused so timing adds no event creation
  // One per group of a ForwardScheduled call, recorded behind the group's
  // logits copy so the host hands each group to the caller as it lands.
  std::vector<cudaEvent_t> group_done;
  std::vector<std::pair<std::string, float>> prof;
  int launches = 0;
};

namespace {

#define TRY(x)                     \
  do {                             \
    int rc_ = (x);                 \
    if (rc_ != ESMCU_OK) return rc_; \
  } while (0)

// Launch wrapper: checks the launch and counts it.
#define LAUNCH(m, call)                                   \
  do {                                                    \
    cudaError_t e_ = (call);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
    ++(m)->launches;                                      \
  } while (0)

int upload(esmcu_model* m, void** dst, const void* src, size_t bytes) {
  void* p = nullptr;
  ESMCU_CUDA(cudaMalloc(&p, bytes == 0 ? 16 : bytes));
  m->owned.push_back(p);
  if (bytes) ESMCU_CUDA(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice));
  *dst = p;
  return ESMCU_OK;
}

template <class T>
int upload_vec(esmcu_model* m, T** dst, const T* src, size_t count, const char* name) {
  if (src == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
  return upload(m, reinterpret_cast<void**>(dst), src, count * sizeof(T));
}

// Upload int8 [rows, K] (densely packed) into rows of stride ldk, zero-padded.
int upload_i8_padded(esmcu_model* m, int8_t** dst, const int8_t* const* parts, const int* part_rows,
                     int nparts, int K, long ldk) {
  long rows = 0;
  for (int i = 0; i < nparts; ++i) rows += part_rows[i];
  std::vector<int8_t> host(static_cast<size_t>(rows * ldk), 0);
  long r0 = 0;
  for (int i = 0; i < nparts; ++i) {
    if (parts[i] == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "int8 weight is null");
    for (long r = 0; r < part_rows[i]; ++r)
      std::memcpy(&host[static_cast<size_t>((r0 + r) * ldk)], parts[i] + r * K, static_cast<size_t>(K));
    r0 += part_rows[i];
  }
  return upload(m, reinterpret_cast<void**>(dst), host.data(), host.size());
}

int upload_concat_f32(esmcu_model* m, float** dst, const float* const* parts, const size_t* counts,
                      int nparts, const char* name) {
  size_t total = 0;
  for (int i = 0; i < nparts; ++i) total += counts[i];
  std::vector<float> host(total);
  size_t off = 0;
  for (int i = 0; i < nparts; ++i) {
    if (parts[i] == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    std::memcpy(host.data() + off, parts[i], counts[i] * sizeof(float));
    off += counts[i];
  }
  return upload(m, reinterpret_cast<void**>(dst), host.data(), total * sizeof(float));
}

// The per-forward reduction state, zeroed at the start of every forward: 4
// absmax slot groups per layer (+8 spare), then one grid-barrier counter per
// fused LayerNorm + quantise launch (2 per layer, +8 spare).
size_t amax_region_bytes(int num_layers) {
  return static_cast<size_t>(4 * num_layers + 8) * kAmaxSlots * 4 +
         static_cast<size_t>(2 * num_layers + 8) * 4;
}

Arena plan_arena(const esmcu_model* m, int T, int B) {
  const auto& c = m->cfg;
  Arena a{};
  size_t cur = 0;
  auto take = [&](size_t bytes) {
    const size_t off = cur;
    cur = align_up(cur + std::max<size_t>(bytes, 16), 256);
    return off;
  };
  const size_t Tz = static_cast<size_t>(T), d = static_cast<size_t>(c.hidden_size),
               ffn = static_cast<size_t>(c.intermediate_size);
  a.ids = take(Tz * 4);
  a.masks = take(Tz * 4);
  a.cu = take((static_cast<size_t>(B) + 1) * 4);
  a.pos = take(Tz * 4);
  a.hidden = take(Tz * d * 4);
  a.ln = take(Tz * d * 4);
  a.q8 = take(Tz * static_cast<size_t>(std::max(m->ldk_d, m->ldk_ffn)));
  a.ascale = take(std::max<size_t>(Tz, 1) * 4);
  a.q = take(Tz * d * 4);
  a.k = take(Tz * d * 4);
  a.v = take(Tz * d * 4);
  a.attn = take(Tz * d * 4);
  a.inter = take(Tz * ffn * 4);
  a.qkv = take(Tz * 3 * d * 4);
  a.logits = take(Tz * static_cast<size_t>(c.vocab_size) * 4);
  a.amax = take(amax_region_bytes(c.num_layers));
  a.lnstat = take(Tz * 8);
  a.rows = take((static_cast<size_t>(B) + 1) * 4);
  a.total = cur;
  return a;
}

int ensure_arena(esmcu_model* m, size_t bytes) {
  if (bytes <= m->arena_bytes) return ESMCU_OK;
  ESMCU_CUDA(cudaStreamSynchronize(m->ctx->stream));
  if (m->arena) ESMCU_CUDA(cudaFree(m->arena));
  m->arena = nullptr;
  m->arena_bytes = 0;
  const size_t want = align_up(bytes + bytes / 8, 1 << 21);
  ESMCU_CUDA(cudaMalloc(&m->arena, want));
  m->arena_bytes = want;
  return ESMCU_OK;
}

int ensure_pinned(esmcu_model* m, size_t bytes) {
  if (bytes <= m->pinned_bytes) return ESMCU_OK;
  ESMCU_CUDA(cudaStreamSynchronize(m->ctx->stream));
  if (m->pinned) ESMCU_CUDA(cudaFreeHost(m->pinned));
  m->pinned = nullptr;
  m->pinned_bytes = 0;
  const size_t want = align_up(bytes + bytes / 8, 1 << 20);
  ESMCU_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->pinned), want, cudaHostAllocDefault));
  m->pinned_bytes = want;
  return ESMCU_OK;
}

int ensure_rope(esmcu_model* m, int max_len) {
  if (max_len <= m->rope_len) return ESMCU_OK;
  const int len = std::max(max_len, 1024);
  const int dh = m->cfg.head_dim;
  std::vector<float> c(static_cast<size_t>(len) * dh), s(static_cast<size_t>(len) * dh);
  RopeBuildTables(len, dh, c.data(), s.data());
  ESMCU_CUDA(cudaStreamSynchronize(m->ctx->stream));
  if (m->cos_t) ESMCU_CUDA(cudaFree(m->cos_t));
  if (m->sin_t) ESMCU_CUDA(cudaFree(m->sin_t));
  m->cos_t = m->sin_t = nullptr;
  ESMCU_CUDA(cudaMalloc(&m->cos_t, c.size() * 4));
  ESMCU_CUDA(cudaMalloc(&m->sin_t, s.size() * 4));
  ESMCU_CUDA(cudaMemcpy(m->cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
  ESMCU_CUDA(cudaMemcpy(m->sin_t, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  m->rope_len = len;
  return ESMCU_OK;
}

// CUDA-event section timer, active only when profiling (names follow the
// reference's ESM_PROFILE sections, model.cpp:948-1064).
struct Sections {
  esmcu_model* m;
  std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> ev;
  explicit Sections(esmcu_model* mm) : m(mm) {}
  cudaEvent_t take() {
    cudaEvent_t e;
    if (m->event_pool.empty()) {
      cudaEventCreate(&e);
    } else {
      e = m->event_pool.back();
      m->event_pool.pop_back();
    }
    return e;
  }
  void begin(const char* name) {
    if (!m->profiling) return;
    cudaEvent_t a = take(), b = take();
    cudaEventRecord(a, m->ctx->stream);
    ev.push_back({name, {a, b}});
  }
  void end() {
    if (!m->profiling || ev.empty()) return;
    cudaEventRecord(ev.back().second.second, m->ctx->stream);
  }
};

// Reads the section events of the forwards issued since the last read and
// accumulates them per section name into m->prof (after a stream sync).
void collect_profile(esmcu_model* m, bool reset) {
  if (reset) m->prof.clear();
  if (m->pending.empty()) return;
  cudaStreamSynchronize(m->ctx->stream);
  for (auto& e : m->pending) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e.second.first, e.second.second);
    auto it = std::find_if(m->prof.begin(), m->prof.end(),
                           [&](const auto& p) { return p.first == e.first; });
    if (it == m->prof.end()) m->prof.push_back({e.first, ms});
    else it->second += ms;
    m->event_pool.push_back(e.second.first);
    m->event_pool.push_back(e.second.second);
  }
  m->pending.clear();
}

// Copies a device tensor of one observer site to the host and hands it to
// the observer, which feeds its reservoir on a worker thread.
int observe_site(Observer* obs, int layer, int site, const float* dev, size_t n, cudaStream_t s) {
  static const char* kSites[4] = {"attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu"};
  std::vector<float> h(n);
  if (n) {
    ESMCU_CUDA(cudaMemcpyAsync(h.data(), dev, n * 4, cudaMemcpyDeviceToHost, s));
    ESMCU_CUDA(cudaStreamSynchronize(s));
  }
  obs->observe_async("layer" + std::to_string(layer) + "." + kSites[site], std::move(h));
  return ESMCU_OK;
}

// The packed forward on device buffers already in the arena.  When obs is
// non-null (calibration, ForwardWithObserver), the four Linear inputs of
// every layer are fed to it under the reference's site keys
// (model.cpp:952-1050).
// hidden (device, nullable): [num_layers + 1, T, d] receives the hidden
// states of ForwardPackedInto's hidden_packed_out (model.cpp:1142-1189): the
// embedding output, each layer's output, and in the last entry the final
// LayerNorm's output in place of the last layer's.
// rows (device, nullable): the LM head runs on the R packed rows rows[0..R)
// only, and logits [R, V] receive their log-softmax (the masked-marginal
// head of eval/proteingym.py:84-98).
int forward_device(esmcu_model* m, const Arena& a, const int* ids, const int* mk, float* logits,
                   int T, int B, int max_len, Observer* obs, float* hidden_out = nullptr,
                   const int* rows = nullptr, int R = 0) {
  const auto& c = m->cfg;
  esmcu_context* ctx = m->ctx;
  cudaStream_t s = ctx->stream;
  char* base = m->arena;
  auto F = [&](size_t off) { return reinterpret_cast<float*>(base + off); };
  const int* cu = reinterpret_cast<const int*>(base + a.cu);
  int* pos = reinterpret_cast<int*>(base + a.pos);
  float* hidden = F(a.hidden);
  float* ln = F(a.ln);
  int8_t* q8 = reinterpret_cast<int8_t*>(base + a.q8);
  float* ascale = F(a.ascale);
  float *q = F(a.q), *k = F(a.k), *v = F(a.v), *attn = F(a.attn), *inter = F(a.inter);
  float* qkv = F(a.qkv);
  uint32_t* amax = reinterpret_cast<uint32_t*>(base + a.amax);
  const int d = c.hidden_size, ffn = c.intermediate_size, H = c.num_heads, dh = c.head_dim;
  const bool quant = c.weights_quantized != 0;
  const bool per_token = c.act_quant == ESMCU_ACT_PER_TOKEN;
  const float q_scale = 1.0f / std::sqrt(static_cast<float>(dh));  // model.cpp:978
  const bool fused_rope = quant && dh == 64 && (d % 64) == 0;

  Sections sec(m);

  ESMCU_CUDA(cudaMemsetAsync(amax, 0, amax_region_bytes(c.num_layers), s));
  uint32_t* ln_sync = amax + static_cast<size_t>(4 * c.num_layers + 8) * kAmaxSlots;
  float2* lnstat = reinterpret_cast<float2*>(base + a.lnstat);
  // LayerNorm + per-tensor quantisation in one kernel (no fp32 LN output)
  // unless an observer needs that output.
  // Reference-rounding mode: LayerNorm, GELU and attention reproduce the
  // reference's default x86 kernels (refmath.cu), unfused.
  const bool avx = ctx->math_mode == ESMCU_MATH_AVX512;
  const bool ln_fused = quant && !per_token && obs == nullptr && !avx && d % 128 == 0 &&
                        (d <= 2048 || d == 2560);
  const bool qk_bf16 = !avx && attention_bf16_enabled(c.head_dim);
  LAUNCH(m, launch_positions(cu, B, pos, s));
  sec.begin("embed");
  LAUNCH(m, launch_embed(m->embed, d, ids, mk, cu, B, c.mask_token_id, hidden, s));
  sec.end();
  const size_t Tdh = static_cast<size_t>(T) * c.hidden_size;
  if (hidden_out) ESMCU_CUDA(cudaMemcpyAsync(hidden_out, hidden, Tdh * 4, cudaMemcpyDeviceToDevice, s));

  // INT8 GEMM helper: A = quantised activations in q8 (row stride lda).
  auto gemm_i8 = [&](const int8_t* W, long ldk, int N, const float* ws, const float* bias,
                     EpiParams epi, int M = -1) -> int {
    GemmI8Args g;
    g.A = q8;
    g.lda = ldk;
    g.W = W;
    g.ldw = ldk;
    g.M = M < 0 ? T : M;
    g.N = N;
    g.K = static_cast<int>(ldk);
    g.w_scale = ws;
    g.a_scale = ascale;
    g.per_token = per_token ? 1 : 0;
    g.bias = bias;
    g.epi = epi;
    g.status = ctx->d_status;
    g.num_sms = ctx->num_sms;
    LAUNCH(m, launch_gemm_i8(g, s));
    return ESMCU_OK;
  };
  auto gemm_f32 = [&](const float* A, int K, const float* W, int N, const float* bias,
                      EpiParams epi, int M = -1) -> int {
    GemmF32Args g;
    g.A = A;
    g.lda = K;
    g.W = W;
    g.ldw = K;
    g.M = M < 0 ? T : M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.epi = epi;
    LAUNCH(m, launch_gemm_f32(g, s));
    return ESMCU_OK;
  };
  // Quantise an fp32 activation [T, K] into q8 with row stride ldk.
  auto quantize = [&](const float* x, int K, long ldk, uint32_t* am, int M = -1) -> int {
    const int rows_q = M < 0 ? T : M;
    if (per_token) LAUNCH(m, launch_quantize_per_token(x, K, rows_q, K, q8, ldk, ascale, s));
    else LAUNCH(m, launch_quantize_per_tensor(x, K, rows_q, K, am, q8, ldk, ascale, s));
    return ESMCU_OK;
  };
  auto observe = [&](int layer, int site, const float* x, size_t n) -> int {
    return obs ? observe_site(obs, layer, site, x, n, s) : ESMCU_OK;
  };
  const size_t Td = static_cast<size_t>(T) * d;

  for (int li = 0; li < c.num_layers; ++li) {
    const DevLayer& L = m->layers[static_cast<size_t>(li)];
    uint32_t* am = amax + 4 * li * kAmaxSlots;  // 4 tensors x kAmaxSlots slots
    // ---- attention block
    sec.begin("attn_ln");
    if (ln_fused) {
      LAUNCH(m, launch_layernorm_quant(hidden, L.ln1_w, L.ln1_b, c.layer_norm_eps, T, d, am, lnstat,
                                       ln_sync + 2 * li, q8, m->ldk_d, ascale, ctx->d_status, s));
    } else if (avx) {
      LAUNCH(m, launch_layernorm_avx(hidden, L.ln1_w, L.ln1_b, c.layer_norm_eps, ln, T, d,
                                     quant && !per_token ? am : nullptr, s));
    } else if (quant && per_token) {
      LAUNCH(m, launch_layernorm(hidden, L.ln1_w, L.ln1_b, c.layer_norm_eps, nullptr, T, d, nullptr,
                                 q8, m->ldk_d, ascale, s));
    } else {
      LAUNCH(m, launch_layernorm(hidden, L.ln1_w, L.ln1_b, c.layer_norm_eps, ln, T, d,
                                 quant ? am : nullptr, nullptr, 0, nullptr, s));
    }
    sec.end();
    TRY(observe(li, 0, ln, Td));
    if (quant && (avx || !per_token) && !ln_fused) {
      sec.begin("quantize");
      TRY(quantize(ln, d, m->ldk_d, am));
      sec.end();
    }
    sec.begin("qkv_proj");
    if (quant) {
      EpiParams e;
      if (fused_rope) {
        e.kind = kEpiQkvRope;
        e.q = q;
        e.k = k;
        e.v = v;
        e.d = d;
        e.pos = pos;
        e.cos_t = m->cos_t;
        e.sin_t = m->sin_t;
        e.q_scale = q_scale;
        e.qk_bf16 = qk_bf16 ? 1 : 0;
      } else {
        e.kind = kEpiStore;
        e.C = qkv;
        e.ldc = 3L * d;
      }
      TRY(gemm_i8(L.wqkv, m->ldk_d, 3 * d, L.sqkv, L.bqkv, e));
    } else {
      EpiParams e;
      e.kind = kEpiStore;
      e.C = qkv;
      e.ldc = 3L * d;
      TRY(gemm_f32(ln, d, L.fqkv, 3 * d, L.bqkv, e));
    }
    sec.end();
    if (!fused_rope) {
      sec.begin("q_scale_rope");
      LAUNCH(m, launch_split_qkv_rope(qkv, q, k, v, T, d, H, dh, pos, m->cos_t, m->sin_t, q_scale, s,
                                      qk_bf16));
      sec.end();
    }
    sec.begin("attention");
    // With ESM_AMX_ATTENTION, q and k arrive rounded to bf16 from the QKV
    // epilogue or the split kernel.
    if (avx) {
      LAUNCH(m, launch_attention_avx(q, k, v, cu, B, H, dh, T, max_len, attn,
                                     (quant && !per_token) ? am + 1 * kAmaxSlots : nullptr, s));
    } else {
      LAUNCH(m, launch_attention_varlen(q, k, v, cu, B, H, dh, T, a.min_len, max_len, attn,
                                        (quant && !per_token) ? am + 1 * kAmaxSlots : nullptr,
                                        ctx->d_status, ctx->num_sms, s, qk_bf16));
    }
    sec.end();
    TRY(observe(li, 1, attn, Td));
    if (quant) {
      sec.begin("quantize");
      TRY(quantize(attn, d, m->ldk_d, am + 1 * kAmaxSlots));
      sec.end();
    }
    sec.begin("attn_out_proj");
    {
      EpiParams e;
      e.kind = kEpiResidual;  // hidden += out_proj(attn)  (model.cpp:1002-1015)
      e.C = hidden;
      e.ldc = d;
      if (quant) {
        TRY(gemm_i8(L.wo, m->ldk_d, d, L.so, L.bo, e));
      } else {
        TRY(gemm_f32(attn, d, L.fo, d, L.bo, e));
      }
    }
    sec.end();
    // ---- FFN block
    // Layer 0 with the fp16 escape: LN to fp32, observe, round, then quantise
    // from the rounded values (their absmax is the per-tensor scale).
    const bool round0 = m->fc1_fp16 && li == 0;
    sec.begin("ffn_ln");
    if (ln_fused && !round0) {
      LAUNCH(m, launch_layernorm_quant(hidden, L.ln2_w, L.ln2_b, c.layer_norm_eps, T, d,
                                       am + 2 * kAmaxSlots, lnstat, ln_sync + 2 * li + 1, q8,
                                       m->ldk_d, ascale, ctx->d_status, s));
    } else if (avx) {
      LAUNCH(m, launch_layernorm_avx(hidden, L.ln2_w, L.ln2_b, c.layer_norm_eps, ln, T, d,
                                     quant && !per_token && !round0 ? am + 2 * kAmaxSlots : nullptr,
                                     s));
    } else if (quant && per_token && !round0) {
      LAUNCH(m, launch_layernorm(hidden, L.ln2_w, L.ln2_b, c.layer_norm_eps, nullptr, T, d, nullptr,
                                 q8, m->ldk_d, ascale, s));
    } else {
      LAUNCH(m, launch_layernorm(hidden, L.ln2_w, L.ln2_b, c.layer_norm_eps, ln, T, d,
                                 quant && !round0 ? am + 2 * kAmaxSlots : nullptr, nullptr, 0, nullptr,
                                 s));
    }
    sec.end();
    TRY(observe(li, 2, ln, Td));
    if (round0)
      LAUNCH(m, launch_round_fp16(ln, static_cast<long>(Td), quant && !per_token ? am + 2 * kAmaxSlots : nullptr,
                                  s));
    if (quant && (round0 || avx || (!per_token && !ln_fused))) {
      sec.begin("quantize");
      TRY(quantize(ln, d, m->ldk_d, am + 2 * kAmaxSlots));
      sec.end();
    }
    sec.begin("fc1");
    {
      EpiParams e;
      e.kind = avx ? kEpiStore : kEpiGelu;  // fc1 -> GELU (model.cpp:1036-1046)
      e.C = inter;
      e.ldc = ffn;
      if (quant) {
        e.amax = per_token || avx ? nullptr : am + 3 * kAmaxSlots;
        TRY(gemm_i8(L.w1, m->ldk_d, ffn, L.s1, L.b1, e));
      } else {
        TRY(gemm_f32(ln, d, L.f1, ffn, L.b1, e));
      }
      if (avx)
        LAUNCH(m, launch_gelu_avx(inter, inter, static_cast<long>(T) * ffn,
                                  quant && !per_token ? am + 3 * kAmaxSlots : nullptr, s));
    }
    sec.end();
    TRY(observe(li, 3, inter, static_cast<size_t>(T) * ffn));
    if (quant) {
      sec.begin("quantize");
      TRY(quantize(inter, ffn, m->ldk_ffn, am + 3 * kAmaxSlots));
      sec.end();
    }
    sec.begin("fc2");
    {
      EpiParams e;
      e.kind = kEpiResidual;  // hidden += fc2(inter_gelu) (model.cpp:1052-1065)
      e.C = hidden;
      e.ldc = d;
      if (quant) {
        TRY(gemm_i8(L.w2, m->ldk_ffn, d, L.s2, L.b2, e));
      } else {
        TRY(gemm_f32(inter, ffn, L.f2, d, L.b2, e));
      }
    }
    sec.end();
    if (hidden_out && li + 1 < c.num_layers)
      ESMCU_CUDA(cudaMemcpyAsync(hidden_out + (li + 1) * Tdh, hidden, Tdh * 4,
                                 cudaMemcpyDeviceToDevice, s));
  }

  // ---- final LN + LM head (model.cpp:1181-1239), FP32 unless lm_head.dense
  // is INT8.  Its per-tensor activation scale is the absmax of all T rows
  // of the final LN output (the reference quantises the whole operand), taken
  // by the LN itself into the first spare amax slot.
  const bool lm_int8 = m->lm_wq != nullptr;
  uint32_t* am_lm = amax + 4 * c.num_layers * kAmaxSlots;
  sec.begin("final_ln");
  if (avx)
    LAUNCH(m, launch_layernorm_avx(hidden, m->final_ln_w, m->final_ln_b, c.layer_norm_eps, ln, T,
                                   d, lm_int8 && !per_token ? am_lm : nullptr, s));
  else
    LAUNCH(m, launch_layernorm(hidden, m->final_ln_w, m->final_ln_b, c.layer_norm_eps, ln, T, d,
                               lm_int8 && !per_token ? am_lm : nullptr, nullptr, 0, nullptr, s));
  sec.end();
  if (hidden_out)  // the last entry is the final LayerNorm's output
    ESMCU_CUDA(cudaMemcpyAsync(hidden_out + static_cast<size_t>(c.num_layers) * Tdh, ln, Tdh * 4,
                               cudaMemcpyDeviceToDevice, s));
  // The LM head is row-wise: with `rows` it runs on the selected rows only,
  // gathered into `hidden` (free after the final LayerNorm).
  const float* head_in = ln;
  int TH = T;
  if (rows) {
    LAUNCH(m, launch_gather_rows(ln, rows, R, d, hidden, s));
    head_in = hidden;
    TH = R;
  }
  sec.begin("lm_dense");
  {
    EpiParams e;
    e.kind = avx ? kEpiStore : kEpiGelu;  // dense -> GELU (model.cpp:1192-1223)
    e.C = attn;
    e.ldc = d;
    if (lm_int8) {  // LinearInt8 (model.cpp:1209-1211)
      TRY(quantize(head_in, d, m->ldk_d, am_lm, TH));
      TRY(gemm_i8(m->lm_wq, m->ldk_d, d, m->lm_ws, m->lm_b, e, TH));
    } else if (d % 4 == 0) {
      // 3xTF32 on the tensor cores; the lo part of `ln` goes to `k` (free
      // once the layers are done).
      LAUNCH(m, launch_tf32_lo(head_in, k, static_cast<long>(TH) * d, s));
      GemmTf32Args g;
      g.A = head_in;
      g.A_lo = k;
      g.lda = d;
      g.W = m->lm_w;
      g.W_lo = m->lm_w_lo;
      g.ldw = d;
      g.M = TH;
      g.N = d;
      g.K = d;
      g.bias = m->lm_b;
      g.epi = e;
      g.status = ctx->d_status;
      g.num_sms = ctx->num_sms;
      LAUNCH(m, launch_gemm_tf32x3(g, s));
    } else {
      TRY(gemm_f32(head_in, d, m->lm_w, d, m->lm_b, e, TH));
    }
    if (avx) LAUNCH(m, launch_gelu_avx(attn, attn, static_cast<long>(TH) * d, nullptr, s));
  }
  sec.end();
  sec.begin("lm_ln");
  if (avx)
    LAUNCH(m, launch_layernorm_avx(attn, m->lm_ln_w, m->lm_ln_b, c.layer_norm_eps, q, TH, d, nullptr, s));
  else
    LAUNCH(m, launch_layernorm(attn, m->lm_ln_w, m->lm_ln_b, c.layer_norm_eps, q, TH, d, nullptr,
                               nullptr, 0, nullptr, s));
  sec.end();
  sec.begin("lm_decoder");
  {
    EpiParams e;
    e.kind = kEpiStore;  // tied decoder: lm_ln . embed^T + bias (model.cpp:1234-1239)
    e.C = logits;
    e.ldc = c.vocab_size;
    if (d % 4 == 0) {  // 3xTF32, the lo part of `q` into `v`
      LAUNCH(m, launch_tf32_lo(q, v, static_cast<long>(TH) * d, s));
      GemmTf32Args g;
      g.A = q;
      g.A_lo = v;
      g.lda = d;
      g.W = m->embed;
      g.W_lo = m->embed_lo;
      g.ldw = d;
      g.M = TH;
      g.N = c.vocab_size;
      g.K = d;
      g.bias = m->lm_bias;
      g.epi = e;
      g.status = ctx->d_status;
      g.num_sms = ctx->num_sms;
      LAUNCH(m, launch_gemm_tf32x3(g, s));
    } else {
      TRY(gemm_f32(q, d, m->embed, c.vocab_size, m->lm_bias, e, TH));
    }
  }
  sec.end();
  if (rows) LAUNCH(m, launch_log_softmax_rows(logits, R, c.vocab_size, s));
  for (auto& e : sec.ev) m->pending.push_back(std::move(e));
  return ESMCU_OK;
}

bool model_ready(esmcu_model* m) {
  if (!m->embed_set || !m->head_set) return false;
  for (auto& l : m->layers)
    if (!l.set) return false;
  return true;
}

// Validates a packed batch (host cu_seqlens) and prepares rope tables and the
// arena; returns max_len through *max_len_out.
int prepare(esmcu_model* m, int T, bool has_masks, const int32_t* cu, int B, Arena* a,
            int* max_len_out) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  if (!model_ready(m)) return fail(ESMCU_ERR_INVALID_ARGUMENT, "model weights are not fully set");
  if (cu == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "cu_seqlens is null");
  std::string msg = ValidateBatchView(T, has_masks ? T : 0, cu, B + 1, B);
  if (!msg.empty()) return fail(ESMCU_ERR_INVALID_ARGUMENT, msg);
  int max_len = 0, min_len = B > 0 ? cu[1] - cu[0] : 0;
  for (int b = 0; b < B; ++b) {
    max_len = std::max(max_len, cu[b + 1] - cu[b]);
    min_len = std::min(min_len, cu[b + 1] - cu[b]);
  }
  TRY(ensure_rope(m, max_len));
  *a = plan_arena(m, T, B);
  a->min_len = min_len;
  TRY(ensure_arena(m, a->total));
  *max_len_out = max_len;
  return ESMCU_OK;
}

// Packed forward from host buffers; logits (host) [T, V].
int forward_packed_host(esmcu_model* m, const int32_t* ids, const int32_t* masks, int T,
                        const int32_t* cu, int B, float* logits, Observer* obs,
                        float* hidden = nullptr) {
  Arena a;
  int max_len = 0;
  TRY(prepare(m, T, masks != nullptr, cu, B, &a, &max_len));
  if (T == 0) return ESMCU_OK;  // model.cpp:1105-1108
  if (ids == nullptr || (logits == nullptr && obs == nullptr && hidden == nullptr))
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "ids/logits is null");
  for (int t = 0; t < T; ++t)
    if (ids[t] < 0 || ids[t] >= m->cfg.vocab_size)
      return fail(ESMCU_ERR_OUT_OF_RANGE, "token id " + std::to_string(ids[t]) + " out of range");
  m->launches = 0;
  cudaStream_t s = m->ctx->stream;
  char* base = m->arena;
  const size_t V = static_cast<size_t>(m->cfg.vocab_size);
  const size_t n_ids = static_cast<size_t>(T) * 4, n_cu = static_cast<size_t>(B + 1) * 4;
  const size_t n_logits = logits ? static_cast<size_t>(T) * V * 4 : 0;
  const size_t off_masks = align_up(n_ids, 256), off_cu = off_masks + align_up(masks ? n_ids : 0, 256);
  const size_t off_logits = off_cu + align_up(n_cu, 256);
  TRY(ensure_pinned(m, off_logits + n_logits));
  char* pin = m->pinned;
  std::memcpy(pin, ids, n_ids);
  if (masks) std::memcpy(pin + off_masks, masks, n_ids);
  std::memcpy(pin + off_cu, cu, n_cu);
  ESMCU_CUDA(cudaMemcpyAsync(base + a.ids, pin, n_ids, cudaMemcpyHostToDevice, s));
  if (masks) ESMCU_CUDA(cudaMemcpyAsync(base + a.masks, pin + off_masks, n_ids, cudaMemcpyHostToDevice, s));
  ESMCU_CUDA(cudaMemcpyAsync(base + a.cu, pin + off_cu, n_cu, cudaMemcpyHostToDevice, s));
  float* d_logits = reinterpret_cast<float*>(base + a.logits);
  const size_t n_hidden = hidden ? static_cast<size_t>(m->cfg.num_layers + 1) * T * m->cfg.hidden_size * 4 : 0;
  if (n_hidden > m->hs_bytes) {
    ESMCU_CUDA(cudaStreamSynchronize(s));
    if (m->hs_dev) ESMCU_CUDA(cudaFree(m->hs_dev));
    m->hs_dev = nullptr;
    m->hs_bytes = 0;
    ESMCU_CUDA(cudaMalloc(&m->hs_dev, n_hidden));
    m->hs_bytes = n_hidden;
  }
  TRY(forward_device(m, a, reinterpret_cast<const int*>(base + a.ids),
                     masks ? reinterpret_cast<const int*>(base + a.masks) : nullptr, d_logits, T, B,
                     max_len, obs, hidden ? m->hs_dev : nullptr));
  if (logits) ESMCU_CUDA(cudaMemcpyAsync(pin + off_logits, d_logits, n_logits, cudaMemcpyDeviceToHost, s));
  ESMCU_CUDA(cudaStreamSynchronize(s));
  if (logits) std::memcpy(logits, pin + off_logits, n_logits);
  if (hidden) ESMCU_CUDA(cudaMemcpy(hidden, m->hs_dev, n_hidden, cudaMemcpyDeviceToHost));
  if (obs) obs->wait();
  if (m->profiling) collect_profile(m, true);
  return check_device_status(m->ctx);
}

// Several scheduled groups on one device, enqueued back to back: every
// group's ids / masks / cu go through its own region of the pinned staging
// buffer, its forward runs in the (shared, stream-ordered) arena and its
// logits come back into its own pinned region; one synchronisation at the
// end, then the logits are scattered into caller order.  The host packing of
// group g+1 and the scatter no longer sit between the GPU's groups.
// score_rows (host, nullable): one row per sequence; the output is then
// [n, V], the log-softmax of sequence i's logits at row score_rows[i].
int run_groups(esmcu_model* m, const std::vector<std::vector<int>>& groups, const int32_t* ids_concat,
               const std::vector<long>& offsets, const int32_t* lens, const int32_t* masks_concat,
               float* logits, const int32_t* score_rows = nullptr) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  if (!model_ready(m)) return fail(ESMCU_ERR_INVALID_ARGUMENT, "model weights are not fully set");
  const size_t V = static_cast<size_t>(m->cfg.vocab_size);
  struct Packed {
    const std::vector<int>* group;
    std::vector<int32_t> ids, masks, cu, rows;
    int T = 0, B = 0, max_len = 0;
    Arena a{};
    size_t off_ids = 0, off_masks = 0, off_cu = 0, off_rows = 0, off_logits = 0;
  };
  std::vector<Packed> ps;
  size_t arena_need = 0, pin = 0;
  int max_len_all = 0;
  for (const auto& g : groups) {
    if (g.empty()) continue;
    Packed p;
    p.group = &g;
    p.cu.assign(g.size() + 1, 0);
    for (size_t gi = 0; gi < g.size(); ++gi) {
      const int idx = g[gi];
      const int32_t* src = ids_concat + offsets[static_cast<size_t>(idx)];
      p.ids.insert(p.ids.end(), src, src + lens[idx]);
      if (masks_concat) {
        const int32_t* ms = masks_concat + offsets[static_cast<size_t>(idx)];
        p.masks.insert(p.masks.end(), ms, ms + lens[idx]);
      }
      p.cu[gi + 1] = p.cu[gi] + lens[idx];
    }
    p.T = p.cu.back();
    p.B = static_cast<int>(g.size());
    if (score_rows) {
      for (size_t gi = 0; gi < g.size(); ++gi) {
        const int idx = g[gi];
        if (score_rows[idx] < 0 || score_rows[idx] >= lens[idx])
          return fail(ESMCU_ERR_OUT_OF_RANGE, "row " + std::to_string(score_rows[idx]) +
                                                  " of sequence " + std::to_string(idx) + " (length " +
                                                  std::to_string(lens[idx]) + ")");
        p.rows.push_back(p.cu[gi] + score_rows[idx]);
      }
    }
    if (p.T == 0) continue;
    std::string msg = ValidateBatchView(p.T, masks_concat ? p.T : 0, p.cu.data(), p.B + 1, p.B);
    if (!msg.empty()) return fail(ESMCU_ERR_INVALID_ARGUMENT, msg);
    for (int32_t id : p.ids)
      if (id < 0 || id >= m->cfg.vocab_size)
        return fail(ESMCU_ERR_OUT_OF_RANGE, "token id " + std::to_string(id) + " out of range");
    int min_len = p.cu[1] - p.cu[0];
    for (int b = 0; b < p.B; ++b) {
      p.max_len = std::max(p.max_len, p.cu[b + 1] - p.cu[b]);
      min_len = std::min(min_len, p.cu[b + 1] - p.cu[b]);
    }
    max_len_all = std::max(max_len_all, p.max_len);
    p.a = plan_arena(m, p.T, p.B);
    p.a.min_len = min_len;
    arena_need = std::max(arena_need, p.a.total);
    const size_t n_ids = static_cast<size_t>(p.T) * 4;
    p.off_ids = pin;
    pin += align_up(n_ids, 256);
    p.off_masks = pin;
    if (masks_concat) pin += align_up(n_ids, 256);
    p.off_cu = pin;
    pin += align_up(static_cast<size_t>(p.B + 1) * 4, 256);
    p.off_rows = pin;
    if (score_rows) pin += align_up(static_cast<size_t>(p.B) * 4, 256);
    p.off_logits = pin;
    pin += align_up(static_cast<size_t>(score_rows ? p.B : p.T) * V * 4, 256);
    ps.push_back(std::move(p));
  }
  if (ps.empty()) return ESMCU_OK;
  TRY(ensure_rope(m, max_len_all));
  TRY(ensure_arena(m, arena_need));
  TRY(ensure_pinned(m, pin));
  m->launches = 0;
  cudaStream_t s = m->ctx->stream;
  char* base = m->arena;
  char* hp = m->pinned;
  while (m->group_done.size() < ps.size()) {
    cudaEvent_t e = nullptr;
    ESMCU_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    m->group_done.push_back(e);
  }
  for (size_t pi = 0; pi < ps.size(); ++pi) {
    auto& p = ps[pi];
    const size_t n_ids = static_cast<size_t>(p.T) * 4, n_cu = static_cast<size_t>(p.B + 1) * 4;
    std::memcpy(hp + p.off_ids, p.ids.data(), n_ids);
    if (masks_concat) std::memcpy(hp + p.off_masks, p.masks.data(), n_ids);
    std::memcpy(hp + p.off_cu, p.cu.data(), n_cu);
    ESMCU_CUDA(cudaMemcpyAsync(base + p.a.ids, hp + p.off_ids, n_ids, cudaMemcpyHostToDevice, s));
    if (masks_concat)
      ESMCU_CUDA(cudaMemcpyAsync(base + p.a.masks, hp + p.off_masks, n_ids, cudaMemcpyHostToDevice, s));
    ESMCU_CUDA(cudaMemcpyAsync(base + p.a.cu, hp + p.off_cu, n_cu, cudaMemcpyHostToDevice, s));
    const int* d_rows = nullptr;
    if (score_rows) {
      const size_t n_rows = static_cast<size_t>(p.B) * 4;
      std::memcpy(hp + p.off_rows, p.rows.data(), n_rows);
      ESMCU_CUDA(cudaMemcpyAsync(base + p.a.rows, hp + p.off_rows, n_rows, cudaMemcpyHostToDevice, s));
      d_rows = reinterpret_cast<const int*>(base + p.a.rows);
    }
    float* d_logits = reinterpret_cast<float*>(base + p.a.logits);
    TRY(forward_device(m, p.a, reinterpret_cast<const int*>(base + p.a.ids),
                       masks_concat ? reinterpret_cast<const int*>(base + p.a.masks) : nullptr,
                       d_logits, p.T, p.B, p.max_len, nullptr, nullptr, d_rows, p.B));
    ESMCU_CUDA(cudaMemcpyAsync(hp + p.off_logits, d_logits,
                               static_cast<size_t>(score_rows ? p.B : p.T) * V * 4,
                               cudaMemcpyDeviceToHost, s));
    ESMCU_CUDA(cudaEventRecord(m->group_done[pi], s));
  }
  // Every group is queued; each is copied to the caller's rows as soon as
  // its logits have landed, while the device runs the later groups.
  for (size_t pi = 0; pi < ps.size(); ++pi) {
    const auto& p = ps[pi];
    ESMCU_CUDA(cudaEventSynchronize(m->group_done[pi]));
    const float* src = reinterpret_cast<const float*>(hp + p.off_logits);
    for (size_t gi = 0; gi < p.group->size(); ++gi) {
      const int idx = (*p.group)[gi];
      if (score_rows)
        std::memcpy(logits + static_cast<size_t>(idx) * V, src + gi * V, V * sizeof(float));
      else
        std::memcpy(logits + offsets[static_cast<size_t>(idx)] * static_cast<long>(V),
                    src + static_cast<size_t>(p.cu[gi]) * V,
                    static_cast<size_t>(lens[idx]) * V * sizeof(float));
    }
  }
  if (m->profiling) collect_profile(m, true);
  return check_device_status(m->ctx);
}

int check_sched_args(const int32_t* ids_concat, const int32_t* lens, int n, float* logits) {
  if (n < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "n < 0");
  if (n > 0 && (lens == nullptr || ids_concat == nullptr || logits == nullptr))
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "null ids/lens/logits");
  for (int i = 0; i < n; ++i)
    if (lens[i] < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "negative sequence length");
  return ESMCU_OK;
}

}  // namespace

extern "C" {

int esmcu_model_create(esmcu_context* ctx, const esmcu_config* cfg, esmcu_model** out) {
  if (out == nullptr || cfg == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  TRY(use_device(ctx));
  const auto& c = *cfg;
  if (c.num_layers <= 0 || c.hidden_size <= 0 || c.num_heads <= 0 || c.head_dim <= 0 ||
      c.intermediate_size <= 0 || c.vocab_size <= 0)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "config dimensions must be positive");
  if (c.num_heads * c.head_dim != c.hidden_size)
    return fail(ESMCU_ERR_SHAPE_MISMATCH, "num_heads * head_dim != hidden_size");
  if (c.head_dim % 4 != 0 || c.head_dim > 128)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "head_dim must be a multiple of 4 and <= 128");
  if (c.act_quant != ESMCU_ACT_PER_TENSOR && c.act_quant != ESMCU_ACT_PER_TOKEN)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad act_quant");
  auto* m = new esmcu_model();
  m->ctx = ctx;
  m->cfg = c;
  m->ldk_d = static_cast<long>(align_up(static_cast<size_t>(c.hidden_size), 16));
  m->ldk_ffn = static_cast<long>(align_up(static_cast<size_t>(c.intermediate_size), 16));
  m->layers.resize(static_cast<size_t>(c.num_layers));
  const char* prof = std::getenv("ESM_PROFILE");
  m->profiling = prof && *prof && std::string(prof) != "0";
  *out = m;
  return ESMCU_OK;
}

int esmcu_model_destroy(esmcu_model* m) {
  if (m == nullptr) return ESMCU_OK;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (void* p : m->owned) cudaFree(p);
  if (m->arena) cudaFree(m->arena);
  if (m->pinned) cudaFreeHost(m->pinned);
  if (m->cu_ring) cudaFreeHost(m->cu_ring);
  if (m->cu_ring_lap) cudaEventDestroy(m->cu_ring_lap);
  for (auto& e : m->pending) {
    cudaEventDestroy(e.second.first);
    cudaEventDestroy(e.second.second);
  }
  for (auto e : m->event_pool) cudaEventDestroy(e);
  for (auto e : m->group_done) cudaEventDestroy(e);
  if (m->cos_t) cudaFree(m->cos_t);
  if (m->sin_t) cudaFree(m->sin_t);
  if (m->hs_dev) cudaFree(m->hs_dev);
  delete m;
  return ESMCU_OK;
}

int esmcu_model_config(const esmcu_model* m, esmcu_config* out) {
  if (m == nullptr || out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  *out = m->cfg;
  return ESMCU_OK;
}

// *lo (allocated once) = x - tf32(x) over n floats of device data x.
static int make_lo(esmcu_model* m, float** lo, const float* x, size_t n, const char* name) {
  if (*lo == nullptr) {
    void* p = nullptr;
    if (cudaMalloc(&p, (n == 0 ? 1 : n) * sizeof(float)) != cudaSuccess)
      return fail(ESMCU_ERR_CUDA, std::string("cudaMalloc(") + name + ") failed");
    m->owned.push_back(p);
    *lo = static_cast<float*>(p);
  }
  cudaError_t e = launch_tf32_lo(x, *lo, static_cast<long>(n), m->ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->ctx->stream);
  return e == cudaSuccess ? ESMCU_OK : cuda_fail(e, name);
}

int esmcu_model_set_embeddings(esmcu_model* m, const float* embed) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  const size_t n = static_cast<size_t>(m->cfg.vocab_size) * m->cfg.hidden_size;
  TRY(upload_vec(m, &m->embed, embed, n, "embed"));
  TRY(make_lo(m, &m->embed_lo, m->embed, n, "embed_lo"));  // the decoder's W_lo
  m->embed_set = true;
  return ESMCU_OK;
}

int esmcu_model_set_head(esmcu_model* m, const float* final_ln_w, const float* final_ln_b,
                         const float* lm_dense_w, const float* lm_dense_b, const float* lm_ln_w,
                         const float* lm_ln_b, const float* lm_decoder_bias) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  const size_t d = static_cast<size_t>(m->cfg.hidden_size);
  TRY(upload_vec(m, &m->final_ln_w, final_ln_w, d, "final_ln_w"));
  TRY(upload_vec(m, &m->final_ln_b, final_ln_b, d, "final_ln_b"));
  TRY(upload_vec(m, &m->lm_w, lm_dense_w, d * d, "lm_dense_w"));
  // Its lo part for the 3xTF32 GEMM, formed once on the device.
  TRY(make_lo(m, &m->lm_w_lo, m->lm_w, d * d, "lm_w_lo"));
  TRY(upload_vec(m, &m->lm_b, lm_dense_b, d, "lm_dense_b"));
  TRY(upload_vec(m, &m->lm_ln_w, lm_ln_w, d, "lm_ln_w"));
  TRY(upload_vec(m, &m->lm_ln_b, lm_ln_b, d, "lm_ln_b"));
  TRY(upload_vec(m, &m->lm_bias, lm_decoder_bias, static_cast<size_t>(m->cfg.vocab_size), "lm_bias"));
  m->head_set = true;
  return ESMCU_OK;
}

int esmcu_model_set_first_block_fc1_fp16(esmcu_model* m, int enabled) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  m->fc1_fp16 = enabled != 0;
  return ESMCU_OK;
}

int esmcu_model_set_head_int8(esmcu_model* m, const int8_t* lm_dense_wq, const float* lm_dense_ws) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  if (lm_dense_wq == nullptr) {  // back to the FP32 head (the buffers stay owned)
    m->lm_wq = nullptr;
    m->lm_ws = nullptr;
    return ESMCU_OK;
  }
  const int d = m->cfg.hidden_size;
  int8_t* wq = nullptr;
  float* ws = nullptr;
  TRY(upload_i8_padded(m, &wq, &lm_dense_wq, &d, 1, d, m->ldk_d));
  TRY(upload_vec(m, &ws, lm_dense_ws, static_cast<size_t>(d), "lm_dense_ws"));
  m->lm_wq = wq;
  m->lm_ws = ws;
  return ESMCU_OK;
}

int esmcu_model_set_layer(esmcu_model* m, int layer, const esmcu_layer_weights* w) {
  if (m == nullptr || w == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  if (layer < 0 || layer >= m->cfg.num_layers)
    return fail(ESMCU_ERR_OUT_OF_RANGE, "layer index out of range");
  TRY(use_device(m->ctx));
  DevLayer& L = m->layers[static_cast<size_t>(layer)];
  const int d = m->cfg.hidden_size, ffn = m->cfg.intermediate_size;
  const size_t dz = static_cast<size_t>(d), fz = static_cast<size_t>(ffn);
  TRY(upload_vec(m, &L.ln1_w, w->attn_ln_w, dz, "attn_ln_w"));
  TRY(upload_vec(m, &L.ln1_b, w->attn_ln_b, dz, "attn_ln_b"));
  TRY(upload_vec(m, &L.ln2_w, w->ffn_ln_w, dz, "ffn_ln_w"));
  TRY(upload_vec(m, &L.ln2_b, w->ffn_ln_b, dz, "ffn_ln_b"));
  {
    const float* parts[3] = {w->q_b, w->k_b, w->v_b};
    const size_t counts[3] = {dz, dz, dz};
    TRY(upload_concat_f32(m, &L.bqkv, parts, counts, 3, "q/k/v bias"));
  }
  TRY(upload_vec(m, &L.bo, w->out_b, dz, "out_b"));
  TRY(upload_vec(m, &L.b1, w->fc1_b, fz, "fc1_b"));
  TRY(upload_vec(m, &L.b2, w->fc2_b, dz, "fc2_b"));
  if (m->cfg.weights_quantized) {
    {
      const int8_t* parts[3] = {w->q_wq, w->k_wq, w->v_wq};
      const int rows[3] = {d, d, d};
      TRY(upload_i8_padded(m, &L.wqkv, parts, rows, 3, d, m->ldk_d));
      const float* sp[3] = {w->q_ws, w->k_ws, w->v_ws};
      const size_t sc[3] = {dz, dz, dz};
      TRY(upload_concat_f32(m, &L.sqkv, sp, sc, 3, "q/k/v scales"));
    }
    {
      const int8_t* p[1] = {w->out_wq};
      const int r[1] = {d};
      TRY(upload_i8_padded(m, &L.wo, p, r, 1, d, m->ldk_d));
      TRY(upload_vec(m, &L.so, w->out_ws, dz, "out scales"));
    }
    {
      const int8_t* p[1] = {w->fc1_wq};
      const int r[1] = {ffn};
      TRY(upload_i8_padded(m, &L.w1, p, r, 1, d, m->ldk_d));
      TRY(upload_vec(m, &L.s1, w->fc1_ws, fz, "fc1 scales"));
    }
    {
      const int8_t* p[1] = {w->fc2_wq};
      const int r[1] = {d};
      TRY(upload_i8_padded(m, &L.w2, p, r, 1, ffn, m->ldk_ffn));
      TRY(upload_vec(m, &L.s2, w->fc2_ws, dz, "fc2 scales"));
    }
  } else {
    const float* parts[3] = {w->q_w, w->k_w, w->v_w};
    const size_t counts[3] = {dz * dz, dz * dz, dz * dz};
    TRY(upload_concat_f32(m, &L.fqkv, parts, counts, 3, "q/k/v weight"));
    TRY(upload_vec(m, &L.fo, w->out_w, dz * dz, "out_w"));
    TRY(upload_vec(m, &L.f1, w->fc1_w, fz * dz, "fc1_w"));
    TRY(upload_vec(m, &L.f2, w->fc2_w, dz * fz, "fc2_w"));
  }
  L.set = true;
  return ESMCU_OK;
}

// ---- on-device weight preparation

namespace {

// SmoothQuantScales (smoothquant.cpp:49-74) for one channel, with the same
// float arithmetic and C library powf as the reference.
float smooth_scale(float px, float pw, float alpha) {
  if (px <= 0.0f || pw <= 0.0f) return 1.0f;
  const float num = std::pow(px, alpha);
  const float den = std::pow(pw, 1.0f - alpha);
  float val = num / den;
  if (!std::isfinite(val) || val <= 0.0f) return 1.0f;
  if (val < 1e-3f) val = 1e-3f;
  if (val > 1e3f) val = 1e3f;
  return val;
}

// Column absmax of a device [N, K] matrix, to the host.
int col_absmax_host(esmcu_model* m, const float* W, int N, int K, uint32_t* d_tmp,
                    std::vector<float>* out) {
  cudaStream_t s = m->ctx->stream;
  ESMCU_CUDA(launch_col_absmax(W, N, K, d_tmp, s));
  out->resize(static_cast<size_t>(K));
  ESMCU_CUDA(cudaMemcpyAsync(out->data(), d_tmp, static_cast<size_t>(K) * 4, cudaMemcpyDeviceToHost, s));
  ESMCU_CUDA(cudaStreamSynchronize(s));
  return ESMCU_OK;
}

void release(esmcu_model* m, void* p) {
  if (p == nullptr) return;
  cudaFree(p);
  m->owned.erase(std::remove(m->owned.begin(), m->owned.end(), p), m->owned.end());
}

// Quantize (pack.cpp:149-177) of a device FP32 [N, K] matrix into freshly
// allocated int8 rows of stride ldk (zero padding) and [N] scales.
int quantize_device(esmcu_model* m, const float* W, int N, int K, long ldk, int8_t** q,
                    float** scales) {
  cudaStream_t s = m->ctx->stream;
  void* pq = nullptr;
  void* ps = nullptr;
  ESMCU_CUDA(cudaMalloc(&pq, static_cast<size_t>(N) * ldk));
  m->owned.push_back(pq);
  ESMCU_CUDA(cudaMalloc(&ps, static_cast<size_t>(N) * 4));
  m->owned.push_back(ps);
  ESMCU_CUDA(cudaMemsetAsync(pq, 0, static_cast<size_t>(N) * ldk, s));
  ESMCU_CUDA(launch_quantize_weights(W, N, K, static_cast<int8_t*>(pq), ldk, static_cast<float*>(ps), s));
  *q = static_cast<int8_t*>(pq);
  *scales = static_cast<float*>(ps);
  return ESMCU_OK;
}

int copy_out(void* dst, const void* src, size_t bytes) {
  if (dst == nullptr) return ESMCU_OK;
  if (src == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "the model holds no such tensor");
  ESMCU_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
  return ESMCU_OK;
}

// Rows [r0, r0 + n) of a device int8 matrix with row stride ldk, K bytes each,
// to dense host rows.
int copy_out_i8(int8_t* dst, const int8_t* src, long r0, int n, int K, long ldk) {
  if (dst == nullptr) return ESMCU_OK;
  if (src == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "the model holds no int8 weights");
  ESMCU_CUDA(cudaMemcpy2D(dst, static_cast<size_t>(K), src + r0 * ldk, static_cast<size_t>(ldk),
                          static_cast<size_t>(K), static_cast<size_t>(n), cudaMemcpyDeviceToHost));
  return ESMCU_OK;
}

}  // namespace

int esmcu_model_apply_smoothquant(esmcu_model* m, const float* stats, float alpha) {
  if (m == nullptr || stats == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  TRY(use_device(m->ctx));
  if (!model_ready(m)) return fail(ESMCU_ERR_INVALID_ARGUMENT, "model weights are not fully set");
  if (m->cfg.weights_quantized)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "apply_smoothquant runs on FP32 weights, before quantize");
  const int d = m->cfg.hidden_size, ffn = m->cfg.intermediate_size;
  cudaStream_t s = m->ctx->stream;
  void* tmp = nullptr;  // column maxima, then the scales
  ESMCU_CUDA(cudaMalloc(&tmp, static_cast<size_t>(std::max(d, ffn)) * 8));
  uint32_t* d_cmax = static_cast<uint32_t*>(tmp);
  float* d_s = reinterpret_cast<float*>(d_cmax + std::max(d, ffn));
  auto scales = [&](float px, const std::vector<float>& pw) {
    std::vector<float> sc(pw.size());
    for (size_t k = 0; k < pw.size(); ++k) sc[k] = smooth_scale(px, pw[k], alpha);
    return sc;
  };
  auto upload_s = [&](const std::vector<float>& sc) -> int {
    ESMCU_CUDA(cudaMemcpyAsync(d_s, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice, s));
    return ESMCU_OK;
  };
  int rc = ESMCU_OK;
  std::vector<float> pw;
  for (int li = 0; li < m->cfg.num_layers && rc == ESMCU_OK; ++li) {
    DevLayer& L = m->layers[static_cast<size_t>(li)];
    auto step = [&]() -> int {
      // Site 1: attn_ln_output -> Q, K, V (smoothquant.cpp:110-138).  Wq|Wk|Wv
      // are one [3d, d] matrix, so its column max is the max over the three.
      TRY(col_absmax_host(m, L.fqkv, 3 * d, d, d_cmax, &pw));
      TRY(upload_s(scales(stats[li * 4 + 0], pw)));
      ESMCU_CUDA(launch_div_vec2(L.ln1_w, L.ln1_b, d, d_s, s));
      ESMCU_CUDA(launch_mul_cols(L.fqkv, 3L * d, d, d_s, s));
      // Site 2: attn_out -> out_proj; V's rows and bias divided
      // (smoothquant.cpp:140-166).
      TRY(col_absmax_host(m, L.fo, d, d, d_cmax, &pw));
      TRY(upload_s(scales(stats[li * 4 + 1], pw)));
      ESMCU_CUDA(launch_div_rows(L.fqkv + 2L * d * d, d, d, L.bqkv + 2L * d, d_s, s));
      ESMCU_CUDA(launch_mul_cols(L.fo, d, d, d_s, s));
      // Site 3: ffn_ln_output -> fc1 (smoothquant.cpp:168-180).  fc2 is not
      // migrated.
      TRY(col_absmax_host(m, L.f1, ffn, d, d_cmax, &pw));
      TRY(upload_s(scales(stats[li * 4 + 2], pw)));
      ESMCU_CUDA(launch_div_vec2(L.ln2_w, L.ln2_b, d, d_s, s));
      ESMCU_CUDA(launch_mul_cols(L.f1, ffn, d, d_s, s));
      ESMCU_CUDA(cudaStreamSynchronize(s));
      return ESMCU_OK;
    };
    rc = step();
  }
  cudaFree(tmp);
  return rc;
}

int esmcu_model_quantize_weights(esmcu_model* m, int quantize_lm_head) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  if (!model_ready(m)) return fail(ESMCU_ERR_INVALID_ARGUMENT, "model weights are not fully set");
  if (m->cfg.weights_quantized) return ESMCU_OK;  // model.cpp:1471
  const int d = m->cfg.hidden_size, ffn = m->cfg.intermediate_size;
  for (auto& L : m->layers) {
    TRY(quantize_device(m, L.fqkv, 3 * d, d, m->ldk_d, &L.wqkv, &L.sqkv));
    TRY(quantize_device(m, L.fo, d, d, m->ldk_d, &L.wo, &L.so));
    TRY(quantize_device(m, L.f1, ffn, d, m->ldk_d, &L.w1, &L.s1));
    TRY(quantize_device(m, L.f2, d, ffn, m->ldk_ffn, &L.w2, &L.s2));
  }
  if (quantize_lm_head) TRY(quantize_device(m, m->lm_w, d, d, m->ldk_d, &m->lm_wq, &m->lm_ws));
  ESMCU_CUDA(cudaStreamSynchronize(m->ctx->stream));
  for (auto& L : m->layers) {  // the FP32 copies are no longer read
    release(m, L.fqkv);
    release(m, L.fo);
    release(m, L.f1);
    release(m, L.f2);
    L.fqkv = L.fo = L.f1 = L.f2 = nullptr;
  }
  m->cfg.weights_quantized = 1;
  return ESMCU_OK;
}

int esmcu_model_get_layer(esmcu_model* m, int layer, const esmcu_layer_buffers* out) {
  if (m == nullptr || out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  if (layer < 0 || layer >= m->cfg.num_layers)
    return fail(ESMCU_ERR_OUT_OF_RANGE, "layer index out of range");
  TRY(use_device(m->ctx));
  ESMCU_CUDA(cudaStreamSynchronize(m->ctx->stream));
  const DevLayer& L = m->layers[static_cast<size_t>(layer)];
  if (!L.set) return fail(ESMCU_ERR_INVALID_ARGUMENT, "layer weights are not set");
  const size_t d = static_cast<size_t>(m->cfg.hidden_size), f = static_cast<size_t>(m->cfg.intermediate_size);
  const int di = m->cfg.hidden_size, fi = m->cfg.intermediate_size;
  TRY(copy_out(out->attn_ln_w, L.ln1_w, d * 4));
  TRY(copy_out(out->attn_ln_b, L.ln1_b, d * 4));
  TRY(copy_out(out->ffn_ln_w, L.ln2_w, d * 4));
  TRY(copy_out(out->ffn_ln_b, L.ln2_b, d * 4));
  TRY(copy_out(out->q_b, L.bqkv, d * 4));
  TRY(copy_out(out->k_b, L.bqkv ? L.bqkv + d : nullptr, d * 4));
  TRY(copy_out(out->v_b, L.bqkv ? L.bqkv + 2 * d : nullptr, d * 4));
  TRY(copy_out(out->out_b, L.bo, d * 4));
  TRY(copy_out(out->fc1_b, L.b1, f * 4));
  TRY(copy_out(out->fc2_b, L.b2, d * 4));
  TRY(copy_out(out->q_w, L.fqkv, d * d * 4));
  TRY(copy_out(out->k_w, L.fqkv ? L.fqkv + d * d : nullptr, d * d * 4));
  TRY(copy_out(out->v_w, L.fqkv ? L.fqkv + 2 * d * d : nullptr, d * d * 4));
  TRY(copy_out(out->out_w, L.fo, d * d * 4));
  TRY(copy_out(out->fc1_w, L.f1, f * d * 4));
  TRY(copy_out(out->fc2_w, L.f2, d * f * 4));
  TRY(copy_out_i8(out->q_wq, L.wqkv, 0, di, di, m->ldk_d));
  TRY(copy_out_i8(out->k_wq, L.wqkv, di, di, di, m->ldk_d));
  TRY(copy_out_i8(out->v_wq, L.wqkv, 2L * di, di, di, m->ldk_d));
  TRY(copy_out_i8(out->out_wq, L.wo, 0, di, di, m->ldk_d));
  TRY(copy_out_i8(out->fc1_wq, L.w1, 0, fi, di, m->ldk_d));
  TRY(copy_out_i8(out->fc2_wq, L.w2, 0, di, fi, m->ldk_ffn));
  TRY(copy_out(out->q_ws, L.sqkv, d * 4));
  TRY(copy_out(out->k_ws, L.sqkv ? L.sqkv + d : nullptr, d * 4));
  TRY(copy_out(out->v_ws, L.sqkv ? L.sqkv + 2 * d : nullptr, d * 4));
  TRY(copy_out(out->out_ws, L.so, d * 4));
  TRY(copy_out(out->fc1_ws, L.s1, f * 4));
  TRY(copy_out(out->fc2_ws, L.s2, d * 4));
  return ESMCU_OK;
}

int esmcu_model_get_head_int8(esmcu_model* m, int8_t* lm_dense_wq, float* lm_dense_ws) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(use_device(m->ctx));
  if (m->lm_wq == nullptr) return fail(ESMCU_ERR_NOT_FOUND, "the LM head is FP32");
  const int d = m->cfg.hidden_size;
  TRY(copy_out_i8(lm_dense_wq, m->lm_wq, 0, d, d, m->ldk_d));
  TRY(copy_out(lm_dense_ws, m->lm_ws, static_cast<size_t>(d) * 4));
  return ESMCU_OK;
}

int esmcu_model_forward_packed(esmcu_model* m, const int32_t* ids, const int32_t* masks, int T,
                               const int32_t* cu, int B, float* logits) {
  return forward_packed_host(m, ids, masks, T, cu, B, logits, nullptr);
}

int esmcu_model_forward_hidden_states(esmcu_model* m, const int32_t* ids, const int32_t* masks,
                                      int T, const int32_t* cu, int B, float* logits,
                                      float* hidden_out) {
  if (hidden_out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "hidden_out is null");
  return forward_packed_host(m, ids, masks, T, cu, B, logits, nullptr, hidden_out);
}

int esmcu_model_forward_packed_device(esmcu_model* m, const int32_t* d_ids,
                                      const int32_t* d_masks, int T, const int32_t* cu, int B,
                                      float* d_logits) {
  Arena a;
  int max_len = 0;
  TRY(prepare(m, T, d_masks != nullptr, cu, B, &a, &max_len));
  if (T == 0) return ESMCU_OK;
  if (d_ids == nullptr || d_logits == nullptr)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "ids/logits is null");
  m->launches = 0;
  cudaStream_t s = m->ctx->stream;
  constexpr size_t kRing = 1u << 20;
  const size_t n_cu = static_cast<size_t>(B + 1) * 4;
  if (n_cu > kRing) {  // a batch beyond the ring: plain (synchronising) copy
    ESMCU_CUDA(cudaMemcpyAsync(m->arena + a.cu, cu, n_cu, cudaMemcpyHostToDevice, s));
  } else {
    if (m->cu_ring == nullptr) {
      ESMCU_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->cu_ring), kRing, cudaHostAllocDefault));
      ESMCU_CUDA(cudaEventCreateWithFlags(&m->cu_ring_lap, cudaEventDisableTiming));
    }
    if (m->cu_ring_off + n_cu > kRing) {  // wrap: the lap's copies must have run
      ESMCU_CUDA(cudaEventRecord(m->cu_ring_lap, s));
      ESMCU_CUDA(cudaEventSynchronize(m->cu_ring_lap));
      m->cu_ring_off = 0;
    }
    char* src = m->cu_ring + m->cu_ring_off;
    m->cu_ring_off = align_up(m->cu_ring_off + n_cu, 256);
    std::memcpy(src, cu, n_cu);
    ESMCU_CUDA(cudaMemcpyAsync(m->arena + a.cu, src, n_cu, cudaMemcpyHostToDevice, s));
  }
  return forward_device(m, a, d_ids, d_masks, d_logits, T, B, max_len, nullptr);
}

int esmcu_model_forward_observed(esmcu_model* m, esmcu_observer* obs, const int32_t* ids, int T,
                                 const int32_t* cu, int B, float* logits) {
  if (m == nullptr || obs == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  if (m->cfg.weights_quantized)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "calibration runs on the unquantised model");
  return forward_packed_host(m, ids, nullptr, T, cu, B, logits, reinterpret_cast<Observer*>(obs));
}

int esmcu_model_observe_packed(esmcu_model* m, const int32_t* ids, int T, const int32_t* cu,
                               int B, float pctile, float* stats_out) {
  if (m == nullptr || stats_out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  if (m->cfg.weights_quantized)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "calibration runs on the unquantised model");
  Observer obs;
  TRY(forward_packed_host(m, ids, nullptr, T, cu, B, nullptr, &obs));
  static const char* kSites[4] = {"attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu"};
  for (int li = 0; li < m->cfg.num_layers; ++li)
    for (int j = 0; j < 4; ++j) {
      const Observer::Reservoir* r = obs.find("layer" + std::to_string(li) + "." + kSites[j]);
      stats_out[li * 4 + j] = r ? r->percentile(pctile) : 0.0f;
    }
  return ESMCU_OK;
}

int esmcu_model_forward_scheduled(esmcu_model* m, const int32_t* ids_concat, const int32_t* lens,
                                  const int32_t* masks_concat, int n, float threshold,
                                  int max_batch, float* logits) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(check_sched_args(ids_concat, lens, n, logits));
  if (n == 0) return ESMCU_OK;
  std::vector<int> lengths(lens, lens + n);
  std::vector<long> offsets(static_cast<size_t>(n) + 1, 0);
  for (int i = 0; i < n; ++i) offsets[static_cast<size_t>(i) + 1] = offsets[static_cast<size_t>(i)] + lens[i];
  auto plan = PlanBatches(lengths, threshold, max_batch);
  return run_groups(m, plan, ids_concat, offsets, lens, masks_concat, logits);
}

int esmcu_model_masked_marginals(esmcu_model* m, const int32_t* ids_concat, const int32_t* lens,
                                 const int32_t* masks_concat, const int32_t* rows, int n,
                                 float threshold, int max_batch, float* log_probs) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  TRY(check_sched_args(ids_concat, lens, n, log_probs));
  if (n == 0) return ESMCU_OK;
  if (rows == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "rows is null");
  std::vector<int> lengths(lens, lens + n);
  std::vector<long> offsets(static_cast<size_t>(n) + 1, 0);
  for (int i = 0; i < n; ++i) offsets[static_cast<size_t>(i) + 1] = offsets[static_cast<size_t>(i)] + lens[i];
  auto plan = PlanBatches(lengths, threshold, max_batch);
  return run_groups(m, plan, ids_concat, offsets, lens, masks_concat, log_probs, rows);
}

int esmcu_forward_scheduled_multi(esmcu_model** models, int n_models, const int32_t* ids_concat,
                                  const int32_t* lens, const int32_t* masks_concat, int n,
                                  float threshold, int max_batch, float* logits) {
  if (models == nullptr || n_models <= 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "no models");
  TRY(check_sched_args(ids_concat, lens, n, logits));
  if (n == 0) return ESMCU_OK;
  std::vector<int> lengths(lens, lens + n);
  std::vector<long> offsets(static_cast<size_t>(n) + 1, 0);
  for (int i = 0; i < n; ++i) offsets[static_cast<size_t>(i) + 1] = offsets[static_cast<size_t>(i)] + lens[i];
  auto plan = PlanBatches(lengths, threshold, max_batch);
  // Longest-processing-time assignment on sum_b(24 d^2 L_b + 4 d L_b^2).
  const double d = models[0]->cfg.hidden_size;
  std::vector<std::pair<double, int>> cost;
  for (size_t g = 0; g < plan.size(); ++g) {
    double c = 0.0;
    for (int idx : plan[g]) {
      const double L = lens[idx];
      c += 24.0 * d * d * L + 4.0 * d * L * L;
    }
    cost.push_back({c, static_cast<int>(g)});
  }
  std::sort(cost.begin(), cost.end(), [](auto& a, auto& b) { return a.first > b.first; });
  std::vector<double> load(static_cast<size_t>(n_models), 0.0);
  std::vector<std::vector<int>> assign(static_cast<size_t>(n_models));
  for (auto& cg : cost) {
    const size_t best = static_cast<size_t>(std::min_element(load.begin(), load.end()) - load.begin());
    load[best] += cg.first;
    assign[best].push_back(cg.second);
  }
  std::vector<int> rc(static_cast<size_t>(n_models), ESMCU_OK);
  std::vector<std::string> err(static_cast<size_t>(n_models));
  std::vector<std::thread> threads;
  for (int w = 0; w < n_models; ++w) {
    threads.emplace_back([&, w]() {
      std::vector<std::vector<int>> mine;
      for (int g : assign[static_cast<size_t>(w)]) mine.push_back(plan[static_cast<size_t>(g)]);
      int r = run_groups(models[w], mine, ids_concat, offsets, lens, masks_concat, logits);
      if (r != ESMCU_OK) {
        rc[static_cast<size_t>(w)] = r;
        err[static_cast<size_t>(w)] = esmcu_last_error();
      }
    });
  }
  for (auto& t : threads) t.join();
  for (int w = 0; w < n_models; ++w)
    if (rc[static_cast<size_t>(w)] != ESMCU_OK)
      return fail(rc[static_cast<size_t>(w)], "device worker " + std::to_string(w) + ": " + err[static_cast<size_t>(w)]);
  return ESMCU_OK;
}

int esmcu_model_set_profiling(esmcu_model* m, int enabled) {
  if (m == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null model");
  collect_profile(m, true);
  m->profiling = enabled != 0;
  return ESMCU_OK;
}

int esmcu_model_profile(esmcu_model* m, const char** names, float* ms, int n) {
  if (m == nullptr) return -1;
  collect_profile(m, false);
  int i = 0;
  for (; i < n && i < static_cast<int>(m->prof.size()); ++i) {
    names[i] = m->prof[static_cast<size_t>(i)].first.c_str();
    ms[i] = m->prof[static_cast<size_t>(i)].second;
  }
  return i;
}

int esmcu_model_last_launch_count(const esmcu_model* m) { return m ? m->launches : 0; }

}  // extern "C"

// C ABI over the reference esm.cpp CPU engine, compiled from the reference's
// own sources by oracle/Makefile into oracle/_ref/libesmref.so.
//
// TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline / reference arm load this library as the checker or as the
// timed CPU baseline.  The product (esm-cpp_b200/) never links or loads it.
//
// Every entry point forwards to one reference function; the comment on each
// names the reference symbol (path:line inside the reference project).

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "esm_cpp/batch.h"
#include "esm_cpp/cpu_features.h"
#include "esm_cpp/kernels.h"
#include "esm_cpp/model.h"
#include "esm_cpp/observer.h"
#include "esm_cpp/quant.h"
#include "esm_cpp/scheduler.h"
#include "esm_cpp/thread_pool.h"

namespace esm::kernels {
// Defined with external linkage in src/kernels/gemm_int8.cpp (AVX-512 TU) and
// src/kernels/gemm_amx.cpp; not declared in any public header.
void QuantizeActPrefixAvx512(const float* A, std::size_t MK, std::uint8_t* a_u8,
                             float* act_scale_out);
void LinearVnni(const float* A, const esm::quant::QuantizedTensor& W,
                const float* bias, float* C, int M, int N, int K);
void LinearAmx(const float* A, const esm::quant::QuantizedTensor& W,
               const float* bias, float* C, int M, int N, int K);
}  // namespace esm::kernels

namespace {
thread_local std::string g_err;

template <class F>
int Guard(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  } catch (...) {
    g_err = "unknown exception";
    return -1;
  }
}

esm::quant::QuantizedTensor MakeQt(const std::int8_t* packed, const float* scales,
                                   int N, int K) {
  esm::quant::QuantizedTensor qt;
  qt.N = N;
  qt.K = K;
  qt.packed.assign(packed, packed + static_cast<std::size_t>(N) * K);
  qt.per_channel_scales.assign(scales, scales + N);
  esm::quant::BuildKernelCache(&qt);  // pack.cpp:107-117
  return qt;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// cpu_features.cpp: HostIsa / CurrentIsa / IsaToString.
const char* ref_host_isa() {
  static std::string s;
  s = std::string(esm::IsaToString(esm::HostIsa()));
  return s.c_str();
}
const char* ref_current_isa() {
  static std::string s;
  s = std::string(esm::IsaToString(esm::CurrentIsa()));
  return s.c_str();
}
// ESM_FORCE_ISA is re-read on every CurrentIsa() call (cpu_features.h:29-32).
void ref_force_isa(const char* isa) {
  if (isa == nullptr || *isa == '\0') {
    unsetenv("ESM_FORCE_ISA");
  } else {
    setenv("ESM_FORCE_ISA", isa, 1);
  }
}
int ref_num_threads() { return static_cast<int>(esm::GlobalPool().size()); }

// ---- kernel facade (include/esm_cpp/kernels.h) ----------------------------
int ref_linear_f32(const float* A, const float* W, const float* bias, float* C,
                   int M, int N, int K) {
  return Guard([&] { esm::kernels::Linear(A, W, bias, C, M, N, K); });
}
int ref_linear_f32_ref(const float* A, const float* W, const float* bias,
                       float* C, int M, int N, int K) {
  return Guard([&] { esm::kernels::LinearRef(A, W, bias, C, M, N, K); });
}
// dispatch.cpp:80-103 (AMX / VNNI / Ref by CurrentIsa()).
int ref_linear_int8(const float* A, const std::int8_t* packed, const float* scales,
                    const float* bias, float* C, int M, int N, int K) {
  return Guard([&] {
    auto qt = MakeQt(packed, scales, N, K);
    esm::kernels::LinearInt8(A, qt, bias, C, M, N, K);
  });
}
// gemm_int8.cpp:510-555: one per-tensor activation scale over all M rows.
int ref_linear_int8_vnni(const float* A, const std::int8_t* packed,
                         const float* scales, const float* bias, float* C,
                         int M, int N, int K) {
  return Guard([&] {
    auto qt = MakeQt(packed, scales, N, K);
    esm::kernels::LinearVnni(A, qt, bias, C, M, N, K);
  });
}
// gemm_amx.cpp:218-309 (M%32 tail re-quantised with its own scale).
int ref_linear_int8_amx(const float* A, const std::int8_t* packed,
                        const float* scales, const float* bias, float* C,
                        int M, int N, int K) {
  return Guard([&] {
    auto qt = MakeQt(packed, scales, N, K);
    esm::kernels::LinearAmx(A, qt, bias, C, M, N, K);
  });
}
// gemm_int8.cpp:49-64 (W8A16 scalar twin).
int ref_linear_int8_ref(const float* A, const std::int8_t* packed,
                        const float* scales, const float* bias, float* C, int M,
                        int N, int K) {
  return Guard([&] {
    auto qt = MakeQt(packed, scales, N, K);
    esm::kernels::LinearInt8Ref(A, qt, bias, C, M, N, K);
  });
}
// pack.cpp:149-177.
int ref_quantize_weights(const float* W, int N, int K, std::int8_t* packed_out,
                         float* scales_out) {
  return Guard([&] {
    esm::quant::QuantizedTensor qt;
    esm::quant::Quantize(W, N, K, &qt);
    std::memcpy(packed_out, qt.packed.data(), qt.packed.size());
    std::memcpy(scales_out, qt.per_channel_scales.data(),
                qt.per_channel_scales.size() * sizeof(float));
  });
}
// pack.cpp:119-132 / 134-147.
int ref_quantize_act(const float* x, std::size_t n, float scale, std::uint8_t* q) {
  return Guard([&] { esm::quant::QuantizeActivationRef(x, n, scale, q); });
}
int ref_quantize_act_sym(const float* x, std::size_t n, float scale,
                         std::int8_t* q) {
  return Guard([&] { esm::quant::QuantizeActivationSymmetricRef(x, n, scale, q); });
}
// gemm_int8.cpp:391-508: global absmax -> scale -> u8 (zero point 128).
int ref_quant_act_prefix(const float* A, std::size_t MK, std::uint8_t* q,
                         float* scale_out) {
  return Guard([&] { esm::kernels::QuantizeActPrefixAvx512(A, MK, q, scale_out); });
}
int ref_layernorm(const float* x, const float* g, const float* b, float eps,
                  float* out, int rows, int d) {
  return Guard([&] { esm::kernels::LayerNorm(x, g, b, eps, out, rows, d); });
}
int ref_layernorm_ref(const float* x, const float* g, const float* b, float eps,
                      float* out, int rows, int d) {
  return Guard([&] { esm::kernels::LayerNormRef(x, g, b, eps, out, rows, d); });
}
int ref_gelu(const float* x, float* out, std::size_t n) {
  return Guard([&] { esm::kernels::Gelu(x, out, n); });
}
int ref_gelu_ref(const float* x, float* out, std::size_t n) {
  return Guard([&] { esm::kernels::GeluRef(x, out, n); });
}
int ref_residual_add(float* y, const float* x, std::size_t n) {
  return Guard([&] { esm::kernels::ResidualAddInplace(y, x, n); });
}
int ref_scale(float* x, std::size_t n, float s) {
  return Guard([&] { esm::kernels::ScaleInplace(x, n, s); });
}
int ref_rope_build_tables(int L, int dh, float* cos, float* sin) {
  return Guard([&] { esm::kernels::RopeBuildTables(L, dh, cos, sin); });
}
int ref_rope_apply_varlen(float* x, const float* cos, const float* sin,
                          const int* cu, int B, int H, int dh) {
  return Guard([&] { esm::kernels::RopeApplyVarlen(x, cos, sin, cu, B, H, dh); });
}
int ref_rope_apply_varlen_ref(float* x, const float* cos, const float* sin,
                              const int* cu, int B, int H, int dh) {
  return Guard(
      [&] { esm::kernels::RopeApplyVarlenRef(x, cos, sin, cu, B, H, dh); });
}
int ref_attention_varlen(const float* q, const float* k, const float* v,
                         const int* cu, int B, int H, int dh, float* out) {
  return Guard(
      [&] { esm::kernels::AttentionVarlen(q, k, v, cu, B, H, dh, out); });
}
int ref_attention_varlen_ref(const float* q, const float* k, const float* v,
                             const int* cu, int B, int H, int dh, float* out) {
  return Guard(
      [&] { esm::kernels::AttentionVarlenRef(q, k, v, cu, B, H, dh, out); });
}

// ---- scheduler (scheduler.cpp:54-75) --------------------------------------
// Writes the plan as a flat list of caller indices (order_out[n]) plus the
// size of each group (group_sizes_out[<= n]); returns the group count.
int ref_plan_batches(const int* lengths, int n, float threshold, int max_batch,
                     int* order_out, int* group_sizes_out) {
  int groups = -1;
  Guard([&] {
    esm::SchedulerConfig cfg;
    cfg.imbalance_threshold = threshold;
    cfg.max_batch_size = max_batch;
    std::vector<int> lens(lengths, lengths + n);
    auto plan = esm::PlanBatches(lens, cfg);
    int pos = 0;
    for (std::size_t g = 0; g < plan.size(); ++g) {
      group_sizes_out[g] = static_cast<int>(plan[g].size());
      for (int idx : plan[g]) order_out[pos++] = idx;
    }
    groups = static_cast<int>(plan.size());
  });
  return groups;
}

// BatchView validation (batch.cpp:8-45): 0 when valid, -1 with the message.
int ref_batch_view_check(const int* ids, int T, const int* masks, int n_masks,
                         const int* cu, int n_cu, int B) {
  return Guard([&] {
    esm::BatchView v(std::span<const std::int32_t>(ids, static_cast<std::size_t>(T)),
                     std::span<const std::int32_t>(masks, static_cast<std::size_t>(n_masks)),
                     std::span<const std::int32_t>(cu, static_cast<std::size_t>(n_cu)), B);
    (void)v;
  });
}

// ---- model (model.h / model.cpp) ------------------------------------------
void* ref_model_load(const char* path) {
  esm::Model* out = nullptr;
  Guard([&] { out = esm::Model::Load(path).release(); });  // model.cpp:300-303
  return out;
}
void ref_model_free(void* m) { delete static_cast<esm::Model*>(m); }

// [layers, hidden, heads, head_dim, ffn, vocab, quantized]
int ref_model_config(void* m, int* out7) {
  return Guard([&] {
    const auto& c = static_cast<esm::Model*>(m)->config();
    out7[0] = c.num_hidden_layers;
    out7[1] = c.hidden_size;
    out7[2] = c.num_attention_heads;
    out7[3] = c.head_dim;
    out7[4] = c.intermediate_size;
    out7[5] = c.vocab_size;
    out7[6] = c.weights_quantized ? 1 : 0;
  });
}

// Model::ForwardPacked (model.cpp:1291-1296 -> 1093-1255). logits_out is the
// packed [T, V] buffer (per-sequence outputs concatenated in pack order).
int ref_model_forward_packed(void* m, const int* ids, const int* masks, int T,
                             const int* cu, int B, float* logits_out) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    std::span<const std::int32_t> ids_s(ids, static_cast<std::size_t>(T));
    std::span<const std::int32_t> masks_s;
    if (masks) masks_s = std::span<const std::int32_t>(masks, static_cast<std::size_t>(T));
    std::span<const std::int32_t> cu_s(cu, static_cast<std::size_t>(B) + 1);
    esm::BatchView view(ids_s, masks_s, cu_s, B);
    auto outs = model->ForwardPacked(view);
    std::size_t off = 0;
    for (auto& o : outs) {
      std::memcpy(logits_out + off, o.data(), o.size() * sizeof(float));
      off += o.size();
    }
  });
}

// Model::ForwardScheduled (model.cpp:1298-1421). Inputs are concatenated
// with per-sequence lengths; outputs concatenated in caller order.
int ref_model_forward_scheduled(void* m, const int* ids_concat, const int* lens,
                                int n, float threshold, int max_batch,
                                float* logits_out) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    std::vector<std::vector<std::int32_t>> ids(static_cast<std::size_t>(n));
    std::size_t off = 0;
    for (int i = 0; i < n; ++i) {
      ids[static_cast<std::size_t>(i)].assign(ids_concat + off, ids_concat + off + lens[i]);
      off += static_cast<std::size_t>(lens[i]);
    }
    esm::SchedulerConfig cfg;
    cfg.imbalance_threshold = threshold;
    cfg.max_batch_size = max_batch;
    auto outs = model->ForwardScheduled(ids, {}, cfg);
    std::size_t o = 0;
    for (auto& v : outs) {
      std::memcpy(logits_out + o, v.data(), v.size() * sizeof(float));
      o += v.size();
    }
  });
}

// Model::ForwardWithHiddenStates (model.cpp:Forward*): writes the N+1 hidden
// states [N+1, L, d] for one sequence plus its logits [L, V].
int ref_model_forward_hidden(void* m, const int* ids, int L, float* logits_out,
                             float* hidden_out) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    std::vector<std::vector<float>> hs;
    auto logits = model->ForwardWithHiddenStates(
        std::span<const std::int32_t>(ids, static_cast<std::size_t>(L)), {},
        hidden_out ? &hs : nullptr);
    std::memcpy(logits_out, logits.data(), logits.size() * sizeof(float));
    if (hidden_out) {
      std::size_t off = 0;
      for (auto& h : hs) {
        std::memcpy(hidden_out + off, h.data(), h.size() * sizeof(float));
        off += h.size();
      }
    }
  });
}

// The calibrate -> migrate recipe of python/esm_cpp/quantize.py:35-91:
// ForwardWithObserver over each calibration sequence, Percentile(pctile),
// then ApplySmoothQuant(stats, alpha) (smoothquant.cpp:100-185).
int ref_model_calibrate_smoothquant(void* m, const int* ids_concat,
                                    const int* lens, int n, float pctile,
                                    float alpha) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    esm::ActivationObserver obs;
    std::size_t off = 0;
    for (int i = 0; i < n; ++i) {
      model->ForwardWithObserver(
          std::span<const std::int32_t>(ids_concat + off, static_cast<std::size_t>(lens[i])),
          {}, &obs);
      off += static_cast<std::size_t>(lens[i]);
    }
    model->ApplySmoothQuant(obs.Percentile(pctile), alpha);
  });
}

// ActivationObserver (observer.h:14-44, observer.cpp:8-51) as a handle.
void* ref_observer_new() { return new esm::ActivationObserver(); }
void ref_observer_free(void* o) { delete static_cast<esm::ActivationObserver*>(o); }
int ref_observer_observe(void* o, const char* key, const float* values, std::size_t n) {
  return Guard([&] { static_cast<esm::ActivationObserver*>(o)->Observe(key, values, n); });
}
// Percentile of one site; -1 with an error when the site was never observed.
int ref_observer_percentile(void* o, const char* key, float pctile, float* out) {
  return Guard([&] {
    auto p = static_cast<esm::ActivationObserver*>(o)->Percentile(pctile);
    auto it = p.find(key);
    if (it == p.end()) throw std::runtime_error(std::string("no site ") + key);
    *out = it->second;
  });
}

// python/esm_cpp/quantize.py:35-47 (calibrate): ForwardWithObserver over each
// sequence, then Percentile(pctile); stats_out[layer * 4 + site] with sites
// attn_ln_output, attn_out, ffn_ln_output, inter_gelu (model.cpp:952-1050).
int ref_model_observe(void* m, const int* ids_concat, const int* lens, int n, float pctile,
                      float* stats_out) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    esm::ActivationObserver obs;
    std::size_t off = 0;
    for (int i = 0; i < n; ++i) {
      model->ForwardWithObserver(
          std::span<const std::int32_t>(ids_concat + off, static_cast<std::size_t>(lens[i])),
          {}, &obs);
      off += static_cast<std::size_t>(lens[i]);
    }
    auto p = obs.Percentile(pctile);
    static const char* kSites[4] = {"attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu"};
    const int L = model->config().num_hidden_layers;
    for (int li = 0; li < L; ++li)
      for (int j = 0; j < 4; ++j) {
        auto it = p.find("layer" + std::to_string(li) + "." + kSites[j]);
        stats_out[li * 4 + j] = it == p.end() ? 0.0f : it->second;
      }
  });
}

// Model::ApplySmoothQuant (model.cpp:1462-1468 -> smoothquant.cpp:100-185)
// with the statistics given as stats[layer * 4 + site] (sites as above).
int ref_model_apply_smoothquant(void* m, const float* stats, float alpha) {
  return Guard([&] {
    auto* model = static_cast<esm::Model*>(m);
    static const char* kSites[4] = {"attn_ln_output", "attn_out", "ffn_ln_output", "inter_gelu"};
    std::unordered_map<std::string, float> act;
    const int L = model->config().num_hidden_layers;
    for (int li = 0; li < L; ++li)
      for (int j = 0; j < 4; ++j) act["layer" + std::to_string(li) + "." + kSites[j]] = stats[li * 4 + j];
    model->ApplySmoothQuant(act, alpha);
  });
}

int ref_model_quantize(void* m) {  // model.cpp:1470-1494
  return Guard([&] { static_cast<esm::Model*>(m)->QuantizeWeights(); });
}
int ref_model_save_gguf(void* m, const char* path) {  // model.cpp:562-725
  return Guard([&] { static_cast<esm::Model*>(m)->SaveToGguf(path); });
}

}  // extern "C"

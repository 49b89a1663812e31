// C ABI: context management and the kernel facade (device pointers).
// Each esmcu_* facade function replaces the esm::kernels function of the
// reference named in include/esm_b200.h and enqueues on the context stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../kernels.cuh"
#include "context.h"
#include "esm_b200.h"

namespace esmb200 {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return ESMCU_ERR_CUDA;
}

int use_device(esmcu_context* ctx) {
  if (ctx == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null context");
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != ctx->device) {
    ESMCU_CUDA(cudaSetDevice(ctx->device));
  }
  return ESMCU_OK;
}

bool attention_bf16_enabled(int head_dim) {
  if (head_dim % 32 != 0) return false;  // attention.cpp:695: FP32 otherwise
  const char* v = std::getenv("ESM_AMX_ATTENTION");
  if (v == nullptr) return false;
  const std::string s = v;
  return s == "on" || s == "1" || s == "true";
}

int ensure_scratch(esmcu_context* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return ESMCU_OK;
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  if (ctx->scratch) ESMCU_CUDA(cudaFree(ctx->scratch));
  ctx->scratch = nullptr;
  ctx->scratch_bytes = 0;
  const size_t want = align_up(bytes, 1 << 20);
  ESMCU_CUDA(cudaMalloc(&ctx->scratch, want));
  ctx->scratch_bytes = want;
  return ESMCU_OK;
}

int check_device_status(esmcu_context* ctx) {
  uint32_t st = 0;
  ESMCU_CUDA(cudaMemcpy(&st, ctx->d_status, sizeof(st), cudaMemcpyDeviceToHost));
  if (st != 0) {
    ESMCU_CUDA(cudaMemset(ctx->d_status, 0, sizeof(uint32_t)));
    return fail(ESMCU_ERR_TIMEOUT,
                "a device-side wait ran past its bound (status 0x" + std::to_string(st) + ")");
  }
  return ESMCU_OK;
}

}  // namespace esmb200

using namespace esmb200;

namespace {

int check_ptr(const void* p, const char* name) {
  if (p == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
  return ESMCU_OK;
}

#define ESMCU_TRY(x)           \
  do {                         \
    int rc_ = (x);             \
    if (rc_ != ESMCU_OK) return rc_; \
  } while (0)

}  // namespace

extern "C" {

const char* esmcu_last_error(void) {
  static thread_local std::string copy;
  copy = esmb200::g_last_error;
  return copy.c_str();
}

const char* esmcu_version(void) { return "esm_b200 0.1.0 (sm_100a)"; }

int esmcu_device_count(int* count) {
  if (count == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "count is null");
  *count = 0;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  return ESMCU_OK;
}

int esmcu_open(int device, esmcu_context** out) {
  if (out == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
    return fail(ESMCU_ERR_NO_DEVICE, "no CUDA device is visible");
  if (device < 0 || device >= n)
    return fail(ESMCU_ERR_OUT_OF_RANGE, "device " + std::to_string(device) + " out of range");
  ESMCU_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  ESMCU_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(ESMCU_ERR_NO_DEVICE, std::string("device is not sm_100 (B200): ") + prop.name);
  auto* ctx = new esmcu_context();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(uint32_t));
  if (e != cudaSuccess) {
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return cuda_fail(e, "esmcu_open");
  }
  // The no-alloc entry point's fixed scratch is committed here, on this
  // device, so that its first call allocates nothing.
  if (noalloc_prepare() != ESMCU_OK) {
    const std::string msg = esmcu_last_error();
    cudaFree(ctx->d_status);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return fail(ESMCU_ERR_CUDA, "esmcu_open: " + msg);
  }
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return ESMCU_OK;
}

int esmcu_close(esmcu_context* ctx) {
  if (ctx == nullptr) return ESMCU_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return ESMCU_OK;
}

int esmcu_set_stream(esmcu_context* ctx, void* stream) {
  ESMCU_TRY(use_device(ctx));
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return ESMCU_OK;
}

void* esmcu_get_stream(esmcu_context* ctx) { return ctx ? ctx->stream : nullptr; }

int esmcu_set_math_mode(esmcu_context* ctx, int mode) {
  if (ctx == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null context");
  if (mode != ESMCU_MATH_DEFAULT && mode != ESMCU_MATH_AVX512)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad math mode");
  ctx->math_mode = mode;
  return ESMCU_OK;
}

int esmcu_get_math_mode(const esmcu_context* ctx, int* mode) {
  if (ctx == nullptr || mode == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "null argument");
  *mode = ctx->math_mode;
  return ESMCU_OK;
}

int esmcu_synchronize(esmcu_context* ctx) {
  ESMCU_TRY(use_device(ctx));
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  return check_device_status(ctx);
}

int esmcu_malloc(esmcu_context* ctx, size_t bytes, void** dptr) {
  ESMCU_TRY(use_device(ctx));
  ESMCU_TRY(check_ptr(dptr, "dptr"));
  ESMCU_CUDA(cudaMalloc(dptr, bytes));
  return ESMCU_OK;
}
int esmcu_free(esmcu_context* ctx, void* dptr) {
  ESMCU_TRY(use_device(ctx));
  ESMCU_CUDA(cudaFree(dptr));
  return ESMCU_OK;
}
int esmcu_memcpy_h2d(esmcu_context* ctx, void* dst, const void* src, size_t bytes) {
  ESMCU_TRY(use_device(ctx));
  ESMCU_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  return ESMCU_OK;
}
int esmcu_memcpy_d2h(esmcu_context* ctx, void* dst, const void* src, size_t bytes) {
  ESMCU_TRY(use_device(ctx));
  ESMCU_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  return ESMCU_OK;
}

// ------------------------------------------------------------------ facade
int esmcu_linear(esmcu_context* ctx, const float* A, const float* W, const float* bias, float* C,
                 int M, int N, int K) {
  ESMCU_TRY(use_device(ctx));
  if (M < 0 || N < 0 || K < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "negative shape");
  if (M == 0 || N == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(A, "A"));
  ESMCU_TRY(check_ptr(W, "W"));
  ESMCU_TRY(check_ptr(C, "C"));
  EpiParams epi;
  epi.kind = kEpiStore;
  epi.C = C;
  epi.ldc = N;
  // 3xTF32 on the tensor cores when K and the operands allow 16-byte TMA
  // rows (the lo parts of A and W go to the context scratch); FP32 SIMT
  // otherwise.
  const bool tc = (K % 4 == 0) &&
                  ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W)) & 15) == 0;
  if (tc) {
    const size_t na = static_cast<size_t>(M) * K, nw = static_cast<size_t>(N) * K;
    const size_t off_w = align_up(na * sizeof(float), 256);
    ESMCU_TRY(ensure_scratch(ctx, off_w + nw * sizeof(float)));
    float* a_lo = static_cast<float*>(ctx->scratch);
    float* w_lo = reinterpret_cast<float*>(static_cast<char*>(ctx->scratch) + off_w);
    ESMCU_CUDA(launch_tf32_lo(A, a_lo, static_cast<long>(na), ctx->stream));
    ESMCU_CUDA(launch_tf32_lo(W, w_lo, static_cast<long>(nw), ctx->stream));
    GemmTf32Args g;
    g.A = A;
    g.A_lo = a_lo;
    g.lda = K;
    g.W = W;
    g.W_lo = w_lo;
    g.ldw = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.epi = epi;
    g.status = ctx->d_status;
    g.num_sms = ctx->num_sms;
    ESMCU_CUDA(launch_gemm_tf32x3(g, ctx->stream));
    return ESMCU_OK;
  }
  GemmF32Args a;
  a.A = A;
  a.lda = K;
  a.W = W;
  a.ldw = K;
  a.M = M;
  a.N = N;
  a.K = K;
  a.bias = bias;
  a.epi = epi;
  ESMCU_CUDA(launch_gemm_f32(a, ctx->stream));
  return ESMCU_OK;
}

int esmcu_quantize_activations(esmcu_context* ctx, const float* A, int M, int K, int8_t* q_out,
                               int ldq, float* scales_out, int act_quant) {
  ESMCU_TRY(use_device(ctx));
  if (M < 0 || K <= 0 || ldq < K || (ldq % 16) != 0)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad shape: need K > 0, ldq >= K, ldq % 16 == 0");
  if (M == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(A, "A"));
  ESMCU_TRY(check_ptr(q_out, "q_out"));
  ESMCU_TRY(check_ptr(scales_out, "scales_out"));
  if (act_quant == ESMCU_ACT_PER_TOKEN) {
    ESMCU_CUDA(launch_quantize_per_token(A, K, M, K, q_out, ldq, scales_out, ctx->stream));
    return ESMCU_OK;
  }
  if (act_quant != ESMCU_ACT_PER_TENSOR) return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad act_quant");
  ESMCU_TRY(ensure_scratch(ctx, kAmaxSlots * sizeof(uint32_t)));
  uint32_t* amax = static_cast<uint32_t*>(ctx->scratch);
  ESMCU_CUDA(cudaMemsetAsync(amax, 0, kAmaxSlots * sizeof(uint32_t), ctx->stream));
  ESMCU_CUDA(launch_absmax(A, static_cast<long>(M) * K, amax, ctx->stream));
  ESMCU_CUDA(launch_quantize_per_tensor(A, K, M, K, amax, q_out, ldq, scales_out, ctx->stream));
  return ESMCU_OK;
}

int esmcu_quantize_weights(esmcu_context* ctx, const float* W, int N, int K, int8_t* q,
                           float* scales) {
  ESMCU_TRY(use_device(ctx));
  if (N < 0 || K < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad shape");
  if (N == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(scales, "scales"));
  if (K == 0) {  // every row is all-zero: scale 0
    ESMCU_CUDA(cudaMemsetAsync(scales, 0, static_cast<size_t>(N) * sizeof(float), ctx->stream));
    return ESMCU_OK;
  }
  ESMCU_TRY(check_ptr(W, "W"));
  ESMCU_TRY(check_ptr(q, "q"));
  ESMCU_CUDA(launch_quantize_weights(W, N, K, q, K, scales, ctx->stream));
  return ESMCU_OK;
}

int esmcu_gemm_int8_s32(esmcu_context* ctx, const int8_t* q, int ldq, const int8_t* W, int ldw,
                        int32_t* acc, int M, int N, int K) {
  ESMCU_TRY(use_device(ctx));
  if (M < 0 || N < 0 || K <= 0 || (K % 16) || (ldq % 16) || (ldw % 16) || ldq < K || ldw < K)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "K, ldq, ldw must be multiples of 16 (>= K)");
  if (M == 0 || N == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(q, "q"));
  ESMCU_TRY(check_ptr(W, "W"));
  ESMCU_TRY(check_ptr(acc, "acc"));
  GemmI8Args a;
  a.A = q;
  a.lda = ldq;
  a.W = W;
  a.ldw = ldw;
  a.M = M;
  a.N = N;
  a.K = K;
  a.acc_out = acc;
  a.status = ctx->d_status;
  a.num_sms = ctx->num_sms;
  ESMCU_CUDA(launch_gemm_i8(a, ctx->stream));
  return ESMCU_OK;
}

int esmcu_linear_int8(esmcu_context* ctx, const float* A, const int8_t* W, const float* w_scales,
                      const float* bias, float* C, int M, int N, int K, int act_quant) {
  ESMCU_TRY(use_device(ctx));
  if (M < 0 || N < 0 || K < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "negative shape");
  if (M == 0 || N == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(A, "A"));
  ESMCU_TRY(check_ptr(W, "W"));
  ESMCU_TRY(check_ptr(w_scales, "w_scales"));
  ESMCU_TRY(check_ptr(C, "C"));
  if (act_quant != ESMCU_ACT_PER_TENSOR && act_quant != ESMCU_ACT_PER_TOKEN)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad act_quant");
  if (K == 0) {  // gemm_int8.cpp:512-519: K <= 0 zeroes C
    ESMCU_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(M) * N, ctx->stream));
    return ESMCU_OK;
  }
  const long ldq = static_cast<long>(align_up(static_cast<size_t>(K), 16));
  const bool pad_w = (ldq != K) || (reinterpret_cast<uintptr_t>(W) & 15);
  // Scratch layout: [amax slots 256B][scales M*4 -> 256-aligned][q M*ldq][padded W N*ldq]
  const size_t off_scales = kAmaxSlots * sizeof(uint32_t);
  const size_t off_q = align_up(off_scales + sizeof(float) * static_cast<size_t>(M), 256);
  const size_t off_w = align_up(off_q + static_cast<size_t>(M) * ldq, 256);
  const size_t total = off_w + (pad_w ? static_cast<size_t>(N) * ldq : 0);
  ESMCU_TRY(ensure_scratch(ctx, total));
  char* base = static_cast<char*>(ctx->scratch);
  uint32_t* amax = reinterpret_cast<uint32_t*>(base);
  float* scales = reinterpret_cast<float*>(base + off_scales);
  int8_t* q = reinterpret_cast<int8_t*>(base + off_q);
  const int8_t* w_dev = W;
  if (pad_w) {
    int8_t* wp = reinterpret_cast<int8_t*>(base + off_w);
    ESMCU_CUDA(cudaMemsetAsync(wp, 0, static_cast<size_t>(N) * ldq, ctx->stream));
    ESMCU_CUDA(cudaMemcpy2DAsync(wp, ldq, W, K, K, N, cudaMemcpyDeviceToDevice, ctx->stream));
    w_dev = wp;
  }
  if (act_quant == ESMCU_ACT_PER_TOKEN) {
    ESMCU_CUDA(launch_quantize_per_token(A, K, M, K, q, ldq, scales, ctx->stream));
  } else {
    ESMCU_CUDA(cudaMemsetAsync(amax, 0, kAmaxSlots * sizeof(uint32_t), ctx->stream));
    ESMCU_CUDA(launch_absmax(A, static_cast<long>(M) * K, amax, ctx->stream));
    ESMCU_CUDA(launch_quantize_per_tensor(A, K, M, K, amax, q, ldq, scales, ctx->stream));
  }
  GemmI8Args a;
  a.A = q;
  a.lda = ldq;
  a.W = w_dev;
  a.ldw = ldq;
  a.M = M;
  a.N = N;
  a.K = static_cast<int>(ldq);
  a.w_scale = w_scales;
  a.a_scale = scales;
  a.per_token = act_quant == ESMCU_ACT_PER_TOKEN;
  a.bias = bias;
  a.epi.kind = kEpiStore;
  a.epi.C = C;
  a.epi.ldc = N;
  a.status = ctx->d_status;
  a.num_sms = ctx->num_sms;
  ESMCU_CUDA(launch_gemm_i8(a, ctx->stream));
  return ESMCU_OK;
}

int esmcu_layernorm(esmcu_context* ctx, const float* x, const float* gamma, const float* beta,
                    float eps, float* out, int num_rows, int d) {
  ESMCU_TRY(use_device(ctx));
  if (num_rows < 0 || d <= 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad shape");
  if (num_rows == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(x, "x"));
  ESMCU_TRY(check_ptr(gamma, "gamma"));
  ESMCU_TRY(check_ptr(beta, "beta"));
  ESMCU_TRY(check_ptr(out, "out"));
  if (ctx->math_mode == ESMCU_MATH_AVX512) {
    if (d % 16 != 0)
      return fail(ESMCU_ERR_INVALID_ARGUMENT, "the AVX-512 math mode needs d % 16 == 0");
    ESMCU_CUDA(launch_layernorm_avx(x, gamma, beta, eps, out, num_rows, d, nullptr, ctx->stream));
    return ESMCU_OK;
  }
  ESMCU_CUDA(launch_layernorm(x, gamma, beta, eps, out, num_rows, d, nullptr, nullptr, 0, nullptr,
                              ctx->stream));
  return ESMCU_OK;
}

int esmcu_gelu(esmcu_context* ctx, const float* x, float* out, size_t n) {
  ESMCU_TRY(use_device(ctx));
  if (n == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(x, "x"));
  ESMCU_TRY(check_ptr(out, "out"));
  if (ctx->math_mode == ESMCU_MATH_AVX512) {
    ESMCU_CUDA(launch_gelu_avx(x, out, static_cast<long>(n), nullptr, ctx->stream));
    return ESMCU_OK;
  }
  ESMCU_CUDA(launch_gelu(x, out, static_cast<long>(n), ctx->stream));
  return ESMCU_OK;
}

int esmcu_residual_add_inplace(esmcu_context* ctx, float* y, const float* x, size_t n) {
  ESMCU_TRY(use_device(ctx));
  if (n == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(y, "y"));
  ESMCU_TRY(check_ptr(x, "x"));
  ESMCU_CUDA(launch_residual_add(y, x, static_cast<long>(n), ctx->stream));
  return ESMCU_OK;
}

int esmcu_scale_inplace(esmcu_context* ctx, float* x, size_t n, float scale) {
  ESMCU_TRY(use_device(ctx));
  if (n == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(x, "x"));
  ESMCU_CUDA(launch_scale(x, static_cast<long>(n), scale, ctx->stream));
  return ESMCU_OK;
}

int esmcu_rope_apply_varlen(esmcu_context* ctx, float* x, const float* cos_t, const float* sin_t,
                            const int* cu, int B, int H, int dh) {
  ESMCU_TRY(use_device(ctx));
  if (B < 0 || H <= 0 || dh <= 0 || (dh & 1)) return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad shape");
  if (B == 0) return ESMCU_OK;
  ESMCU_TRY(check_ptr(x, "x"));
  ESMCU_TRY(check_ptr(cu, "cu_seqlens"));
  ESMCU_CUDA(launch_rope_varlen(x, cos_t, sin_t, cu, B, H, dh, ctx->stream));
  return ESMCU_OK;
}

int esmcu_attention_varlen(esmcu_context* ctx, const float* q, const float* k, const float* v,
                           const int* cu, int B, int H, int dh, float* out) {
  ESMCU_TRY(use_device(ctx));
  if (B < 0 || H <= 0 || dh <= 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad shape");
  if (B == 0) return ESMCU_OK;
  if (dh > 128 || (dh % 4) != 0)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "head_dim must be a multiple of 4 and <= 128");
  ESMCU_TRY(check_ptr(q, "q"));
  ESMCU_TRY(check_ptr(k, "k"));
  ESMCU_TRY(check_ptr(v, "v"));
  ESMCU_TRY(check_ptr(cu, "cu_seqlens"));
  ESMCU_TRY(check_ptr(out, "out"));
  // The sequence lengths decide the kernels (one per length class), so read
  // cu_seqlens back once.
  std::vector<int> cu_h(static_cast<size_t>(B) + 1);
  ESMCU_CUDA(cudaMemcpyAsync(cu_h.data(), cu, cu_h.size() * sizeof(int), cudaMemcpyDeviceToHost,
                             ctx->stream));
  ESMCU_CUDA(cudaStreamSynchronize(ctx->stream));
  int max_len = 0, min_len = cu_h[1] - cu_h[0];
  for (int b = 0; b < B; ++b) {
    max_len = std::max(max_len, cu_h[b + 1] - cu_h[b]);
    min_len = std::min(min_len, cu_h[b + 1] - cu_h[b]);
  }
  if (ctx->math_mode == ESMCU_MATH_AVX512) {
    if (dh != 16 && dh != 32 && dh != 64)
      return fail(ESMCU_ERR_INVALID_ARGUMENT, "the AVX-512 math mode needs head_dim 16, 32 or 64");
    if (max_len == 0) return ESMCU_OK;
    ESMCU_CUDA(launch_attention_avx(q, k, v, cu, B, H, dh, cu_h[B], max_len, out, nullptr,
                                    ctx->stream));
    return ESMCU_OK;
  }
  const bool qk_bf16 = attention_bf16_enabled(dh);
  if (qk_bf16) {
    // The caller's q and k stay untouched: bf16-rounded copies in scratch.
    const size_t n = static_cast<size_t>(cu_h[B]) * H * dh;
    ESMCU_TRY(ensure_scratch(ctx, 2 * n * sizeof(float)));
    float* qb = static_cast<float*>(ctx->scratch);
    float* kb = qb + n;
    ESMCU_CUDA(launch_round_bf16(q, qb, static_cast<long>(n), ctx->stream));
    ESMCU_CUDA(launch_round_bf16(k, kb, static_cast<long>(n), ctx->stream));
    q = qb;
    k = kb;
  }
  ESMCU_CUDA(launch_attention_varlen(q, k, v, cu, B, H, dh, cu_h[B], min_len, max_len, out, nullptr,
                                     ctx->d_status, ctx->num_sms, ctx->stream, qk_bf16));
  return ESMCU_OK;
}

}  // extern "C"

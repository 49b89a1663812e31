// esmcu_linear_int8_noalloc: the W8A8 Linear (esmcu_linear_int8) for callers
// that cannot let the library allocate device memory.
//
// Who needs it: a process that hands all free HBM to its own pool at start-up
// (a serving stack with a fixed memory budget) has nothing left for the
// library's scratch to grow into, and a latency-critical caller cannot accept
// the device-wide synchronisation that cudaMalloc / cudaFree imply when the
// scratch grows mid-stream.  This entry point never allocates: its scratch
// (absmax slots, activation scales, the quantised activations and, for
// K % 16 != 0, a padded copy of W) lives in one fixed array compiled into the
// library, which every GPU that loads the library holds until the process
// exits.
//
// Limits and sharing: the scratch holds kNoAllocScratchBytes (16 MiB), so
// 256 + 4*M (rounded up to 256) + M*ldq bytes, plus N*ldq more when K % 16 != 0
// or W is not 16-byte aligned (W is then copied to padded rows), must fit,
// ldq = K rounded up to 16; larger calls are rejected with
// ESMCU_ERR_OUT_OF_RANGE.  Every call on a device shares the one array, and
// it keeps the last call's contents: the absmax slots are cleared by each
// call, and calls that overlap on the GPU (different streams, or different
// host threads on the same device) race on it -- serialise them.
//
// Set-up: esmcu_open calls noalloc_prepare for its device, with that device
// current.  Looking the array's address up (cudaGetSymbolAddress) loads this
// file's module, which is when the driver commits the 16 MiB; doing it at
// open time means the first noalloc call neither allocates nor waits for a
// module load, even under lazy module loading.  Each call looks the address
// up again (cheap once the module is loaded) instead of caching it, so a
// context torn down and re-created by the caller gets the current address.
#include <cuda_runtime.h>

#include <string>

#include "host/context.h"
#include "kernels.cuh"

namespace esmb200 {

constexpr size_t kNoAllocScratchBytes = 16u << 20;

// The scratch array itself (file scope, one copy per device).  In host code
// `g_noalloc_scratch` names a host-side stand-in, not device memory: kernels
// only ever receive the device address looked up below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

// Device address of the scratch on the current device; nullptr with the
// error recorded on failure.
void* scratch_address() {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_error(std::string("esmcu_linear_int8_noalloc: cudaGetSymbolAddress: ") +
              cudaGetErrorString(e));
    return nullptr;
  }
  return p;
}

}  // namespace

// Called by esmcu_open with the context's device current: loads the module
// that holds the scratch array (committing its memory now, not at the first
// noalloc call).
int noalloc_prepare() { return scratch_address() != nullptr ? ESMCU_OK : ESMCU_ERR_CUDA; }

}  // namespace esmb200

using namespace esmb200;

extern "C" int esmcu_linear_int8_noalloc(esmcu_context* ctx, const float* A, const int8_t* W,
                                         const float* w_scales, const float* bias, float* C,
                                         int M, int N, int K, int act_quant) {
  int rc = use_device(ctx);
  if (rc != ESMCU_OK) return rc;
  // The same checks, in the same order, as esmcu_linear_int8.
  if (M < 0 || N < 0 || K < 0) return fail(ESMCU_ERR_INVALID_ARGUMENT, "negative shape");
  if (M == 0 || N == 0) return ESMCU_OK;
  if (A == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "A is null");
  if (W == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "W is null");
  if (w_scales == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "w_scales is null");
  if (C == nullptr) return fail(ESMCU_ERR_INVALID_ARGUMENT, "C is null");
  if (act_quant != ESMCU_ACT_PER_TENSOR && act_quant != ESMCU_ACT_PER_TOKEN)
    return fail(ESMCU_ERR_INVALID_ARGUMENT, "bad act_quant");
  if (K == 0) {  // gemm_int8.cpp:512-519: K <= 0 zeroes C
    ESMCU_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(M) * N, ctx->stream));
    return ESMCU_OK;
  }
  const size_t ldq = align_up(static_cast<size_t>(K), 16);
  const bool pad_w = (ldq != static_cast<size_t>(K)) || (reinterpret_cast<uintptr_t>(W) & 15);
  // Layout: [absmax slots 256 B][scales 4*M -> 256-aligned][q M*ldq -> 256-aligned][padded W N*ldq]
  const size_t off_scales = kAmaxSlots * sizeof(uint32_t);
  const size_t off_q = align_up(off_scales + sizeof(float) * static_cast<size_t>(M), 256);
  const size_t off_w = align_up(off_q + static_cast<size_t>(M) * ldq, 256);
  const size_t total = off_w + (pad_w ? static_cast<size_t>(N) * ldq : 0);
  if (total > kNoAllocScratchBytes)
    return fail(ESMCU_ERR_OUT_OF_RANGE,
                "esmcu_linear_int8_noalloc: needs " + std::to_string(total) +
                    " bytes of scratch for M=" + std::to_string(M) + ", K=" + std::to_string(K) +
                    "; the fixed scratch holds " + std::to_string(kNoAllocScratchBytes) +
                    " (use esmcu_linear_int8 or split M)");
  char* base = static_cast<char*>(scratch_address());
  if (base == nullptr) return ESMCU_ERR_CUDA;
  uint32_t* amax = reinterpret_cast<uint32_t*>(base);
  float* scales = reinterpret_cast<float*>(base + off_scales);
  int8_t* q = reinterpret_cast<int8_t*>(base + off_q);
  const int8_t* w_dev = W;
  if (pad_w) {
    int8_t* wp = reinterpret_cast<int8_t*>(base + off_w);
    ESMCU_CUDA(cudaMemsetAsync(wp, 0, static_cast<size_t>(N) * ldq, ctx->stream));
    ESMCU_CUDA(cudaMemcpy2DAsync(wp, ldq, W, static_cast<size_t>(K), static_cast<size_t>(K), N,
                                 cudaMemcpyDeviceToDevice, ctx->stream));
    w_dev = wp;
  }
  if (act_quant == ESMCU_ACT_PER_TOKEN) {
    ESMCU_CUDA(launch_quantize_per_token(A, K, M, K, q, static_cast<long>(ldq), scales, ctx->stream));
  } else {
    // The slots keep the previous call's maxima: clear them first.
    ESMCU_CUDA(cudaMemsetAsync(amax, 0, kAmaxSlots * sizeof(uint32_t), ctx->stream));
    ESMCU_CUDA(launch_absmax(A, static_cast<long>(M) * K, amax, ctx->stream));
    ESMCU_CUDA(launch_quantize_per_tensor(A, K, M, K, amax, q, static_cast<long>(ldq), scales,
                                          ctx->stream));
  }
  GemmI8Args a;
  a.A = q;
  a.lda = static_cast<long>(ldq);
  a.W = w_dev;
  a.ldw = static_cast<long>(ldq);
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

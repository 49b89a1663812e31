// Host-side context and error plumbing behind the C ABI (include/esm_b200.h).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "esm_b200.h"

struct esmcu_context {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  cudaStream_t own_stream = nullptr;
  uint32_t* d_status = nullptr;  // device-side status word (timeouts)
  // Scratch for the kernel-facade entry points (quantised activations,
  // absmax, scales, padded weights).  Grows between calls, never shrinks.
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  int math_mode = 0;  // esmcu_math_mode
};

namespace esmb200 {

// Thread-local last error message (esmcu_last_error).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Makes ctx->device current on this thread.
int use_device(esmcu_context* ctx);
// Ensures the context scratch holds at least `bytes`; synchronises the
// stream before re-allocating.
int ensure_scratch(esmcu_context* ctx, size_t bytes);
// Reads (and clears) the device status word after a stream synchronise.
int check_device_status(esmcu_context* ctx);
// Loads the module holding esmcu_linear_int8_noalloc's fixed scratch on the
// current device (noalloc.cu); esmcu_open calls it.
int noalloc_prepare();

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ESM_AMX_ATTENTION = "on" | "1" | "true": the reference's opt-in BF16
// attention (attention.cpp:686-700), Q and K rounded to bf16 before the
// scores, for head dims that are multiples of 32.  Read at every forward (the
// reference reads it once per process).
bool attention_bf16_enabled(int head_dim);

}  // namespace esmb200

#define ESMCU_CUDA(call)                                          \
  do {                                                            \
    cudaError_t e_ = (call);                                      \
    if (e_ != cudaSuccess) return ::esmb200::cuda_fail(e_, #call); \
  } while (0)

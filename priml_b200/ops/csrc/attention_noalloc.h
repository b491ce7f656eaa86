// C interface of the allocation-free flash-attention backward pass.
//
// This interface has no counterpart in the reference framework. It serves
// callers of this library that cannot allocate device memory: code running
// inside another runtime's memory arena or a fixed-budget serving process,
// hosts that speak only a C ABI and own no CUDA allocator, and code that must
// not call cudaMalloc / cudaFree mid-run because those calls synchronize the
// device. The scratch memory the backward needs lives in one static device
// array inside the library (see attention_noalloc.cu for its limits).
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of pb_attn_bwd_noalloc.
enum PbNoallocStatus {
  PB_NOALLOC_OK = 0,
  PB_NOALLOC_BAD_ARGUMENT = 1,  // null / misaligned pointer, unsupported shape
  PB_NOALLOC_TOO_LARGE = 2,     // B * H * S above the scratch array's 524288 rows
  PB_NOALLOC_CUDA_ERROR = 3,    // a CUDA error was pending on entry, or a launch failed
};

// Backward of causal / windowed / full flash attention with grouped KV heads.
//
// All tensors are contiguous bf16 except lse (fp32):
//   q, o, dout, dq : [B, S, H, D]      k, v, dk, dv : [B, T, Hkv, D]
//   lse            : [B, H, S]  (natural log-sum-exp rows of the forward pass)
// D is 64 or 128, H a multiple of Hkv, T >= S when causal (masks are aligned
// bottom-right), and B * H * S <= 524288. window < 0 disables the sliding
// window. Asynchronous on `stream`. Returns a PbNoallocStatus value; an error
// already pending on the calling thread is left in place and reported as
// PB_NOALLOC_CUDA_ERROR without launching anything.
int pb_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                        const float* lse, void* dq, void* dk, void* dv, int B, int S, int T, int H, int Hkv, int D,
                        float scale, int causal, int window, cudaStream_t stream);

// Waits for `stream` (the stream the backward ran on), then returns the status
// word that the last pb_attn_bwd_noalloc call on the current device left: 0
// when no kernel wait timed out, a positive kernel error code otherwise, and
// -1 if the read itself failed.
int pb_attn_bwd_noalloc_status(cudaStream_t stream);

#ifdef __cplusplus
}  // extern "C"
#endif

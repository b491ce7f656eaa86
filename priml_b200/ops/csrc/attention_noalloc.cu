// Allocation-free entry point for the flash-attention backward pass.
//
// This file has no counterpart in the reference framework; it exists for
// callers of this library that cannot allocate device memory themselves:
// code that runs inside another runtime's memory arena or a fixed-budget
// serving process, host code written against a C ABI with no CUDA allocator
// of its own, and code that must not call cudaMalloc / cudaFree at all
// because those calls synchronize the device or are forbidden mid-run.
// They can call `pb_attn_bwd_noalloc` with their own inputs and outputs; the
// scratch memory the backward pass needs (the per-row `delta = rowsum(dO*O)`
// vector, a padded copy of the forward's log-sum-exp rows and the kernels'
// error-status word) lives in one file-scope device array instead of being
// allocated per call.
//
// Limits and rules:
//   * The array holds at most kMaxRows = 524288 rows (B * H * S), i.e. 4 MiB
//     of fp32 scratch, and is resident on every GPU that loads this library
//     until the process exits. Larger problems are rejected with
//     PB_NOALLOC_TOO_LARGE; nothing is launched.
//   * Every call on a device shares that device's array. Calls that overlap on
//     the GPU (different streams, or host threads racing) race on the scratch
//     and produce wrong results; serialize them on one stream.
//   * The scratch keeps the previous call's contents. Each call clears the
//     error-status word before launching and overwrites every scratch value
//     the kernels read for visible (unmasked) positions.
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (that device must be current) and caches it; make
//     that first call before any stream capture begins.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"

namespace {

constexpr long long kMaxRows = 524288;
constexpr long long kPad = 128;       // tail padding read by the 64-row bulk copies
constexpr long long kStatusFloats = 64;
constexpr long long kScratchFloats = kStatusFloats + 2 * (kMaxRows + kPad);

// [status (int) | delta (kMaxRows + kPad) | lse copy (kMaxRows + kPad)]
static __device__ __align__(256) float g_attn_bwd_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Resolve (once per device) the device address of the scratch array. In host
// code the array's name is only a stand-in for the symbol, never a pointer a
// kernel may use; the device address comes from cudaGetSymbolAddress with the
// device current.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_attn_bwd_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

enum {
  PB_NOALLOC_OK = 0,
  PB_NOALLOC_BAD_ARGUMENT = 1,
  PB_NOALLOC_TOO_LARGE = 2,
  PB_NOALLOC_CUDA_ERROR = 3,
};

// Backward of causal / windowed / full flash attention with grouped KV heads.
//
// All tensors are contiguous bf16 except lse (fp32):
//   q, o, dout, dq : [B, S, H, D]      k, v, dk, dv : [B, T, Hkv, D]
//   lse            : [B, H, S]  (natural log-sum-exp from the forward pass)
// D must be 64 or 128, H a multiple of Hkv, T >= S for causal masks, and
// B * H * S <= 524288. `window` < 0 disables the sliding window. The call is
// asynchronous on `stream`; it returns PB_NOALLOC_OK or an error code (a CUDA
// launch error returns PB_NOALLOC_CUDA_ERROR). Kernel wait timeouts are
// recorded in the first int of the scratch array's status word.
__attribute__((visibility("default"))) int pb_attn_bwd_noalloc(
    const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse, void* dq,
    void* dk, void* dv, int B, int S, int T, int H, int Hkv, int D, float scale, int causal, int window,
    cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr || dout == nullptr || lse == nullptr ||
      dq == nullptr || dk == nullptr || dv == nullptr)
    return PB_NOALLOC_BAD_ARGUMENT;
  if (B <= 0 || S <= 0 || T <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || (D != 64 && D != 128))
    return PB_NOALLOC_BAD_ARGUMENT;
  if (causal && T < S) return PB_NOALLOC_BAD_ARGUMENT;
  for (const void* p : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (!aligned16(p)) return PB_NOALLOC_BAD_ARGUMENT;
  const long long rows = static_cast<long long>(B) * H * S;
  if (rows > kMaxRows) return PB_NOALLOC_TOO_LARGE;

  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return PB_NOALLOC_CUDA_ERROR;
  int* status = reinterpret_cast<int*>(scratch);
  float* delta = scratch + kStatusFloats;
  float* lse_copy = delta + (kMaxRows + kPad);

  // Clear the status word; stage lse into padded scratch so the kernels' 64-row
  // bulk reads never run past the caller's buffer.
  if (cudaMemsetAsync(status, 0, sizeof(int), stream) != cudaSuccess) return PB_NOALLOC_CUDA_ERROR;
  if (cudaMemcpyAsync(lse_copy, lse, rows * sizeof(float), cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
    return PB_NOALLOC_CUDA_ERROR;

  const long long qs = static_cast<long long>(H) * D, ks = static_cast<long long>(Hkv) * D;
  pb::AttnTensor tq{const_cast<void*>(q), B, S, S * qs, qs};
  pb::AttnTensor to{const_cast<void*>(o), B, S, S * qs, qs};
  pb::AttnTensor tdo{const_cast<void*>(dout), B, S, S * qs, qs};
  pb::AttnTensor tdq{dq, B, S, S * qs, qs};
  pb::AttnTensor tk{const_cast<void*>(k), B, T, T * ks, ks};
  pb::AttnTensor tv{const_cast<void*>(v), B, T, T * ks, ks};
  pb::AttnTensor tdk{dk, B, T, T * ks, ks};
  pb::AttnTensor tdv{dv, B, T, T * ks, ks};
  try {
    pb::attn_bwd(tq, tk, tv, to, tdo, lse_copy, delta, tdq, tdk, tdv, H, Hkv, D, scale, causal != 0, window, status,
                 stream);
  } catch (...) {
    return PB_NOALLOC_CUDA_ERROR;
  }
  return cudaGetLastError() == cudaSuccess ? PB_NOALLOC_OK : PB_NOALLOC_CUDA_ERROR;
}

// Reads (synchronously, on the current device) the status word of
// the most recent pb_attn_bwd_noalloc call: 0 means no kernel wait timed out.
__attribute__((visibility("default"))) int pb_attn_bwd_noalloc_status(void) {
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return -1;
  int host = 0;
  if (cudaMemcpy(&host, scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return host;
}

}  // extern "C"

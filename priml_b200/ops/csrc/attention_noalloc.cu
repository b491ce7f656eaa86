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
//     that first call before any stream capture begins. The cache is keyed by
//     device ordinal and assumes the device's primary context (the one the
//     CUDA runtime and torch use); it is not refreshed after cudaDeviceReset,
//     so a caller that resets a device or drives it from its own driver-API
//     context must not use this entry point on that device afterwards.
//   * For D = 64 the regular entry point runs a fused single-kernel backward
//     that accumulates dQ in an fp32 buffer of B * H * S * D floats; that
//     buffer is too large for a static array, so this entry point always runs
//     the two-kernel backward (dK/dV, then dQ), which needs only per-row
//     scratch.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include "attention_noalloc.h"

#include <cuda_runtime.h>

#include <cstdint>
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

// Contract in attention_noalloc.h. Kernel wait timeouts are recorded in the
// first int of the scratch array (the status word).
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
  // An error left by earlier, unrelated work stays visible to its owner: report
  // it without clearing it, and launch nothing.
  if (cudaPeekAtLastError() != cudaSuccess) return PB_NOALLOC_CUDA_ERROR;

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

// Contract in attention_noalloc.h: the copy is queued on the caller's stream,
// behind the backward kernels, and the stream is then synchronized, so the
// read sees this call's status even on a non-blocking stream.
__attribute__((visibility("default"))) int pb_attn_bwd_noalloc_status(cudaStream_t stream) {
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return -1;
  int host = 0;
  if (cudaMemcpyAsync(&host, scratch, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  return host;
}

}  // extern "C"

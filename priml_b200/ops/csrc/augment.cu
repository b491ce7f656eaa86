// Fused image augmentation: reflect/replicate/constant pad -> random crop ->
// optional horizontal flip -> cutout, in one pass (one gathered read per output
// pixel, no padded intermediate). Per-image offsets, flip flags and cutout
// corners are drawn by the caller (device tensors), so the kernel is a pure
// function of its inputs (`priml/data/augmentation_gpu.py:14-112`).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "kernels.h"

namespace pb {
namespace {

// Index into [0, n) of padded coordinate `p` (p in [-pad, n + pad)).
__device__ __forceinline__ int src_index(int p, int n, int mode, bool& inside) {
  inside = true;
  if (p >= 0 && p < n) return p;
  if (mode == 0) {  // constant
    inside = false;
    return 0;
  }
  if (mode == 1) return p < 0 ? 0 : n - 1;  // replicate
  // reflect (edge not repeated): -1 -> 1, n -> n - 2
  if (n == 1) return 0;
  const int period = 2 * (n - 1);
  int q = p % period;
  if (q < 0) q += period;
  return q < n ? q : period - q;
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(uint8_t v) { return static_cast<float>(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <>
__device__ __forceinline__ uint8_t from_f<uint8_t>(float v) { return static_cast<uint8_t>(v); }

template <typename T>
__global__ void pad_crop_flip_cutout_kernel(const T* __restrict__ in, T* __restrict__ out, int B, int C, int H, int W,
                                            int crop, int pad, int mode, float fill, const int32_t* __restrict__ dy,
                                            const int32_t* __restrict__ dx, const uint8_t* __restrict__ flip,
                                            const int32_t* __restrict__ cy, const int32_t* __restrict__ cx, int cut) {
  const long long total = static_cast<long long>(B) * C * crop * crop;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % crop);
    const int y = static_cast<int>((i / crop) % crop);
    const long long bc = i / (static_cast<long long>(crop) * crop);
    const int b = static_cast<int>(bc / C);
    const int xs = (flip != nullptr && flip[b]) ? crop - 1 - x : x;
    const int py = y + dy[b] - pad, px = xs + dx[b] - pad;
    bool in_y, in_x;
    const int sy = src_index(py, H, mode, in_y), sx = src_index(px, W, mode, in_x);
    float v = (in_y && in_x) ? to_f(in[(bc * H + sy) * W + sx]) : fill;
    if (cut > 0 && y >= cy[b] && y < cy[b] + cut && x >= cx[b] && x < cx[b] + cut) v = 0.f;
    out[i] = from_f<T>(v);
  }
}

}  // namespace

void pad_crop_flip_cutout(const void* in, void* out, int dtype, int B, int C, int H, int W, int crop, int pad,
                          int mode, float fill, const int32_t* dy, const int32_t* dx, const uint8_t* flip,
                          const int32_t* cy, const int32_t* cx, int cut, cudaStream_t stream) {
  const long long total = static_cast<long long>(B) * C * crop * crop;
  if (total == 0) return;
  const int threads = 256;
  const int blocks = static_cast<int>((total + threads - 1) / threads < 148LL * 32 ? (total + threads - 1) / threads
                                                                                   : 148LL * 32);
  if (dtype == 0) {
    pad_crop_flip_cutout_kernel<float><<<blocks, threads, 0, stream>>>(
        static_cast<const float*>(in), static_cast<float*>(out), B, C, H, W, crop, pad, mode, fill, dy, dx, flip, cy, cx,
        cut);
  } else if (dtype == 1) {
    pad_crop_flip_cutout_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(in), static_cast<__nv_bfloat16*>(out), B, C, H, W, crop, pad, mode, fill, dy,
        dx, flip, cy, cx, cut);
  } else {
    pad_crop_flip_cutout_kernel<uint8_t><<<blocks, threads, 0, stream>>>(
        static_cast<const uint8_t*>(in), static_cast<uint8_t*>(out), B, C, H, W, crop, pad, mode, fill, dy, dx, flip, cy,
        cx, cut);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("augment launch: ") + cudaGetErrorString(e));
}

}  // namespace pb

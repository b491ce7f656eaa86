// Host utilities: SM count cache and TMA tensor-map encoding. The driver's
// cuTensorMapEncodeTiled is reached through cudaGetDriverEntryPoint so the
// extension links against the runtime only.
#include <cudaTypedefs.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace pb {

int device_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cached[dev] = n;
  return n;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      throw std::runtime_error("cuTensorMapEncodeTiled is not available from the driver");
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// The driver's tensor-map encoder needs a current context on the calling thread.
// Autograd runs backward on its own worker threads, which may not have bound the
// primary context yet; bind it once per thread and device.
static void ensure_context() {
  static thread_local int bound_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (bound_dev != dev) {
    cudaSetDevice(dev);  // initializes the primary context and makes it current (CUDA >= 12)
    bound_dev = dev;
  }
}

static void check_encode(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) throw std::runtime_error(std::string("cuTensorMapEncodeTiled failed: ") + what +
                                                  " (error " + std::to_string(static_cast<int>(r)) + ")");
}

void make_tmap_2d_bf16(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                       int box_inner, int box_outer) {
  ensure_context();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride * 2) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  check_encode(encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
               "2d");
}

static void encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int esize, const void* base, long long inner,
                      long long outer, long long row_stride, int box_inner, int box_outer, CUtensorMapSwizzle swz,
                      const char* what) {
  ensure_context();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride * esize) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * esize)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  check_encode(encode_fn()(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
               what);
}

void make_tmap_2d_bf16_sw64(CUtensorMap* map, const void* base, long long inner, long long outer,
                            long long row_stride, int box_inner, int box_outer) {
  if (box_inner * 2 != 64) throw std::runtime_error("64-byte swizzle needs a 64-byte box row");
  encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, inner, outer, row_stride, box_inner, box_outer,
            CU_TENSOR_MAP_SWIZZLE_64B, "2d bf16 sw64");
}

void make_tmap_2d_f32_sw128(CUtensorMap* map, const void* base, long long inner, long long outer,
                            long long row_stride, int box_inner, int box_outer) {
  if (box_inner * 4 != 128) throw std::runtime_error("128-byte swizzle needs a 128-byte box row");
  encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, inner, outer, row_stride, box_inner, box_outer,
            CU_TENSOR_MAP_SWIZZLE_128B, "2d f32 sw128");
}

void make_tmap_2d_u8(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                     int box_inner, int box_outer) {
  ensure_context();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if (row_stride % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  check_encode(encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
               "2d u8");
}

// 2-D byte map without swizzle (MXFP8 scale atoms: 512-byte boxes copied as they are).
void make_tmap_2d_u8_plain(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                           int box_inner, int box_outer) {
  encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, inner, outer, row_stride, box_inner, box_outer,
            CU_TENSOR_MAP_SWIZZLE_NONE, "2d u8 plain");
}

void make_tmap_2d_f32(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                      int box_inner, int box_outer) {
  ensure_context();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride * 4) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 4)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  check_encode(encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
               "2d f32");
}

void make_tmap_3d_bf16(CUtensorMap* map, const void* base, long long inner, long long mid, long long outer,
                       long long mid_stride, long long outer_stride, int box_inner, int box_mid, bool swizzle128) {
  ensure_context();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((mid_stride * 2) % 16 != 0 || (outer_stride * 2) % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(mid), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(mid_stride * 2), static_cast<cuuint64_t>(outer_stride * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_mid), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  check_encode(encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
               "3d");
}

}  // namespace pb

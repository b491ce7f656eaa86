// MXFP8: OCP microscaling fp8 (E4M3 elements, one E8M0 power-of-two scale per
// 32 consecutive elements along the contraction dimension) for sm_100a.
//
//   mx_quantize        bf16 [R, K] -> fp8 [R, K] + scales, blocks of 32 along K
//   mx_quantize_t      bf16 [R, K] -> fp8 [K, R] + scales, blocks of 32 along R
//                      (the transposed operand of the dgrad / wgrad GEMMs, so
//                      every MX GEMM reads K-major operands)
//   mx_gemm            C[M, N] (op)= sum_k A(m,k) 2^sa(m,k/32) B(n,k) 2^sb(n,k/32)
//                      with tcgen05.mma.kind::mxf8f6f4.block_scale (fp32 TMEM
//                      accumulator, scale factors in TMEM).
//
// Scale rule (OCP Microscaling Formats v1.0, section 6.3): with amax the largest
// |x| of a block and emax = 8 the largest exponent of E4M3, the shared exponent
// is floor(log2(amax)) - emax, clamped to the E8M0 range [-127, 127]; elements
// are x * 2^-shared converted with round-to-nearest-even and saturation to
// +-448. floor(log2(amax)) is read from the fp32 exponent field (subnormal or
// zero blocks take the smallest scale).
//
// Scale storage ("blocked" layout, the one the scale-factor copy into tensor
// memory expects): scales of 128 rows x 4 consecutive 32-element blocks form a
// 512-byte atom; row r, block kb of the atom sits at byte
// 16 * (r % 32) + 4 * (r / 32) + kb. Atoms are ordered K-block-group fastest,
// then 128-row block; the row-block count is rounded up to an even number so a
// 256-row GEMM tile always has two atoms. Padding scales are 127 (= 1.0).
//
// GEMM structure: 128 x 256 output tiles, 128-deep K steps (128 bytes of fp8 per
// row = one 128-byte swizzle row), 4 shared-memory stages, one TMA producer
// warp, one MMA warp, four epilogue warps, one fp32 accumulator of 256 TMEM
// columns plus 12 columns of scale factors. Per K step the MMA thread copies the
// A atom and the two B atoms from shared memory into TMEM
// (tcgen05.cp.32x128b.warpx4) and issues four K=32 MMAs that select their
// scale byte through the instruction descriptor. Every wait is bounded.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int XBN = 256, XBK = 128, XSTAGES = 4;
constexpr int kXA = BM * XBK;        // 16 KB
constexpr int kXB = XBN * XBK;       // 32 KB
constexpr int kXSFA = 512;           // one atom
constexpr int kXSFB = 1024;          // two atoms
constexpr int kXStage = kXA + kXB + kXSFA + kXSFB;
constexpr int kXSmem = XSTAGES * kXStage + 1024 + 256;
constexpr uint32_t kAccCols = 256, kSfaCol = 256, kSfbCol = 260, kXTmemCols = 512;

// ---------------------------------------------------------------- scale rule
__device__ __forceinline__ int shared_exponent(float amax) {
  const int field = (__float_as_int(amax) >> 23) & 0xFF;  // biased exponent; 0 for zero / subnormal
  int e = (field == 0 ? -127 : field - 127) - 8;           // floor(log2(amax)) - emax(E4M3)
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

__device__ __forceinline__ float pow2_neg(int e) {  // 2^-e for e in [-127, 119]: an exact power of two
  return __int_as_float((127 - e) << 23);
}

__device__ __forceinline__ long long sf_offset(long long r, int kb, int nkg) {
  return ((r >> 7) * nkg + (kb >> 2)) * 512 + 16 * (r & 31) + 4 * ((r & 127) >> 5) + (kb & 3);
}

__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// One thread per 32-element block of a row: x [R, K] (row stride ldx) -> q [R, K], sf blocked.
__global__ void __launch_bounds__(256) mx_quant_rows_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                            uint8_t* __restrict__ q, uint8_t* __restrict__ sf, int R,
                                                            int K, int nkg) {
  const int kblocks = K / 32;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(R) * kblocks) return;
  const long long r = idx / kblocks;
  const int kb = static_cast<int>(idx - r * kblocks);
  const uint4* src = reinterpret_cast<const uint4*>(x + r * ldx + kb * 32);
  float v[32];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 w = src[i];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[j]));
      v[8 * i + 2 * j] = f.x;
      v[8 * i + 2 * j + 1] = f.y;
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = shared_exponent(amax);
  const float s = pow2_neg(e);
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) packed[i] = pack4(v[4 * i] * s, v[4 * i + 1] * s, v[4 * i + 2] * s, v[4 * i + 3] * s);
  uint4* dst = reinterpret_cast<uint4*>(q + r * K + kb * 32);
  dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  sf[sf_offset(r, kb, nkg)] = static_cast<uint8_t>(e + 127);
}

// One thread per (column k, 32-row block): x [R, K] -> qt [K, R] (blocks along R), sf blocked over qt.
__global__ void __launch_bounds__(256) mx_quant_cols_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                            uint8_t* __restrict__ qt, uint8_t* __restrict__ sf, int R,
                                                            int K, int nkg) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  const int rb = blockIdx.y;  // 32-row block
  if (k >= K) return;
  float v[32];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const long long r = static_cast<long long>(rb) * 32 + i;
    v[i] = r < R ? __bfloat162float(x[r * ldx + k]) : 0.f;
    amax = fmaxf(amax, fabsf(v[i]));
  }
  const int e = shared_exponent(amax);
  const float s = pow2_neg(e);
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) packed[i] = pack4(v[4 * i] * s, v[4 * i + 1] * s, v[4 * i + 2] * s, v[4 * i + 3] * s);
  uint4* dst = reinterpret_cast<uint4*>(qt + static_cast<long long>(k) * R + rb * 32);
  dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  sf[sf_offset(k, rb, nkg)] = static_cast<uint8_t>(e + 127);
}

// ---------------------------------------------------------------- GEMM
// Shared-memory descriptor of a 32-row x 16-byte scale atom slice (K-major, no swizzle:
// 8-row core matrices of 16-byte rows, 128 bytes apart).
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((128u >> 4) & 0x3FFFu) << 32;  // stride between core matrices (rows 8 apart)
  d |= static_cast<uint64_t>(1) << 46;                      // descriptor version for sm_100
  return d;                                                  // layout type 0: no swizzle
}

__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Block-scaled instruction descriptor: E4M3 A and B, K-major, E8M0 scales, fp32 accumulate.
__device__ __forceinline__ uint32_t make_idesc_mx(int m, int n, uint32_t sf_id) {
  return (sf_id << 4)                               // B scale byte
         | (0u << 7) | (0u << 10)                   // A, B format: E4M3
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (1u << 23)                               // scale format: E8M0
         | (static_cast<uint32_t>(m >> 4) << 24)    // M / 16
         | (sf_id << 29);                           // A scale byte
}

__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

struct MxParams {
  GemmParams g;
  const uint8_t* sfa;  // blocked scales of A
  const uint8_t* sfb;  // blocked scales of B
  int nkg;             // 128-deep K groups
};

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const MxParams p) {
  constexpr int S = XSTAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smA + S * kXA;
  uint8_t* smSFA = smB + S * kXB;
  uint8_t* smSFB = smSFA + S * kXSFA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kXStage);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int num_m = (p.g.M + BM - 1) / BM;
  const int num_n = (p.g.N + XBN - 1) / XBN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.g.K + XBK - 1) / XBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kXTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.g.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], kXStage);
        tma_load_2d(smA + stage * kXA, &tmA, &full[stage], kb * XBK, mb * BM);
        tma_load_2d(smB + stage * kXB, &tmB, &full[stage], kb * XBK, nb * XBN);
        bulk_load(smSFA + stage * kXSFA, p.sfa + (static_cast<long long>(mb) * p.nkg + kb) * 512, kXSFA, &full[stage]);
        bulk_load(smSFB + stage * kXSFB, p.sfb + (static_cast<long long>(2 * nb) * p.nkg + kb) * 512, 512, &full[stage]);
        bulk_load(smSFB + stage * kXSFB + 512, p.sfb + (static_cast<long long>(2 * nb + 1) * p.nkg + kb) * 512, 512,
                  &full[stage]);
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      for (int i = 0; i < min(issued, S); ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.g.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    const uint32_t sfa_t = tmem_base + kSfaCol, sfb_t = tmem_base + kSfbCol;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      if (!mbar_wait(tempty, (local & 1) ^ 1u, p.g.status, kTimeoutMma, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.g.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sfa_s = smem_u32(smSFA + stage * kXSFA);
        const uint32_t sfb_s = smem_u32(smSFB + stage * kXSFB);
        tmem_cp_sf(sfa_t, make_sf_desc(sfa_s));
        tmem_cp_sf(sfb_t, make_sf_desc(sfb_s));
        tmem_cp_sf(sfb_t + 4, make_sf_desc(sfb_s + 512));
        const uint32_t a_base = smem_u32(smA + stage * kXA);
        const uint32_t b_base = smem_u32(smB + stage * kXB);
#pragma unroll
        for (int kk = 0; kk < XBK / 32; ++kk) {
          const uint32_t sel = static_cast<uint32_t>(kk) << 30;  // scale byte kk of each TMEM word
          umma_mx(tmem_base, make_sw128_desc(a_base + kk * 32, 16, 1024), make_sw128_desc(b_base + kk * 32, 16, 1024),
                  make_idesc_mx(BM, XBN, static_cast<uint32_t>(kk)), sfa_t | sel, sfb_t | sel,
                  (kb | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(tfull);
    }
    umma_commit(drain);
    mbar_wait(drain, 0, p.g.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      if (!mbar_wait_warp(tfull, local & 1, p.g.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = mb * BM + wq * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
      store_acc_row<XBN, EPI>(p.g, t_row, row, nb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, kXTmemCols);
  }
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <int EPI>
void launch_mx(const CUtensorMap& ta, const CUtensorMap& tb, const MxParams& p, cudaStream_t stream) {
  auto kern = mx_gemm_kernel<EPI>;
  static bool configured = false;
  if (!configured) {
    check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kXSmem), "mx gemm smem attribute");
    configured = true;
  }
  const int tiles = ((p.g.M + BM - 1) / BM) * ((p.g.N + XBN - 1) / XBN);
  const int sms = device_sm_count();
  kern<<<tiles < sms ? tiles : sms, kThreads, kXSmem, stream>>>(ta, tb, p);
  check(cudaGetLastError(), "mx gemm launch");
}

}  // namespace

long long mx_scale_bytes(long long rows, long long k) {
  const long long row_blocks = ((rows + 255) / 256) * 2;
  return row_blocks * ((k + 127) / 128) * 512;
}

void mx_quantize(const void* x, long long ldx, void* q, void* sf, int R, int K, bool transpose, cudaStream_t stream) {
  if (K % 32 != 0 && !transpose) throw std::invalid_argument("mx_quantize: K must be a multiple of 32");
  if (transpose && (R % 32 != 0)) throw std::invalid_argument("mx_quantize (transposed): rows must be a multiple of 32");
  if (ldx % 8 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    throw std::invalid_argument("mx_quantize: x rows must be 16-byte aligned");
  // scales of the output matrix: [R, K] (rows) or [K, R] (transposed)
  const long long out_rows = transpose ? K : R, out_k = transpose ? R : K;
  check(cudaMemsetAsync(sf, 127, mx_scale_bytes(out_rows, out_k), stream), "mx scale init");
  const int nkg = static_cast<int>((out_k + 127) / 128);
  if (!transpose) {
    const long long n = static_cast<long long>(R) * (K / 32);
    const int blocks = static_cast<int>((n + 255) / 256);
    if (n > 0)
      mx_quant_rows_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                       static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), R, K, nkg);
  } else {
    const dim3 grid((K + 255) / 256, R / 32);
    if (K > 0 && R > 0)
      mx_quant_cols_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                     static_cast<uint8_t*>(q), static_cast<uint8_t*>(sf), R, K, nkg);
  }
  check(cudaGetLastError(), "mx quantize launch");
}

void mx_gemm(const void* A, const void* sfa, const void* B, const void* sfb, void* C, long long ldc, int M, int N, int K,
             int epi, int* status, cudaStream_t stream) {
  if (K % 32 != 0 || K <= 0) throw std::invalid_argument("mx_gemm: K must be a positive multiple of 32");
  CUtensorMap ta, tb;
  make_tmap_2d_u8(&ta, A, K, M, K, XBK, BM);
  make_tmap_2d_u8(&tb, B, K, N, K, XBK, XBN);
  MxParams p{};
  p.g = GemmParams{M, N, K, C, ldc, nullptr, status, 0};
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  p.nkg = (K + 127) / 128;
  switch (epi) {
    case 0: launch_mx<0>(ta, tb, p, stream); break;
    case 1: launch_mx<1>(ta, tb, p, stream); break;
    case 2: launch_mx<2>(ta, tb, p, stream); break;
    default: throw std::invalid_argument("mx_gemm: epi 0 (bf16), 1 (fp32) or 2 (fp32 +=)");
  }
}

}  // namespace pb

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
// GEMM structure (1-CTA kernel, used when the output cannot take bulk tensor stores;
// the 2-CTA kernel below is the default): 128 x 256 output tiles, 128-deep K steps
// (128 bytes of fp8 per row = one 128-byte swizzle row), 4 shared-memory stages, one TMA producer
// warp, one MMA warp, four epilogue warps, one fp32 accumulator of 256 TMEM
// columns plus 12 columns of scale factors. Per K step the MMA thread copies the
// A atom and the two B atoms from shared memory into TMEM
// (tcgen05.cp.32x128b.warpx4) and issues four K=32 MMAs that select their
// scale byte through the instruction descriptor. Every wait is bounded.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdlib>
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

// ---------------------------------------------------------------- 2-CTA tiles
// A CTA pair (cluster of 2) computes a 256 x 256 output tile with M = 256 block-scaled MMAs
// (cta_group::2): CTA r holds A rows [128 r, 128 r + 128) and B rows (N) [128 r, 128 r + 128)
// of every 128-deep K step, so each SM streams 32 KB of fp8 operands per step instead of the
// 48 KB of a 1-CTA 128 x 256 tile, for the same MMA time. Scale factors: each CTA copies the
// atom of its own 128 A rows and the two atoms of all 256 B rows into its shared memory;
// CTA 0's MMA thread moves them into both CTAs' TMEM with tcgen05.cp.cta_group::2 (each CTA's
// shared memory to its own TMEM) and issues the MMAs. All completion bytes of a stage land
// on CTA 0's `full` barrier; `empty` and `tfull` commits go to both CTAs.
//
// TMEM: one 256-column fp32 accumulator plus 12 scale columns (two accumulators would leave
// no room for the scales). The eight epilogue warps (two per TMEM lane quarter, 128 columns
// each) read the whole accumulator into registers first and release it right away, so the
// next tile's MMAs start while the tile's values are converted and leave through bulk tensor
// stores (bf16 / fp32) or bulk reduce-adds (fp32 +=).
constexpr int kMxPairThreads = 320;
constexpr int kMxPairA = 128 * XBK;  // this CTA's 128 rows of A: 16 KB
constexpr int kMxPairB = 128 * XBK;  // this CTA's 128 rows (N) of B: 16 KB
constexpr int kMxPairStage = kMxPairA + kMxPairB + kXSFA + kXSFB;

template <int EPI>
struct MxPairCfg {
  static constexpr int kStages = EPI == 0 ? 6 : 5;
  static constexpr int kChunk = EPI == 0 ? 2048 : 4096;  // per epilogue warp: 32 rows x 32 columns
  static constexpr int kSmem = kStages * kMxPairStage + 8 * kChunk + 1024 + 256;
  static_assert(kSmem <= 232448, "MXFP8 pair GEMM shared memory exceeds the per-CTA limit");
};

__device__ __forceinline__ void tmem_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void umma_mx_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kMxPairThreads, 1)
    mx_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                   const __grid_constant__ CUtensorMap tmC, const MxParams p) {
  using Cfg = MxPairCfg<EPI>;
  constexpr int S = Cfg::kStages;
  constexpr int TM = 256, TN = 256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // Operand stages and the swizzled epilogue staging tiles first (1024-byte aligned: the
  // 128-byte swizzle pattern follows address bits 7-9), the unswizzled scale atoms after them.
  uint8_t* smA = smem;
  uint8_t* smB = smA + S * kMxPairA;
  uint8_t* stg = smB + S * kMxPairB;
  uint8_t* smSFA = stg + 8 * Cfg::kChunk;
  uint8_t* smSFB = smSFA + S * kXSFA;
  uint64_t* full = reinterpret_cast<uint64_t*>(smSFB + S * kXSFB);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint64_t* peer_done = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(peer_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  const int num_m = (p.g.M + TM - 1) / TM;
  const int num_n = (p.g.N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.g.K + XBK - 1) / XBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 16);  // eight epilogue warps of both CTAs
    mbar_init(drain, 1);
    mbar_init(peer_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmSA);
    prefetch_tmap(&tmSB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kXTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits of both CTAs visible before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const uint32_t full0 = cluster_addr(full, 0);
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int m0 = mb * TM + 128 * static_cast<int>(rank);
      const int n0 = nb * TN + 128 * static_cast<int>(rank);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.g.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kMxPairStage);
        const uint32_t bar = full0 + 8u * stage;
        tma_load_2d_pair(smA + stage * kMxPairA, &tmA, bar, kb * XBK, m0);
        tma_load_2d_pair(smB + stage * kMxPairB, &tmB, bar, kb * XBK, n0);
        // scale atoms (512 bytes = two 256-byte rows of the scale maps): this CTA's A rows, all 256 B rows
        tma_load_2d_pair(smSFA + stage * kXSFA, &tmSA, bar, 0, 2 * ((2 * mb + static_cast<int>(rank)) * p.nkg + kb));
        tma_load_2d_pair(smSFB + stage * kXSFB, &tmSB, bar, 0, 2 * ((2 * nb) * p.nkg + kb));
        tma_load_2d_pair(smSFB + stage * kXSFB + 512, &tmSB, bar, 0, 2 * ((2 * nb + 1) * p.nkg + kb));
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && leader) {
      for (int i = 0; i < min(issued, S); ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.g.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    if (leader) {
      // ------------------------------------------------------------ MMA issuer (CTA 0)
      const uint32_t empty1 = cluster_addr(empty, 1);
      const uint32_t tfull1 = cluster_addr(tfull, 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      uint32_t sf_slot = 0;  // scale columns rotate over 4 slots of 16: a copy never targets the
                             // columns that the previous K step's MMAs are still reading
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++local) {
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
          const uint32_t sfa_t = tmem_base + kSfaCol + 16u * (sf_slot++ & 3u), sfb_t = sfa_t + 4;
          tmem_cp_sf_pair(sfa_t, make_sf_desc(sfa_s));
          tmem_cp_sf_pair(sfb_t, make_sf_desc(sfb_s));
          tmem_cp_sf_pair(sfb_t + 4, make_sf_desc(sfb_s + 512));
          const uint32_t a_base = smem_u32(smA + stage * kMxPairA);
          const uint32_t b_base = smem_u32(smB + stage * kMxPairB);
#pragma unroll
          for (int kk = 0; kk < XBK / 32; ++kk) {
            const uint32_t sel = static_cast<uint32_t>(kk) << 30;  // scale byte kk of each TMEM word
            umma_mx_pair(tmem_base, make_sw128_desc(a_base + kk * 32, 16, 1024),
                         make_sw128_desc(b_base + kk * 32, 16, 1024), make_idesc_mx(TM, TN, static_cast<uint32_t>(kk)),
                         sfa_t | sel, sfb_t | sel, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage]);
          umma_commit_pair_to(empty1 + 8u * stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          umma_commit_pair(tfull);
          umma_commit_pair_to(tfull1);
        }
      }
      umma_commit_pair(drain);
      mbar_wait(drain, 0, p.g.status, kTimeoutDrain, nullptr);
      mbar_arrive_cluster(cluster_addr(peer_done, 1));  // CTA 1 may free its TMEM now
    } else {
      mbar_wait(peer_done, 0, p.g.status, kTimeoutDrain, nullptr);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int wq = warp & 3;             // TMEM lane quarter this warp may access
    const int c_lo = ((warp - 2) >> 2) * 128;  // this warp's 128 accumulator columns
    const uint32_t tempty0 = cluster_addr(tempty, 0);
    uint8_t* buf = stg + (warp - 2) * Cfg::kChunk;
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int row0 = mb * TM + 128 * static_cast<int>(rank) + wq * 32;
      if (!mbar_wait_warp(tfull, local & 1, p.g.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + c_lo;
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_row + 32 * c, v[c]);
      tmem_wait_ld();
      // the accumulator is in registers: the next tile's MMAs may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (lane == 0) tma_store_wait_read();  // the previous chunk's store has read the buffer
        __syncwarp();
        if constexpr (EPI == 0) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[c][2 * j]), __uint_as_float(v[c][2 * j + 1]));
          stage_row<4>(buf, lane, pk);
        } else {
          stage_row<8>(buf, lane, v[c]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (EPI == 2) {
            tma_reduce_add_2d(&tmC, buf, nb * TN + c_lo + 32 * c, row0);
          } else {
            tma_store_2d(&tmC, buf, nb * TN + c_lo + 32 * c, row0);
          }
          tma_store_commit();
        }
      }
    }
    if (lane == 0) tma_store_wait_all();  // staging read and global writes done before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrive may target a CTA that has exited
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, kXTmemCols);
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

template <int EPI>
void launch_mx_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa, const CUtensorMap& tsb,
                    const CUtensorMap& tc, const MxParams& p, cudaStream_t stream) {
  auto kern = mx_pair_kernel<EPI>;
  static bool configured = false;
  if (!configured) {
    check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MxPairCfg<EPI>::kSmem),
          "mx pair gemm smem attribute");
    configured = true;
  }
  const int tiles = ((p.g.M + 255) / 256) * ((p.g.N + 255) / 256);
  const int pairs_max = device_sm_count() / 2;
  const int pairs = tiles < pairs_max ? tiles : pairs_max;
  kern<<<2 * pairs, kMxPairThreads, MxPairCfg<EPI>::kSmem, stream>>>(ta, tb, tsa, tsb, tc, p);
  check(cudaGetLastError(), "mx pair gemm launch");
}

// The 2-CTA kernel writes through bulk tensor stores, which need a 16-byte aligned output
// base and row stride; PRIML_B200_MX_PAIR=0 selects the 1-CTA kernel (A/B measurements).
bool mx_pair_usable(int epi, const void* C, long long ldc) {
  static const bool on = [] {
    const char* e = std::getenv("PRIML_B200_MX_PAIR");
    return e == nullptr || e[0] != '0';
  }();
  const long long row_bytes = ldc * (epi == 0 ? 2 : 4);
  return on && (reinterpret_cast<uintptr_t>(C) & 15) == 0 && row_bytes % 16 == 0;
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
  if (epi < 0 || epi > 2) throw std::invalid_argument("mx_gemm: epi 0 (bf16), 1 (fp32) or 2 (fp32 +=)");
  MxParams p{};
  p.g = GemmParams{M, N, K, C, ldc, nullptr, status, 0};
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  p.nkg = (K + 127) / 128;
  CUtensorMap ta, tb;
  if (mx_pair_usable(epi, C, ldc)) {
    CUtensorMap tsa, tsb, tc;
    make_tmap_2d_u8(&ta, A, K, M, K, XBK, 128);
    make_tmap_2d_u8(&tb, B, K, N, K, XBK, 128);
    // scale arrays as rows of 256 bytes: one 512-byte atom is a 2-row box
    make_tmap_2d_u8_plain(&tsa, sfa, 256, mx_scale_bytes(M, K) / 256, 256, 256, 2);
    make_tmap_2d_u8_plain(&tsb, sfb, 256, mx_scale_bytes(N, K) / 256, 256, 256, 2);
    if (epi == 0) {
      make_tmap_2d_bf16_sw64(&tc, C, N, M, ldc, 32, 32);
      launch_mx_pair<0>(ta, tb, tsa, tsb, tc, p, stream);
    } else {
      make_tmap_2d_f32_sw128(&tc, C, N, M, ldc, 32, 32);
      if (epi == 1) launch_mx_pair<1>(ta, tb, tsa, tsb, tc, p, stream);
      else launch_mx_pair<2>(ta, tb, tsa, tsb, tc, p, stream);
    }
    return;
  }
  make_tmap_2d_u8(&ta, A, K, M, K, XBK, BM);
  make_tmap_2d_u8(&tb, B, K, N, K, XBK, XBN);
  switch (epi) {
    case 0: launch_mx<0>(ta, tb, p, stream); break;
    case 1: launch_mx<1>(ta, tb, p, stream); break;
    case 2: launch_mx<2>(ta, tb, p, stream); break;
    default: throw std::invalid_argument("mx_gemm: epi 0 (bf16), 1 (fp32) or 2 (fp32 +=)");
  }
}

}  // namespace pb

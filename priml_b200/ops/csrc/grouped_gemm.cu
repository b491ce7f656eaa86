// Grouped expert GEMM for sm_100a (tcgen05 + TMEM + TMA), driven by device-side
// group offsets: no host synchronization, one launch per GEMM of an MoE layer.
//
// Rows are dispatched per expert into 128-row-aligned segments
// (offsets[e] .. offsets[e+1], every offset a multiple of 128, zero rows as
// padding), so each 128-row tile belongs to exactly one expert.
//
//   mode 0  (forward, dgrad)  C[r, :] = A[r, :] @ B_e^T for rows r of expert e.
//           B is the stacked expert weight: K-major [E * b_rows, K] (B_e = rows
//           e * b_rows ...), or N-major [E * b_rows, N] (B_e^T = those rows).
//           Tiles cover only offsets[E] / 128 row blocks (read on the device).
//           Epilogues as in the dense GEMM: 0 bf16, 1 fp32, 2 fp32 +=, 3 fused
//           SwiGLU (gate/up rows of expert e), 4 SwiGLU backward.
//   mode 1  (weight gradient) C[e * out_rows + m, n] = sum over rows r of
//           expert e of A[r, m] * B[r, n]: A [rows, out_rows] and B [rows, N]
//           are both read M/N-major, the K loop runs over the expert's own
//           row segment; an expert without rows gets zeros (epi 1) or is left
//           untouched (epi 2).
// Structure is the dense kernel's (one CTA per SM, TMA producer warp, one MMA
// thread, four epilogue warps, double-buffered TMEM accumulator); every wait is
// bounded and reports through `status`.
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int GBN = 256;
constexpr int kMaxExperts = 1024;
using GCfg = GemmCfg<GBN>;
constexpr int kGroupedSmem = GCfg::kSmemBytes + (kMaxExperts + 1) * 4;

struct GroupedParams {
  GemmParams g;        // M = row capacity (mode 0) or experts * out_rows (mode 1)
  const int* offsets;  // [experts + 1] row offsets (multiples of 128)
  int experts;
  int b_rows;          // mode 0: rows of one expert in the stacked B tensor
  int out_rows;        // mode 1: output rows per expert (multiple of 128)
};

struct TileInfo {
  int m0, n0;          // output tile origin (row within C, column)
  int mb_in;           // mode 1: row block within the expert's output
  int expert;
  int kb0, kb1;        // K blocks [kb0, kb1)
};

template <int MODE>
__device__ __forceinline__ TileInfo tile_info(int tile, const int* off, const GroupedParams& p, int num_n) {
  TileInfo t;
  if constexpr (MODE == 0) {
    const int num_m = off[p.experts] / BM;
    int mb, nb;
    tile_coords(tile, num_m, num_n, mb, nb);
    const int r0 = mb * BM;
    int lo = 0, hi = p.experts;  // largest e with off[e] <= r0
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (off[mid] <= r0) lo = mid; else hi = mid;
    }
    t.m0 = r0;
    t.n0 = nb * GBN;
    t.mb_in = mb;
    t.expert = lo;
    t.kb0 = 0;
    t.kb1 = (p.g.K + BK - 1) / BK;
  } else {
    const int num_mo = p.out_rows / BM;
    const int per = num_mo * num_n;
    const int e = tile / per;
    int mb, nb;
    tile_coords(tile - e * per, num_mo, num_n, mb, nb);
    t.expert = e;
    t.mb_in = mb;
    t.m0 = e * p.out_rows + mb * BM;
    t.n0 = nb * GBN;
    t.kb0 = off[e] / BK;
    t.kb1 = off[e + 1] / BK;
  }
  return t;
}

template <int MODE>
__device__ __forceinline__ int num_tiles_of(const int* off, const GroupedParams& p, int num_n) {
  if constexpr (MODE == 0) return (off[p.experts] / BM) * num_n;
  return p.experts * (p.out_rows / BM) * num_n;
}

template <int MODE, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GroupedParams p) {
  constexpr int S = GCfg::kStages;
  constexpr bool A_MN = MODE == 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * GCfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * GCfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  int* off = reinterpret_cast<int*>(smem + S * GCfg::kStageBytes + 256);  // [experts + 1]

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_n = (p.g.N + GBN - 1) / GBN;

  for (int i = threadIdx.x; i <= p.experts; i += blockDim.x) off[i] = p.offsets[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, GCfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int num_tiles = num_tiles_of<MODE>(off, p, num_n);

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const TileInfo t = tile_info<MODE>(tile, off, p, num_n);
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.g.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], GCfg::kStageBytes);
        uint8_t* a_dst = smA + stage * GCfg::kABytes;
        uint8_t* b_dst = smB + stage * GCfg::kBBytes;
        const int k0 = kb * BK;
        if constexpr (A_MN) {
          const int a0 = t.mb_in * BM;  // column of A = output row within the expert
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * (BK * 128), &tmA, &full[stage], a0 + 64 * j, k0);
        } else {
          tma_load_2d(a_dst, &tmA, &full[stage], k0, t.m0);
        }
        if constexpr (MODE == 1) {
#pragma unroll
          for (int j = 0; j < GBN / 64; ++j) tma_load_2d(b_dst + j * (BK * 128), &tmB, &full[stage], t.n0 + 64 * j, k0);
        } else if constexpr (EPI == 3) {
          const int h0 = t.n0 / 2, base = t.expert * p.b_rows;
          tma_load_2d(b_dst, &tmB, &full[stage], k0, base + h0);
          tma_load_2d(b_dst + (GBN / 2) * 128, &tmB, &full[stage], k0, base + p.g.num_n_half + h0);
        } else if constexpr (B_MN) {
          const int kr = t.expert * p.b_rows + k0;
#pragma unroll
          for (int j = 0; j < GBN / 64; ++j) tma_load_2d(b_dst + j * (BK * 128), &tmB, &full[stage], t.n0 + 64 * j, kr);
        } else {
          tma_load_2d(b_dst, &tmB, &full[stage], k0, t.expert * p.b_rows + t.n0);
        }
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
    constexpr bool b_mn_desc = MODE == 1 || (B_MN && EPI != 3);
    constexpr uint32_t idesc = make_idesc_bf16(BM, GBN, A_MN, b_mn_desc);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const TileInfo t = tile_info<MODE>(tile, off, p, num_n);
      const int b = local & 1;
      if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1u, p.g.status, kTimeoutMma, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * GBN;
      for (int kb = t.kb0; kb < t.kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.g.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smA + stage * GCfg::kABytes);
        const uint32_t b_base = smem_u32(smB + stage * GCfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = A_MN ? make_sw128_desc(a_base + kk * 2048, BK * 128, 1024)
                                   : make_sw128_desc(a_base + kk * 32, 16, 1024);
          const uint64_t bd = b_mn_desc ? make_sw128_desc(b_base + kk * 2048, BK * 128, 1024)
                                        : make_sw128_desc(b_base + kk * 32, 16, 1024);
          umma_f16(d_tmem, ad, bd, idesc, (kb != t.kb0 || kk != 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(&tfull[b]);  // also for an empty K range: the epilogue then writes zeros
    }
    umma_commit(drain);
    mbar_wait(drain, 0, p.g.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const TileInfo t = tile_info<MODE>(tile, off, p, num_n);
      const int b = local & 1;
      if (!mbar_wait_warp(&tfull[b], (local >> 1) & 1, p.g.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = t.m0 + wq * 32 + lane;
      if (t.kb1 > t.kb0) {
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + b * GBN;
        store_acc_row<GBN, EPI>(p.g, t_row, row, t.n0 / GBN);
      } else if (EPI == 1 && row < p.g.M) {
        // an expert without rows: its weight gradient is zero
        float* out = static_cast<float*>(p.g.C) + static_cast<long long>(row) * p.g.ldc;
        for (int c = t.n0; c < min(t.n0 + GBN, p.g.N); ++c) out[c] = 0.f;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, GCfg::kTmemCols);
  }
}

template <int MODE, bool B_MN, int EPI>
void launch_grouped(const CUtensorMap& ta, const CUtensorMap& tb, const GroupedParams& p, int max_tiles,
                    cudaStream_t stream) {
  auto kern = grouped_gemm_kernel<MODE, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGroupedSmem);
    configured = true;
  }
  const int sms = device_sm_count();
  const int grid = max_tiles < sms ? (max_tiles > 0 ? max_tiles : 1) : sms;
  kern<<<grid, kThreads, kGroupedSmem, stream>>>(ta, tb, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("grouped gemm launch: ") + cudaGetErrorString(e));
}

}  // namespace

void grouped_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, bool b_mn, void* C, long long ldc,
                       int rows, int N, int K, const int* offsets, int experts, int b_rows, int mode, int out_rows,
                       int epi, const void* aux, int swiglu_h, int* status, cudaStream_t stream) {
  if (experts < 1 || experts > kMaxExperts) throw std::invalid_argument("grouped gemm: 1..1024 experts");
  if (rows % BM != 0) throw std::invalid_argument("grouped gemm: row capacity must be a multiple of 128");
  CUtensorMap ta, tb;
  GroupedParams p{};
  p.offsets = offsets;
  p.experts = experts;
  p.b_rows = b_rows;
  p.out_rows = out_rows;
  const int num_n = (N + GBN - 1) / GBN;
  if (mode == 1) {
    // weight gradient: A [rows, out_rows], B [rows, N], both read M/N-major; C [experts * out_rows, N]
    if (out_rows % BM != 0) throw std::invalid_argument("grouped wgrad: out_rows must be a multiple of 128");
    if (epi != 1 && epi != 2) throw std::invalid_argument("grouped wgrad: epi must be 1 (fp32) or 2 (fp32 +=)");
    p.g = GemmParams{experts * out_rows, N, K, C, ldc, aux, status, swiglu_h};
    make_tmap_2d_bf16(&ta, A, out_rows, rows, lda, 64, BK);
    make_tmap_2d_bf16(&tb, B, N, rows, ldb, 64, BK);
    const int max_tiles = experts * (out_rows / BM) * num_n;
    if (epi == 1) launch_grouped<1, true, 1>(ta, tb, p, max_tiles, stream);
    else launch_grouped<1, true, 2>(ta, tb, p, max_tiles, stream);
    return;
  }
  p.g = GemmParams{rows, N, K, C, ldc, aux, status, swiglu_h};
  make_tmap_2d_bf16(&ta, A, K, rows, lda, 64, BM);
  const int max_tiles = (rows / BM) * num_n;
  if (epi == 3) {
    if (b_mn) throw std::invalid_argument("grouped gemm epilogue 3 needs B K-major");
    make_tmap_2d_bf16(&tb, B, K, static_cast<long long>(experts) * b_rows, ldb, 64, 128);
    launch_grouped<0, false, 3>(ta, tb, p, max_tiles, stream);
    return;
  }
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, N, static_cast<long long>(experts) * b_rows, ldb, 64, BK);
    switch (epi) {
      case 0: launch_grouped<0, true, 0>(ta, tb, p, max_tiles, stream); break;
      case 4: launch_grouped<0, true, 4>(ta, tb, p, max_tiles, stream); break;
      default: throw std::invalid_argument("grouped gemm (B N-major): epi 0 or 4");
    }
  } else {
    make_tmap_2d_bf16(&tb, B, K, static_cast<long long>(experts) * b_rows, ldb, 64, GBN);
    switch (epi) {
      case 0: launch_grouped<0, false, 0>(ta, tb, p, max_tiles, stream); break;
      case 1: launch_grouped<0, false, 1>(ta, tb, p, max_tiles, stream); break;
      default: throw std::invalid_argument("grouped gemm (B K-major): epi 0, 1 or 3");
    }
  }
}

}  // namespace pb

// Persistent warp-specialized bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M, N] (op)= sum_k A(m, k) * B(n, k)        fp32 accumulation in TMEM
//
// A is given either K-major ([M, K] row-major) or M-major ([K, M] row-major);
// likewise B is N x K K-major ([N, K]) or N-major ([K, N]). These three layouts
// cover every GEMM of a linear layer's training step without any transpose:
//   forward  y  = x  @ W^T : A = x  (K-major), B = W (K-major)
//   dgrad    dx = dy @ W   : A = dy (K-major), B = W (N-major)
//   wgrad    dW = dy^T @ x : A = dy (M-major), B = x (N-major)
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles into a ring of
//               shared-memory stages (128-byte swizzle), completion via mbarrier tx.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) into
//               one of two TMEM accumulators; tcgen05.commit frees smem stages and
//               hands finished accumulators to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, store to
//               global (bf16 / fp32 / fp32 accumulate / fused SwiGLU).
// The double-buffered accumulator lets the epilogue of tile i overlap the MMAs
// of tile i+1. Tiles are visited in GROUP_M-grouped order for L2 reuse.
#include <cstdlib>
#include <stdexcept>

#include "common.cuh"
#include "gemm_common.cuh"
#include "kernels.h"

namespace pb {

namespace {

// EPI: 0 = bf16 store, 1 = fp32 store, 2 = fp32 accumulate (C += acc),
//      4 = SwiGLU backward: acc = dh, aux = [gate | up] -> C = [dgate | dup] (bf16 [M, 2H]),
//      3 = fused SwiGLU: the BN columns hold [gate(BN/2) | up(BN/2)] of the same
//          hidden units; writes bf16 h = silu(gate) * up into C[M, H] and the raw
//          pre-activation [gate | up] into aux-out (bf16 [M, 2H]) for backward.
template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + BK - 1) / BK;

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
    tmem_alloc(tmem_base_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int m0 = mb * BM, n0 = nb * BN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
        uint8_t* a_dst = smA + stage * Cfg::kABytes;
        uint8_t* b_dst = smB + stage * Cfg::kBBytes;
        const int k0 = kb * BK;
        if constexpr (A_MN) {
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * (BK * 128), &tmA, &full[stage], m0 + 64 * j, k0);
        } else {
          tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
        }
        if constexpr (EPI == 3) {
          // gate rows [n0/2, n0/2 + BN/2) and up rows [H + n0/2, ...): one tile holds both halves.
          const int h0 = n0 / 2;
          tma_load_2d(b_dst, &tmB, &full[stage], k0, h0);
          tma_load_2d(b_dst + (BN / 2) * 128, &tmB, &full[stage], k0, p.num_n_half + h0);
        } else if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * (BK * 128), &tmB, &full[stage], n0 + 64 * j, k0);
        } else {
          tma_load_2d(b_dst, &tmB, &full[stage], k0, n0);
        }
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      // Drain: let every load already issued land before the CTA exits.
      for (int i = 0; i < min(issued, S); ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int b = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tempty[b], acc_phase ^ 1u, p.status, kTimeoutMma, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * BN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smA + stage * Cfg::kABytes);
        const uint32_t b_base = smem_u32(smB + stage * Cfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = A_MN ? make_sw128_desc(a_base + kk * 2048, BK * 128, 1024)
                                   : make_sw128_desc(a_base + kk * 32, 16, 1024);
          const uint64_t bd = (B_MN && EPI != 3) ? make_sw128_desc(b_base + kk * 2048, BK * 128, 1024)
                                                 : make_sw128_desc(b_base + kk * 32, 16, 1024);
          umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0);
        }
        umma_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(&tfull[b]);
    }
    // Wait for every MMA this thread issued before anyone frees TMEM.
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int b = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&tfull[b], acc_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = mb * BM + wq * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + b * BN;
      store_acc_row<BN, EPI>(p, t_row, row, nb);
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
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int num_sms, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    configured = true;
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p);
}


// ---------------------------------------------------------------------------- 2-CTA tiles
// A CTA pair (cluster of 2 on neighbouring SMs) computes one 256 x 256 output
// tile with M = 256 tcgen05 MMAs: CTA r holds A rows [128 r, 128 r + 128) and B
// rows (N) [128 r, 128 r + 128) of every K stage and receives D rows
// [128 r, 128 r + 128) in its own TMEM. Per SM this streams 32 KB of operands
// per 64-deep K step instead of the 48 KB of a 1-CTA 128 x 256 tile, for the
// same MMA time -- the 1-CTA kernel is bound by that feed, not by the tensor core.
//   * both CTAs TMA-load their halves; the completion bytes of both land on
//     CTA 0's `full` barrier (CTA 0 expects the pair's total);
//   * CTA 0's MMA thread issues the MMAs and commits `empty` / `tfull` to the
//     barriers of both CTAs (one commit per CTA);
//   * both CTAs' epilogues read their own TMEM and arrive on CTA 0's `tempty`;
//   * TMEM is allocated and freed by warp 1 of both CTAs (cta_group::2).
// The pair kernel runs 10 warps: producer, MMA issuer and EIGHT epilogue warps. Two warps
// share each TMEM lane quarter and split the tile's columns, so each SM sub-partition has two
// epilogue warps to interleave (TMEM-load latency, conversion, SwiGLU math) and the epilogue
// keeps up with the MMAs of a short-K tile (K = 512: about 2 us of tensor work per tile).
constexpr int kPairThreads = 320;
constexpr int kPairEpiWarps = 8;

// TOUT: the epilogue stages each 32-column chunk in shared memory and writes it with a
// bulk tensor store (bf16 / fp32) or bulk tensor reduce-add (fp32 +=), instead of one
// 16-byte store per row and thread. A warp's 32 rows x 64 or 128 bytes leave as one
// asynchronous copy, so the writes are full-line and run while the next chunk is loaded
// from TMEM. One staging buffer per epilogue warp and output stream costs one or two
// pipeline stages of shared memory.
template <int EPI, bool TOUT>
struct PairCfg {
  static constexpr int kStages = !TOUT ? 7 : (EPI == 3 ? 5 : 6);
  static constexpr int kABytes = 128 * BK * 2;  // this CTA's 128 rows of A
  static constexpr int kBBytes = 128 * BK * 2;  // this CTA's 128 rows (N) of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  // per epilogue warp: streams x (32 rows x 32 columns)
  static constexpr int kChunkBytes = (EPI == 1 || EPI == 2) ? 4096 : 2048;
  static constexpr int kStreams = EPI == 3 ? 3 : (EPI == 4 ? 2 : 1);  // epilogue 5 reuses its one buffer
  static constexpr int kStgPerWarp = TOUT ? kStreams * kChunkBytes : 0;
  static constexpr int kSmemBytes = kStages * kStageBytes + kPairEpiWarps * kStgPerWarp + 1024 + 256;
  static_assert(kSmemBytes <= 232448, "pair GEMM shared memory exceeds the per-CTA limit");
};

// TMA-store epilogue of one pair tile for this warp's 32 rows (row0 .. row0 + 31). Rows and
// columns outside the output are clipped by the tensor maps, so no edge handling is needed.
// Columns [c_lo, c_hi) of the accumulator (hidden units for the SwiGLU epilogue). The warp's
// staging buffer is reused once the previous chunk's bulk stores have read it.
template <int EPI>
__device__ __forceinline__ void epilogue_tma_tile(uint32_t t_base, int row0, int nb, int c_lo, int c_hi,
                                                  uint8_t* stg, int lane, const CUtensorMap* tmC,
                                                  const CUtensorMap* tmG, const CUtensorMap* tmU) {
  constexpr int TN = 256;
  if constexpr (EPI == 3) {
    const int h0 = nb * (TN / 2);
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(t_base + c, g);
      tmem_ld_32x32b_x32(t_base + TN / 2 + c, u);
      tmem_wait_ld();
      uint32_t hv[16], gv[16], uv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // gate / up rounded to bf16 first so forward and backward see the same values
        const __nv_bfloat162 gb = __floats2bfloat162_rn(__uint_as_float(g[2 * j]), __uint_as_float(g[2 * j + 1]));
        const __nv_bfloat162 ub = __floats2bfloat162_rn(__uint_as_float(u[2 * j]), __uint_as_float(u[2 * j + 1]));
        const float2 gf = __bfloat1622float2(gb), uf = __bfloat1622float2(ub);
        const float s0 = gf.x * sigmoid_fast(gf.x), s1 = gf.y * sigmoid_fast(gf.y);
        hv[j] = pack_bf16x2(s0 * uf.x, s1 * uf.y);
        gv[j] = *reinterpret_cast<const uint32_t*>(&gb);
        uv[j] = *reinterpret_cast<const uint32_t*>(&ub);
      }
      uint8_t* buf = stg;
      if (lane == 0) tma_store_wait_read();  // the previous chunk's stores have read the buffer
      __syncwarp();
      stage_row<4>(buf, lane, hv);
      stage_row<4>(buf + 2048, lane, gv);
      stage_row<4>(buf + 4096, lane, uv);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, buf, h0 + c, row0);
        tma_store_2d(tmG, buf + 2048, h0 + c, row0);
        tma_store_2d(tmU, buf + 4096, h0 + c, row0);
        tma_store_commit();
      }
    }
  } else if constexpr (EPI == 0) {
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_base + c, v);
      tmem_wait_ld();
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
      uint8_t* buf = stg;
      if (lane == 0) tma_store_wait_read();
      __syncwarp();
      stage_row<4>(buf, lane, pk);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, buf, nb * TN + c, row0);
        tma_store_commit();
      }
    }
  } else {
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_base + c, v);
      tmem_wait_ld();
      uint8_t* buf = stg;
      if (lane == 0) tma_store_wait_read();
      __syncwarp();
      stage_row<8>(buf, lane, v);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (EPI == 2) {
          tma_reduce_add_2d(tmC, buf, nb * TN + c, row0);
        } else {
          tma_store_2d(tmC, buf, nb * TN + c, row0);
        }
        tma_store_commit();
      }
    }
  }
}

// SwiGLU backward epilogue: the saved pre-activations [gate | up] of a 32 x 32 chunk are
// fetched with coalesced 16-byte loads (lane l: rows l / 4 + 8 j, column group l % 4) one
// chunk ahead, passed through the warp's staging buffer to the lane that owns each row, and
// combined with dh from TMEM; dgate / dup leave through the same buffer as bulk tensor stores.
__device__ __forceinline__ void swiglu_bwd_prefetch(const GemmParams& p, int row0, int col, int lane, uint4 (&g)[4],
                                                    uint4 (&u)[4]) {
  const int H = p.num_n_half;
  const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(p.aux);
  const int cc = col + (lane & 3) * 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = row0 + (lane >> 2) + 8 * j;
    if (r < p.M && cc < H) {
      const __nv_bfloat16* src = gu + static_cast<long long>(r) * (2LL * H) + cc;
      g[j] = __ldg(reinterpret_cast<const uint4*>(src));
      u[j] = __ldg(reinterpret_cast<const uint4*>(src + H));
    } else {
      g[j] = make_uint4(0u, 0u, 0u, 0u);
      u[j] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

__device__ __forceinline__ void epilogue_swiglu_bwd_tile(const GemmParams& p, uint32_t t_base, int row0, int nb,
                                                         int c_lo, int c_hi, uint8_t* stg, int lane, uint4 (&g)[4],
                                                         uint4 (&u)[4], const CUtensorMap* tmDG,
                                                         const CUtensorMap* tmDU) {
  constexpr int TN = 256;
#pragma unroll 1
  for (int c = c_lo; c < c_hi; c += 32) {
    const int col = nb * TN + c;
    if (lane == 0) tma_store_wait_read();  // the previous chunk's stores have read the buffer
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = (lane >> 2) + 8 * j;
      const int off = r * 64 + swz_chunk<4>(r, lane & 3) * 16;
      *reinterpret_cast<uint4*>(stg + off) = g[j];
      *reinterpret_cast<uint4*>(stg + 2048 + off) = u[j];
    }
    __syncwarp();
    if (c + 32 < c_hi) swiglu_bwd_prefetch(p, row0, col + 32, lane, g, u);
    uint32_t gw[16], uw[16];
    load_row<4>(stg, lane, gw);
    load_row<4>(stg + 2048, lane, uw);
    __syncwarp();
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_base + c, v);
    tmem_wait_ld();
    uint32_t dg[16], du[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 gf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[j]));
      const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[j]));
      // dh rounded to bf16 first, as the unfused path stores it
      const float2 d = __bfloat1622float2(__floats2bfloat162_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])));
      const float s0 = sigmoid_fast(gf.x), s1 = sigmoid_fast(gf.y);
      du[j] = pack_bf16x2(d.x * (gf.x * s0), d.y * (gf.y * s1));
      dg[j] = pack_bf16x2(d.x * uf.x * s0 * (1.f + gf.x * (1.f - s0)), d.y * uf.y * s1 * (1.f + gf.y * (1.f - s1)));
    }
    stage_row<4>(stg, lane, dg);
    stage_row<4>(stg + 2048, lane, du);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmDG, stg, col, row0);
      tma_store_2d(tmDU, stg + 2048, col, row0);
      tma_store_commit();
    }
  }
}

// Scaled-add epilogue: the matching 32 x 32 chunk of aux is fetched one chunk ahead with
// coalesced 16-byte loads (lane l: rows l / 4 + 8 j, column group l % 4), handed to the lane
// that owns each row through the warp's staging buffer, combined with the accumulator row,
// and the bf16 result leaves through the same buffer as a bulk tensor store.
__device__ __forceinline__ void axpby_prefetch(const GemmParams& p, int row0, int col, int lane, uint4 (&x)[4]) {
  const __nv_bfloat16* aux = static_cast<const __nv_bfloat16*>(p.aux);
  const int cc = col + (lane & 3) * 8;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = row0 + (lane >> 2) + 8 * j;
    x[j] = (r < p.M * p.batch && cc < p.N)
               ? __ldg(reinterpret_cast<const uint4*>(aux + static_cast<long long>(r) * p.ldc + cc))
                                 : make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ void epilogue_axpby_tile(const GemmParams& p, uint32_t t_base, int row0, int nb, int c_lo,
                                                    int c_hi, uint8_t* stg, int lane, uint4 (&x)[4],
                                                    const CUtensorMap* tmC) {
  constexpr int TN = 256;
#pragma unroll 1
  for (int c = c_lo; c < c_hi; c += 32) {
    const int col = nb * TN + c;
    if (lane == 0) tma_store_wait_read();  // the previous chunk's store has read the buffer
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = (lane >> 2) + 8 * j;
      *reinterpret_cast<uint4*>(stg + r * 64 + swz_chunk<4>(r, lane & 3) * 16) = x[j];
    }
    __syncwarp();
    uint32_t xw[16];
    load_row<4>(stg, lane, xw);
    __syncwarp();
    if (c + 32 < c_hi) axpby_prefetch(p, row0, col + 32, lane, x);
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_base + c, v);
    tmem_wait_ld();
    uint32_t out[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[j]));
      out[j] = pack_bf16x2(fmaf(p.alpha, __uint_as_float(v[2 * j]), p.beta * a.x),
                           fmaf(p.alpha, __uint_as_float(v[2 * j + 1]), p.beta * a.y));
    }
    stage_row<4>(stg, lane, out);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, stg, col, row0);
      tma_store_commit();
    }
  }
}

template <bool A_MN, bool B_MN, int EPI, bool TOUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmG,
                     const __grid_constant__ CUtensorMap tmU, const GemmParams p) {
  using Cfg = PairCfg<EPI, TOUT>;
  constexpr int S = Cfg::kStages;
  constexpr int TM = 256, TN = 256;  // pair tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * Cfg::kABytes;
  uint8_t* stg = smem + S * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + kPairEpiWarps * Cfg::kStgPerWarp);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* peer_done = drain + 1;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(peer_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (p.M + TM - 1) / TM;
  const int num_n = (p.N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + BK - 1) / BK;
  // Work unit u = (tile u / splits, K slice u % splits); slices accumulate through the
  // fp32 reduce-add epilogue, so a few output tiles with a long K still fill every SM.
  const int splits = p.splits;
  // Batched launches stack the products along the outer axis of every operand: product b owns rows
  // [b M, (b + 1) M) of A (K-major) and C, [b N, ...) of B (K-major), [b K, ...) of an MN-major operand.
  const int num_units = num_tiles * splits * p.batch;
  const auto k_range = [&](int u, int& lo, int& hi) {
    const int ks = u % splits;
    lo = ks * num_kb / splits;
    hi = (ks + 1) * num_kb / splits;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kPairEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    mbar_init(peer_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (TOUT) {
      prefetch_tmap(&tmC);
      if constexpr (EPI == 3 || EPI == 4) prefetch_tmap(&tmG);
      if constexpr (EPI == 3) prefetch_tmap(&tmU);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits of both CTAs visible before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const uint32_t full0 = cluster_addr(full, 0);
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int u = pair; u < num_units && ok; u += num_pairs) {
      int mb, nb, kb_lo, kb_hi;
      tile_coords((u / splits) % num_tiles, num_m, num_n, mb, nb);
      k_range(u, kb_lo, kb_hi);
      const int bi = u / (splits * num_tiles);
      const int m0 = mb * TM + 128 * static_cast<int>(rank) + (A_MN ? 0 : bi * p.M);
      const int n0 = nb * TN + 128 * static_cast<int>(rank) + (B_MN ? 0 : bi * p.N);
      const int kofs_a = A_MN ? bi * p.K : 0, kofs_b = B_MN ? bi * p.K : 0;
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
        const uint32_t bar = full0 + 8u * stage;
        uint8_t* a_dst = smA + stage * Cfg::kABytes;
        uint8_t* b_dst = smB + stage * Cfg::kBBytes;
        const int k0 = kb * BK;
        if constexpr (A_MN) {
          tma_load_2d_pair(a_dst, &tmA, bar, m0, k0 + kofs_a);
          tma_load_2d_pair(a_dst + BK * 128, &tmA, bar, m0 + 64, k0 + kofs_a);
        } else {
          tma_load_2d_pair(a_dst, &tmA, bar, k0, m0);
        }
        if constexpr (EPI == 3) {
          // Pair tile columns [0, 128) = gate rows h0.., [128, 256) = up rows H + h0..
          const int h0 = nb * (TN / 2);
          tma_load_2d_pair(b_dst, &tmB, bar, k0, leader ? h0 : p.num_n_half + h0);
        } else if constexpr (B_MN) {
          tma_load_2d_pair(b_dst, &tmB, bar, n0, k0 + kofs_b);
          tma_load_2d_pair(b_dst + BK * 128, &tmB, bar, n0 + 64, k0 + kofs_b);
        } else {
          tma_load_2d_pair(b_dst, &tmB, bar, k0, n0);
        }
        ++issued;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && leader) {
      // Drain: the pair's loads already issued complete on this CTA's barriers.
      for (int i = 0; i < min(issued, S); ++i) {
        if (--stage < 0) {
          stage = S - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    if (leader) {
      // ------------------------------------------------------------ MMA issuer (CTA 0)
      constexpr uint32_t idesc = make_idesc_bf16(TM, TN, A_MN, B_MN);
      const uint32_t empty1 = cluster_addr(empty, 1);
      const uint32_t tfull1 = cluster_addr(tfull, 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += num_pairs, ++local) {
        const int b = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        int kb_lo, kb_hi;
        k_range(u, kb_lo, kb_hi);
        if (!mbar_wait(&tempty[b], acc_phase ^ 1u, p.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * TN;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smA + stage * Cfg::kABytes);
          const uint32_t b_base = smem_u32(smB + stage * Cfg::kBBytes);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(a_base + kk * 2048, BK * 128, 1024)
                                     : make_sw128_desc(a_base + kk * 32, 16, 1024);
            const uint64_t bd = (B_MN && EPI != 3) ? make_sw128_desc(b_base + kk * 2048, BK * 128, 1024)
                                                   : make_sw128_desc(b_base + kk * 32, 16, 1024);
            umma_f16_pair(d_tmem, ad, bd, idesc, kb > kb_lo || kk > 0);
          }
          umma_commit_pair(&empty[stage]);
          umma_commit_pair_to(empty1 + 8u * stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          umma_commit_pair(&tfull[b]);
          umma_commit_pair_to(tfull1 + 8u * b);
        }
      }
      umma_commit_pair(drain);
      mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
      mbar_arrive_cluster(cluster_addr(peer_done, 1));  // CTA 1 may free its TMEM now
    } else {
      // CTA 1 frees its TMEM only after CTA 0's MMAs (which write it) are complete.
      mbar_wait(peer_done, 0, p.status, kTimeoutDrain, nullptr);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int wq = warp & 3;           // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;  // which half of the tile's columns
    constexpr int kSpan = (EPI == 3 ? TN / 2 : TN) / 2;  // SwiGLU: a tile holds TN / 2 hidden units
    const int c_lo = half * kSpan, c_hi = c_lo + kSpan;
    const uint32_t tempty0 = cluster_addr(tempty, 0);
    uint8_t* my_stg = stg + (warp - 2) * Cfg::kStgPerWarp;
    int local = 0;
    for (int u = pair; u < num_units; u += num_pairs, ++local) {
      int mb, nb;
      tile_coords((u / splits) % num_tiles, num_m, num_n, mb, nb);
      const int b = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int row0 = (u / (splits * num_tiles)) * p.M + mb * TM + 128 * static_cast<int>(rank) + wq * 32;
      [[maybe_unused]] uint4 pre_g[4], pre_u[4];
      if constexpr (TOUT && EPI == 4) swiglu_bwd_prefetch(p, row0, nb * TN + c_lo, lane, pre_g, pre_u);
      if constexpr (TOUT && EPI == 5) axpby_prefetch(p, row0, nb * TN + c_lo, lane, pre_g);
      if (!mbar_wait_warp(&tfull[b], acc_phase, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + b * TN;
      if constexpr (TOUT && EPI == 4) {
        epilogue_swiglu_bwd_tile(p, t_row, row0, nb, c_lo, c_hi, my_stg, lane, pre_g, pre_u, &tmC, &tmG);
      } else if constexpr (TOUT && EPI == 5) {
        epilogue_axpby_tile(p, t_row, row0, nb, c_lo, c_hi, my_stg, lane, pre_g, &tmC);
      } else if constexpr (TOUT) {
        epilogue_tma_tile<EPI>(t_row, row0, nb, c_lo, c_hi, my_stg, lane, &tmC, &tmG, &tmU);
      } else {
        store_acc_row<TN, EPI>(p, t_row, row0 + lane, nb, c_lo, c_hi);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * b);
    }
    if constexpr (TOUT) {
      if (lane == 0) tma_store_wait_all();  // shared staging is read and global writes are done before exit
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrive may target a CTA that has exited
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

template <bool A_MN, bool B_MN, int EPI, bool TOUT>
void launch_pair_k(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tg,
                   const CUtensorMap& tu, const GemmParams& p, int num_sms, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI, TOUT>;
  using Cfg = PairCfg<EPI, TOUT>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    configured = true;
  }
  const int units = ((p.M + 255) / 256) * ((p.N + 255) / 256) * p.splits * p.batch;
  const int pairs = units < num_sms / 2 ? units : num_sms / 2;
  kern<<<2 * pairs, kPairThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, tg, tu, p);
}

// Split-K factor for an fp32-output GEMM. A work unit costs 1/s of a full-K tile's MMAs plus
// one tile epilogue (an fp32 reduce-add of 256 KB, modelled as 1024 / K of the MMA time), and
// units run in waves of `pairs`: s minimizes ceil(tiles * s / pairs) * (1/s + 1024 / K) and is
// kept only when that beats one slice by 5 % (at most 8 slices of at least 8 K blocks each).
int choose_splits(const GemmParams& p, int num_sms) {
  static const bool on = [] {
    const char* e = std::getenv("PRIML_B200_GEMM_SPLITK");  // 0 disables (A/B measurements)
    return e == nullptr || e[0] != '0';
  }();
  if (!on) return 1;
  const int tiles = ((p.M + 255) / 256) * ((p.N + 255) / 256);
  const int pairs = num_sms / 2;
  const int num_kb = (p.K + BK - 1) / BK;
  const double epi = 1024.0 / static_cast<double>(p.K);
  const auto cost = [&](int s) {
    return static_cast<double>((tiles * s + pairs - 1) / pairs) * (1.0 / s + epi);
  };
  int best = 1;
  double best_cost = cost(1);
  for (int s = 2; s <= 8 && num_kb >= 8 * s; ++s) {
    if (cost(s) < best_cost) {
      best = s;
      best_cost = cost(s);
    }
  }
  return best_cost < 0.95 * cost(1) ? best : 1;
}

// Output tensor maps of a TMA-store epilogue (box 32 x 32, swizzled like the staging tiles:
// 64-byte swizzle for bf16, 128-byte for fp32); false (and the per-row store epilogue) when
// the output's base or row stride is not 16-byte aligned.
bool make_out_maps(int epi, void* C, long long ldc, int M, int N, const void* aux, int swiglu_h, CUtensorMap* tc,
                   CUtensorMap* tg, CUtensorMap* tu) {
  const auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(C)) return false;
  if (epi == 0) {
    if ((ldc * 2) % 16 != 0) return false;
    make_tmap_2d_bf16_sw64(tc, C, N, M, ldc, 32, 32);
    return true;
  }
  if (epi == 1 || epi == 2) {
    if ((ldc * 4) % 16 != 0) return false;
    make_tmap_2d_f32_sw128(tc, C, N, M, ldc, 32, 32);
    return true;
  }
  if (epi == 3) {
    const long long H = swiglu_h;
    if ((ldc * 2) % 16 != 0 || H % 8 != 0 || !aligned(aux)) return false;
    const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(aux);
    make_tmap_2d_bf16_sw64(tc, C, H, M, ldc, 32, 32);
    make_tmap_2d_bf16_sw64(tg, gu, H, M, 2 * H, 32, 32);
    make_tmap_2d_bf16_sw64(tu, gu + H, H, M, 2 * H, 32, 32);
    return true;
  }
  if (epi == 5) {
    if ((ldc * 2) % 16 != 0 || N % 8 != 0 || !aligned(aux)) return false;
    make_tmap_2d_bf16_sw64(tc, C, N, M, ldc, 32, 32);
    return true;
  }
  if (epi == 4) {
    // C = dgu [M, 2H]: dgate and dup views; aux = gu read with 16-byte loads
    const long long H = swiglu_h;
    if ((ldc * 2) % 16 != 0 || H % 8 != 0 || !aligned(aux)) return false;
    __nv_bfloat16* dgu = static_cast<__nv_bfloat16*>(C);
    make_tmap_2d_bf16_sw64(tc, dgu, H, M, ldc, 32, 32);
    make_tmap_2d_bf16_sw64(tg, dgu + H, H, M, ldc, 32, 32);
    return true;
  }
  return false;
}

// TMA-store epilogues are on unless PRIML_B200_GEMM_TMA_STORE=0 (kept for A/B measurements).
bool tma_store_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("PRIML_B200_GEMM_TMA_STORE");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// Epilogue 5 exists only as the 2-CTA kernel with bulk tensor stores.
template <bool A_MN, bool B_MN>
void launch_pair_axpby(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, int num_sms, cudaStream_t stream) {
  CUtensorMap tc{}, tg{}, tu{};
  p.splits = 1;
  if (!make_out_maps(5, p.C, p.ldc, p.M, p.N, p.aux, 0, &tc, &tg, &tu)) {
    throw std::invalid_argument("gemm epilogue 5 needs 16-byte aligned C / aux rows and N % 8 == 0");
  }
  launch_pair_k<A_MN, B_MN, 5, true>(ta, tb, tc, tg, tu, p, num_sms, stream);
}

template <bool A_MN, bool B_MN, int EPI>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, int num_sms, cudaStream_t stream) {
  CUtensorMap tc{}, tg{}, tu{};
  p.splits = 1;
  if (tma_store_enabled() && make_out_maps(EPI, p.C, p.ldc, p.M, p.N, p.aux, p.num_n_half, &tc, &tg, &tu)) {
    if constexpr (EPI == 1 || EPI == 2) {
      const int splits = choose_splits(p, num_sms);
      if (splits > 1) {
        // K slices reduce-add into C: a plain store starts from zero
        if (EPI == 1) {
          cudaMemset2DAsync(p.C, static_cast<size_t>(p.ldc) * 4, 0, static_cast<size_t>(p.N) * 4, p.M, stream);
        }
        p.splits = splits;
        launch_pair_k<A_MN, B_MN, 2, true>(ta, tb, tc, tg, tu, p, num_sms, stream);
        return;
      }
    }
    launch_pair_k<A_MN, B_MN, EPI, true>(ta, tb, tc, tg, tu, p, num_sms, stream);
  } else {
    launch_pair_k<A_MN, B_MN, EPI, false>(ta, tb, tc, tg, tu, p, num_sms, stream);
  }
}
}  // namespace

// 2-CTA tiles are on unless PRIML_B200_GEMM_PAIR=0 (kept for A/B measurements of the two tilings).
static bool pair_gemm_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("PRIML_B200_GEMM_PAIR");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// Public entry. Layout flags: a_mn = A stored [K, M]; b_mn = B stored [K, N].
// lda / ldb are the row strides (elements) of A and B as stored.
void gemm_bf16(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C,
               long long ldc, int M, int N, int K, int epi, const void* aux, int swiglu_h, int* status,
               cudaStream_t stream, float alpha, float beta) {
  const int num_sms = device_sm_count();
  CUtensorMap ta, tb;
  GemmParams p{M, N, K, C, ldc, aux, status, swiglu_h};
  p.alpha = alpha;
  p.beta = beta;
  // 2-CTA 256 x 256 tiles once the problem has enough of them; 1-CTA 128 x 256 otherwise.
  const bool pair = M >= 256 && N >= 256 && pair_gemm_enabled();
  // A tile: 128 (M) x 64 (K) per CTA in both kernels.
  if (a_mn) {
    make_tmap_2d_bf16(&ta, A, /*inner=*/M, /*outer=*/K, lda, /*box_inner=*/64, /*box_outer=*/BK);
  } else {
    make_tmap_2d_bf16(&ta, A, K, M, lda, 64, BM);
  }
  if (epi == 3) {
    // B = up_proj weight [2H, K] (K-major); tile rows are split gate / up.
    make_tmap_2d_bf16(&tb, B, K, 2 * swiglu_h, ldb, 64, 128);
    if (pair) {
      launch_pair<false, false, 3>(ta, tb, p, num_sms, stream);
    } else {
      launch<256, false, false, 3>(ta, tb, p, num_sms, stream);
    }
    return;
  }
  constexpr int BN = 256;
  if (epi == 4) {
    // dgu = swiglu'(gu) * (dy @ W_down): A = dy (K-major), B = W_down stored [K, N = H].
    if (a_mn || !b_mn) throw std::invalid_argument("gemm epilogue 4 needs A K-major and B N-major");
    make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, BK);
    if (pair) {
      launch_pair<false, true, 4>(ta, tb, p, num_sms, stream);
    } else {
      launch<BN, false, true, 4>(ta, tb, p, num_sms, stream);
    }
    return;
  }
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, BK);
  } else {
    make_tmap_2d_bf16(&tb, B, K, N, ldb, 64, pair ? 128 : BN);
  }
  if (epi == 5) {
    if (!pair) throw std::invalid_argument("gemm epilogue 5 needs M >= 256 and N >= 256 (2-CTA tiles)");
    if (a_mn && b_mn) {
      launch_pair_axpby<true, true>(ta, tb, p, num_sms, stream);
    } else if (a_mn) {
      launch_pair_axpby<true, false>(ta, tb, p, num_sms, stream);
    } else if (b_mn) {
      launch_pair_axpby<false, true>(ta, tb, p, num_sms, stream);
    } else {
      launch_pair_axpby<false, false>(ta, tb, p, num_sms, stream);
    }
    return;
  }
#define PB_DISPATCH(AM, BMJ)                                                                  \
  if (pair) {                                                                                 \
    switch (epi) {                                                                            \
      case 0: launch_pair<AM, BMJ, 0>(ta, tb, p, num_sms, stream); break;                     \
      case 1: launch_pair<AM, BMJ, 1>(ta, tb, p, num_sms, stream); break;                     \
      default: launch_pair<AM, BMJ, 2>(ta, tb, p, num_sms, stream); break;                    \
    }                                                                                         \
  } else {                                                                                    \
    switch (epi) {                                                                            \
      case 0: launch<BN, AM, BMJ, 0>(ta, tb, p, num_sms, stream); break;                      \
      case 1: launch<BN, AM, BMJ, 1>(ta, tb, p, num_sms, stream); break;                      \
      default: launch<BN, AM, BMJ, 2>(ta, tb, p, num_sms, stream); break;                     \
    }                                                                                         \
  }
  if (!a_mn && !b_mn) {
    PB_DISPATCH(false, false)
  } else if (!a_mn && b_mn) {
    PB_DISPATCH(false, true)
  } else if (a_mn && !b_mn) {
    PB_DISPATCH(true, false)
  } else {
    PB_DISPATCH(true, true)
  }
#undef PB_DISPATCH
}

// Batched entry: `batch` independent products C_b = A_b B_b^T (epilogues 0 and 5), each operand a
// stack of equal matrices along its outer axis (row strides lda / ldb / ldc within and across them).
// One persistent launch covers every product's tiles. Needs M, N multiples of 256 and K of 64, so
// that no tile reaches into the next product.
void gemm_bf16_batched(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C,
                       long long ldc, int M, int N, int K, int batch, int epi, const void* aux, int* status,
                       cudaStream_t stream, float alpha, float beta) {
  if (M % 256 != 0 || N % 256 != 0 || K % 64 != 0 || batch < 1 || (epi != 0 && epi != 5))
    throw std::invalid_argument("batched GEMM needs M, N % 256 == 0, K % 64 == 0 and epilogue 0 or 5");
  const int num_sms = device_sm_count();
  CUtensorMap ta, tb, tc{}, tg{}, tu{};
  GemmParams p{M, N, K, C, ldc, aux, status, 0};
  p.alpha = alpha;
  p.beta = beta;
  p.batch = batch;
  const long long rows_a = static_cast<long long>(a_mn ? K : M) * batch;
  const long long rows_b = static_cast<long long>(b_mn ? K : N) * batch;
  if (a_mn) {
    make_tmap_2d_bf16(&ta, A, M, rows_a, lda, 64, BK);
  } else {
    make_tmap_2d_bf16(&ta, A, K, rows_a, lda, 64, BM);
  }
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, N, rows_b, ldb, 64, BK);
  } else {
    make_tmap_2d_bf16(&tb, B, K, rows_b, ldb, 64, 128);
  }
  if (!make_out_maps(epi, C, ldc, static_cast<int>(static_cast<long long>(M) * batch), N, aux, 0, &tc, &tg, &tu))
    throw std::invalid_argument("batched GEMM needs 16-byte aligned C rows (and aux rows)");
#define PB_BATCHED(AM, BMJ)                                                                    \
  if (epi == 5) {                                                                              \
    launch_pair_k<AM, BMJ, 5, true>(ta, tb, tc, tg, tu, p, num_sms, stream);                   \
  } else {                                                                                     \
    launch_pair_k<AM, BMJ, 0, true>(ta, tb, tc, tg, tu, p, num_sms, stream);                   \
  }
  if (!a_mn && !b_mn) {
    PB_BATCHED(false, false)
  } else if (!a_mn && b_mn) {
    PB_BATCHED(false, true)
  } else if (a_mn && !b_mn) {
    PB_BATCHED(true, false)
  } else {
    PB_BATCHED(true, true)
  }
#undef PB_BATCHED
}

}  // namespace pb

// Grouped expert GEMMs fused with the expert-parallel token exchange (sm_100a:
// tcgen05 + TMEM + TMA, peer loads and stores over NVLink in the same kernel).
//
// Every rank owns `experts` experts and lays the rows it receives out as
// 128-aligned per-expert segments (device offsets, as in grouped_gemm.cu).
// Each rank also has two IPC-mapped row buffers: `send` (rows this rank offers
// to the expert owners) and `recv` (rows the owners return to this rank).
//
//   ep_pull_gemm   C = A @ B_e^T with A gathered from the sources:
//     receive row r of this rank is row (row_src[r] & 0xFFFFFF) of the send
//     buffer of rank row_src[r] >> 24 (-1: a padding row, written as zeros).
//     One cooperative launch. Two copy warps per CTA pull 16-row pieces over
//     NVLink (16-byte peer loads, 16 in flight per lane) into `a_local`, the
//     A operand that the caller keeps for the weight gradient, and count
//     every piece on its 128-row chunk; the TMA producer loads a chunk once
//     all its pieces are in (bounded wait), so tiles of early chunks run on
//     the tensor cores while later chunks are still crossing NVLink. At
//     kernel start the rank announces its send buffer's epoch on every peer;
//     the copy warps wait for a source's announcement before the first load
//     from it, and the last copy warp of the grid counts this rank on every
//     source ("done reading your send buffer").
//     Epilogues: 3 (SwiGLU forward: h and the gate/up pre-activation) and
//     4 (SwiGLU backward), both into local memory.
//   ep_push_gemm   rows of A @ B_e^T go straight to their sources:
//     output row r is stored into row (row_dst[r] & 0xFFFFFF) of the recv
//     buffer of rank row_dst[r] >> 24 (padding rows are not stored). The
//     epilogue stages 64-column slices in shared memory and every lane
//     bulk-stores its row's 128 bytes to the peer; before the first store it
//     waits until every source has consumed the previous epoch's rows; the
//     last CTA to finish counts this rank on every destination.
//   ep_combine     on the source, once every owner has stored its rows:
//     out[t] = sum_j w[t, j] * recv[t * k + j] (w = 1 without weights), in
//     fp32, optionally keeping a copy of the received rows; then frees the
//     recv buffer on every owner.
//   ep_expand      out[t * k + j] = w[t, j] * dy[t] into the send buffer and
//     dw[t, j] = <dy[t], y[t * k + j]> (the backward of ep_combine).
//
// Dispatch is a pull (the owner reads the rows once, into the operand it keeps
// anyway), combine a push (the rows leave from the GEMM's epilogue), so each
// row crosses NVLink once per direction and no separate exchange kernel runs.
// Every cross-rank wait is bounded by %globaltimer and reports kTimeoutPeer.
// TMA loads read this GPU's memory only (a_local and the weights); peer
// memory is touched by plain loads and bulk stores.
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "gemm_common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int EBN = 256;
using ECfg = GemmCfg<EBN>;
constexpr int kEpMaxExperts = 512;
constexpr int kEpPieceRows = 16;
constexpr int kEpPiecesPerChunk = BM / kEpPieceRows;
constexpr int kEpOutCols = 64;
constexpr int kEpOutPitch = kEpOutCols * 2 + 16;
constexpr int kEpOutWarpBytes = 32 * kEpOutPitch;
// Segment offsets in shared memory, padded to 128 bytes: the push epilogue's staging rows follow
// them and are read by bulk copies, which need 16-byte aligned shared addresses.
constexpr int kEpOffBytes = ((kEpMaxExperts + 1) * 4 + 127) / 128 * 128;
static_assert(kEpOffBytes % 128 == 0 && kEpOutPitch % 16 == 0 && kEpOutWarpBytes % 16 == 0,
              "staging rows must stay 16-byte aligned");
static_assert(ECfg::kSmemBytes - 1024 - 256 == ECfg::kStages * ECfg::kStageBytes, "shared-memory layout");
constexpr int kEpPullSmem = ECfg::kSmemBytes + kEpOffBytes;
constexpr int kEpPushSmem = ECfg::kSmemBytes + kEpOffBytes + 4 * kEpOutWarpBytes;

__device__ __forceinline__ void red_add_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin (sleeping between polls) until ready() or the abort flag; false after timeout_ns.
template <typename F>
__device__ bool wait_until(F ready, volatile int* abort_flag, long long timeout_ns, int* status) {
  const unsigned long long t0 = globaltimer();
  while (!ready()) {
    if (abort_flag != nullptr && *abort_flag) return false;
    if (static_cast<long long>(globaltimer() - t0) > timeout_ns) {
      record_error(status, kTimeoutPeer);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ unsigned long long* sig(const EpGemmParams& p, int rank, int word) {
  return reinterpret_cast<unsigned long long*>(p.signal[rank]) + word;
}

// Output tile -> (row block, column block, expert); n fastest within groups of 16 row blocks.
__device__ __forceinline__ void ep_tile(int tile, const int* off, int experts, int num_m, int num_n, int& m0, int& n0,
                                        int& expert) {
  int mb, nb;
  tile_coords(tile, num_m, num_n, mb, nb);
  m0 = mb * BM;
  n0 = nb * EBN;
  int lo = 0, hi = experts;  // largest e with off[e] <= m0
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (off[mid] <= m0) lo = mid; else hi = mid;
  }
  expert = lo;
}

// PUSH: stage one lane's 64-column slice and bulk-store it to its destination row.
__device__ __forceinline__ void push_slice(const uint32_t (&v)[64], uint8_t* my_row, __nv_bfloat16* dst, int ncols) {
  tma_store_wait_read();  // the previous slice has left the staging row
  uint4* s4 = reinterpret_cast<uint4*>(my_row);
#pragma unroll
  for (int q = 0; q < 8; ++q)
    s4[q] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * q]), __uint_as_float(v[8 * q + 1])),
                       pack_bf16x2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3])),
                       pack_bf16x2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5])),
                       pack_bf16x2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7])));
  fence_proxy_async_smem();
  bulk_store(dst, my_row, static_cast<uint32_t>(ncols) * 2u);
  tma_store_commit();
}

template <bool PULL, bool B_MN, int EPI>
__global__ void __launch_bounds__(PULL ? 256 : 192, 1)
    ep_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const EpGemmParams p) {
  constexpr int S = ECfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * ECfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * ECfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* off = reinterpret_cast<int*>(smem + S * ECfg::kStageBytes + 256);  // [experts + 1]
  uint8_t* stage_out = smem + S * ECfg::kStageBytes + 256 + kEpOffBytes;  // PUSH: [4 warps][32 rows][pitch]

  const int warp = warp_id(), lane = lane_id();
  const int num_n = (p.N + EBN - 1) / EBN;
  GemmParams g{};  // the local epilogue's view (pull)
  g.M = p.M;
  g.N = p.N;
  g.K = p.K;
  g.C = p.C;
  g.ldc = p.ldc;
  g.aux = p.aux;
  g.status = p.status;
  g.num_n_half = p.swiglu_h;
  const int num_kb = (p.K + BK - 1) / BK;

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
    tmem_alloc(tmem_slot, ECfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_m = min(off[p.experts], p.M) / BM;  // rows past the capacity are never read or written
  const int num_tiles = num_m * num_n;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      int m0, n0, e;
      ep_tile(tile, off, p.experts, num_m, num_n, m0, n0, e);
      if constexpr (PULL) {
        const unsigned int* flag = p.chunk_flags + m0 / BM;
        if (!wait_until([&] { return ld_acquire_gpu(flag) >= static_cast<unsigned int>(kEpPiecesPerChunk); },
                        abort_flag, p.timeout_ns, p.status)) {
          ok = false;
          break;
        }
        // the chunk was written by generic stores of other CTAs; the TMA (async proxy) reads it next
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], ECfg::kStageBytes);
        uint8_t* a_dst = smA + stage * ECfg::kABytes;
        uint8_t* b_dst = smB + stage * ECfg::kBBytes;
        const int k0 = kb * BK;
        tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
        if constexpr (EPI == 3) {
          const int h0 = n0 / 2, base = e * p.b_rows;
          tma_load_2d(b_dst, &tmB, &full[stage], k0, base + h0);
          tma_load_2d(b_dst + (EBN / 2) * 128, &tmB, &full[stage], k0, base + p.swiglu_h + h0);
        } else if constexpr (B_MN) {
          const int kr = e * p.b_rows + k0;
#pragma unroll
          for (int j = 0; j < EBN / 64; ++j) tma_load_2d(b_dst + j * (BK * 128), &tmB, &full[stage], n0 + 64 * j, kr);
        } else {
          tma_load_2d(b_dst, &tmB, &full[stage], k0, e * p.b_rows + n0);
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
        mbar_wait(&full[stage], phase, p.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr bool b_mn_desc = B_MN && EPI != 3;
    constexpr uint32_t idesc = make_idesc_bf16(BM, EBN, false, b_mn_desc);
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      const int b = local & 1;
      if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1u, p.status, kTimeoutMma, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * EBN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smA + stage * ECfg::kABytes);
        const uint32_t b_base = smem_u32(smB + stage * ECfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = make_sw128_desc(a_base + kk * 32, 16, 1024);
          const uint64_t bd = b_mn_desc ? make_sw128_desc(b_base + kk * 2048, BK * 128, 1024)
                                        : make_sw128_desc(b_base + kk * 32, 16, 1024);
          umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(&tfull[b]);
    }
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    int local = 0;
    if constexpr (!PULL) {
      // Every source must have consumed the previous epoch's rows before they are overwritten.
      if (p.epoch > 1 && lane == 0) {
        const unsigned long long target = static_cast<unsigned long long>(p.epoch - 1) * p.world;
        const unsigned long long* freed = sig(p, p.rank, kEpSigRecvFree);
        wait_until([&] { return ld_acquire_sys(freed) >= target; }, abort_flag, p.timeout_ns, p.status);
      }
      __syncwarp();
    }
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int m0, n0, e;
      ep_tile(tile, off, p.experts, num_m, num_n, m0, n0, e);
      const int b = local & 1;
      if (!mbar_wait_warp(&tfull[b], (local >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = m0 + wq * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + b * EBN;
      if constexpr (PULL) {
        store_acc_row<EBN, EPI>(g, t_row, row, n0 / EBN);
      } else {
        const int d = row < p.M ? p.row_dst[row] : -1;
        const int dr = d >> 24;
        const long long drow = d & 0xFFFFFF;
        const bool store = d >= 0 && dr < p.world && drow < p.dst_rows;
        if (d >= 0 && !store) record_error(p.status, kBadIndex);
        __nv_bfloat16* dst = store ? reinterpret_cast<__nv_bfloat16*>(p.dst[dr]) + drow * p.N : nullptr;
        uint8_t* my_row = stage_out + wq * kEpOutWarpBytes + lane * kEpOutPitch;
#pragma unroll 1
        for (int c = 0; c < EBN; c += kEpOutCols) {
          uint32_t v[64];
          tmem_ld_32x32b_x32(t_row + c, *reinterpret_cast<uint32_t(*)[32]>(v));
          tmem_ld_32x32b_x32(t_row + c + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          tmem_wait_ld();
          const int col = n0 + c;
          if (!store || col >= p.N || *abort_flag) continue;
          push_slice(v, my_row, dst + col, min(kEpOutCols, p.N - col));  // N % 8 == 0
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if constexpr (!PULL) {
      // this thread's bulk stores are complete, then ordered before the CTA counts itself done
      tma_store_wait_all();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
    }
  } else if (PULL && warp >= 6) {
    // ------------------------------------------------------------ copy warps (dispatch pull)
    const int cw = warp - 6;
    if (blockIdx.x == 0 && cw == 0 && lane == 0) {
      // This rank's send buffer holds this epoch's rows (stream order): tell every rank.
      __threadfence_system();
      for (int q = 0; q < p.world; ++q) st_release_sys(sig(p, q, kEpSigSendReady + p.rank), static_cast<unsigned long long>(p.epoch));
    }
    const int wpr = p.K / 8;  // 16-byte words per row
    unsigned int seen = 0;      // sources whose announcement this warp has seen
    bool ok = true;
    const int pieces = num_m * kEpPiecesPerChunk;
    for (int w = cw * gridDim.x + blockIdx.x; w < pieces && ok; w += 2 * gridDim.x) {
      const int chunk = w / kEpPiecesPerChunk;
      const long long r0 = static_cast<long long>(chunk) * BM + (w - chunk * kEpPiecesPerChunk) * kEpPieceRows;
      int my_src = lane < kEpPieceRows ? p.row_src[r0 + lane] : -1;
      if (my_src >= 0 && ((my_src >> 24) >= p.world || (my_src & 0xFFFFFF) >= p.src_rows)) {
        record_error(p.status, kBadIndex);
        my_src = -1;
      }
      const unsigned int need = __reduce_or_sync(0xffffffffu, my_src >= 0 ? 1u << (my_src >> 24) : 0u) & ~seen;
      if (need) {
        bool good = true;
        if (lane == 0) {
          for (int s = 0; s < p.world && good; ++s)
            if (need & (1u << s)) {
              const unsigned long long* rd = sig(p, p.rank, kEpSigSendReady + s);
              good = wait_until([&] { return ld_acquire_sys(rd) >= static_cast<unsigned long long>(p.epoch); },
                                abort_flag, p.timeout_ns, p.status);
            }
        }
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          ok = false;
          break;
        }
        seen |= need;
      }
      // Two rows at a time, each with one source pointer for the whole warp (a shuffle per row,
      // not per word): every lane keeps 16 loads of 16 bytes in flight and spends a handful of
      // instructions per word, so the copy warps do not steal issue slots from the MMA pipeline.
      uint4* dst = reinterpret_cast<uint4*>(p.a_local) + r0 * wpr;
      constexpr int U = 8;
#pragma unroll 1
      for (int rr = 0; rr < kEpPieceRows; rr += 2) {
        const int s0 = __shfl_sync(0xffffffffu, my_src, rr), s1 = __shfl_sync(0xffffffffu, my_src, rr + 1);
        const uint4* a0 = s0 >= 0 ? reinterpret_cast<const uint4*>(p.src[s0 >> 24]) + static_cast<long long>(s0 & 0xFFFFFF) * wpr : nullptr;
        const uint4* a1 = s1 >= 0 ? reinterpret_cast<const uint4*>(p.src[s1 >> 24]) + static_cast<long long>(s1 & 0xFFFFFF) * wpr : nullptr;
        uint4* d0 = dst + rr * wpr;
        uint4* d1 = d0 + wpr;
#pragma unroll 1
        for (int c = lane; c < wpr; c += 32 * U) {
          uint4 b0[U], b1[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int cc = c + 32 * u;
            b0[u] = a0 != nullptr && cc < wpr ? __ldcg(a0 + cc) : make_uint4(0u, 0u, 0u, 0u);
            b1[u] = a1 != nullptr && cc < wpr ? __ldcg(a1 + cc) : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int cc = c + 32 * u;
            if (cc < wpr) {
              d0[cc] = b0[u];
              d1[cc] = b1[u];
            }
          }
        }
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(p.chunk_flags + chunk, 1u);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    // Done reading the sources' send buffers: the last copy warp of the grid tells every rank.
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
      const unsigned int prev = atomicAdd(p.block_counter, 1u);
      if (prev == 2 * gridDim.x - 1) {
        *p.block_counter = 0;  // reset for the next launch (stream-ordered)
        __threadfence_system();
        for (int q = 0; q < p.world; ++q) red_add_release_sys(sig(p, q, kEpSigSendDone), 1ull);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (!PULL && threadIdx.x == 0) {
    // All of this CTA's rows are stored: the last CTA of the grid tells every destination.
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.block_counter, 1u);
    if (prev == gridDim.x - 1) {
      *p.block_counter = 0;
      __threadfence_system();
      for (int q = 0; q < p.world; ++q) red_add_release_sys(sig(p, q, kEpSigRecvDone), 1ull);
    }
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, ECfg::kTmemCols);
  }
}

// out[t] = sum_j w[t, j] * recv[t * k + j] once every owner has stored its rows (fp32 sums).
__global__ void __launch_bounds__(256) ep_combine_kernel(const EpCombineParams p) {
  __shared__ int go;
  if (threadIdx.x == 0) {
    const unsigned long long* done = reinterpret_cast<const unsigned long long*>(p.signal[p.rank]) + kEpSigRecvDone;
    go = wait_until([&] { return ld_acquire_sys(done) >= p.done_target; }, nullptr, p.timeout_ns, p.status) ? 1 : 0;
  }
  __syncthreads();
  if (go) {
    const int wpr = p.cols / 8;
    const long long total = static_cast<long long>(p.tokens) * wpr;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long t = i / wpr;
      const int c = static_cast<int>(i - t * wpr);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < p.k; ++j) {
        const long long slot = t * p.k + j;
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.recv) + slot * wpr + c);
        if (p.keep != nullptr) reinterpret_cast<uint4*>(p.keep)[slot * wpr + c] = v;
        const float wt = p.weights != nullptr ? p.weights[slot] : 1.f;
        const uint32_t vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vs[q]));
          acc[2 * q] = fmaf(wt, f.x, acc[2 * q]);
          acc[2 * q + 1] = fmaf(wt, f.y, acc[2 * q + 1]);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(p.out)[t * wpr + c] = o;
    }
  }
  // The recv rows may be overwritten once every CTA here has read them: the last CTA frees them.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(p.block_counter, 1u);
    if (prev == gridDim.x - 1) {
      *p.block_counter = 0;
      __threadfence_system();
      for (int q = 0; q < p.world; ++q)
        red_add_release_sys(reinterpret_cast<unsigned long long*>(p.signal[q]) + kEpSigRecvFree, 1ull);
    }
  }
}

// out[t * k + j] = bf16(w[t, j] * dy[t]) and dw[t, j] = <dy[t], y[t * k + j]> (fp32); one warp per slot.
__global__ void __launch_bounds__(256) ep_expand_kernel(const __nv_bfloat16* __restrict__ dy,
                                                        const float* __restrict__ w, const __nv_bfloat16* __restrict__ y,
                                                        __nv_bfloat16* __restrict__ out, float* __restrict__ dw,
                                                        long long slots, int k, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wpr = cols / 8;
  for (long long s = blockIdx.x * 8LL + warp; s < slots; s += gridDim.x * 8LL) {
    const long long t = s / k;
    const float wt = w[s];
    const uint4* d4 = reinterpret_cast<const uint4*>(dy) + t * wpr;
    const uint4* y4 = reinterpret_cast<const uint4*>(y) + s * wpr;
    uint4* o4 = reinterpret_cast<uint4*>(out) + s * wpr;
    float dot = 0.f;
    for (int c = lane; c < wpr; c += 32) {
      const uint4 dv = d4[c], yv = y4[c];
      const uint32_t ds[4] = {dv.x, dv.y, dv.z, dv.w}, ys[4] = {yv.x, yv.y, yv.z, yv.w};
      uint32_t os[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ds[q]));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ys[q]));
        dot = fmaf(a.x, b.x, fmaf(a.y, b.y, dot));
        os[q] = pack_bf16x2(wt * a.x, wt * a.y);
      }
      o4[c] = make_uint4(os[0], os[1], os[2], os[3]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0 && dw != nullptr) dw[s] = dot;
  }
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <bool PULL, bool B_MN, int EPI>
void launch_ep(const CUtensorMap& ta, const CUtensorMap& tb, const EpGemmParams& p, cudaStream_t stream) {
  auto kern = ep_gemm_kernel<PULL, B_MN, EPI>;
  constexpr int smem = PULL ? kEpPullSmem : kEpPushSmem;
  static bool configured = false;
  if (!configured) {
    check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "ep gemm smem attribute");
    configured = true;
  }
  // Every CTA of the pull kernel must be resident (its copy warps feed the others' tiles);
  // the push kernel's CTA count is fixed too, because its last CTA signals completion.
  const int grid = device_sm_count();
  if (PULL) {
    void* args[] = {const_cast<CUtensorMap*>(&ta), const_cast<CUtensorMap*>(&tb), const_cast<EpGemmParams*>(&p)};
    check(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(256), args, smem, stream),
          "ep_pull_gemm cooperative launch");
  } else {
    kern<<<grid, 192, smem, stream>>>(ta, tb, p);
    check(cudaGetLastError(), "ep_push_gemm launch");
  }
}

void check_params(const EpGemmParams& p, long long rows) {
  if (p.experts < 1 || p.experts > kEpMaxExperts) throw std::invalid_argument("ep gemm: 1..512 experts per rank");
  if (rows % BM != 0) throw std::invalid_argument("ep gemm: row capacity must be a multiple of 128");
  if (p.K % 64 != 0 || p.N % 64 != 0) throw std::invalid_argument("ep gemm: K and N must be multiples of 64");
  if (p.world < 1 || p.world > kMaxRanks || p.rank < 0 || p.rank >= p.world) throw std::invalid_argument("ep gemm: rank/world");
}

}  // namespace

void ep_pull_gemm(const EpGemmParams& p, const void* B, long long ldb, bool b_mn, cudaStream_t stream) {
  check_params(p, p.M);
  const long long chunks = p.M / BM;
  check(cudaMemsetAsync(p.chunk_flags, 0, sizeof(unsigned int) * chunks, stream), "ep chunk flags reset");
  CUtensorMap ta, tb;
  make_tmap_2d_bf16(&ta, p.a_local, p.K, p.M, p.K, 64, BM);
  const long long b_total = static_cast<long long>(p.experts) * p.b_rows;
  if (p.epi == 3) {
    if (b_mn) throw std::invalid_argument("ep_pull_gemm epilogue 3 needs B K-major");
    make_tmap_2d_bf16(&tb, B, p.K, b_total, ldb, 64, 128);
    launch_ep<true, false, 3>(ta, tb, p, stream);
  } else if (p.epi == 4) {
    if (!b_mn) throw std::invalid_argument("ep_pull_gemm epilogue 4 needs B N-major");
    make_tmap_2d_bf16(&tb, B, p.N, b_total, ldb, 64, BK);
    launch_ep<true, true, 4>(ta, tb, p, stream);
  } else {
    throw std::invalid_argument("ep_pull_gemm: epilogue 3 (SwiGLU) or 4 (SwiGLU backward)");
  }
}

void ep_push_gemm(const EpGemmParams& p, const void* A, long long lda, const void* B, long long ldb, bool b_mn,
                  cudaStream_t stream) {
  check_params(p, p.M);
  if (p.N % 8 != 0) throw std::invalid_argument("ep_push_gemm: N % 8");
  CUtensorMap ta, tb;
  make_tmap_2d_bf16(&ta, A, p.K, p.M, lda, 64, BM);
  const long long b_total = static_cast<long long>(p.experts) * p.b_rows;
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, p.N, b_total, ldb, 64, BK);
    launch_ep<false, true, 0>(ta, tb, p, stream);
  } else {
    make_tmap_2d_bf16(&tb, B, p.K, b_total, ldb, 64, EBN);
    launch_ep<false, false, 0>(ta, tb, p, stream);
  }
}

void ep_combine(const EpCombineParams& p, cudaStream_t stream) {
  if (p.cols % 8 != 0) throw std::invalid_argument("ep_combine: channels must be a multiple of 8");
  ep_combine_kernel<<<2 * device_sm_count(), 256, 0, stream>>>(p);
  check(cudaGetLastError(), "ep_combine launch");
}

void ep_expand(const void* dy, const float* w, const void* y, void* out, float* dw, long long slots, int k, int cols,
               cudaStream_t stream) {
  if (cols % 8 != 0) throw std::invalid_argument("ep_expand: channels must be a multiple of 8");
  long long blocks = (slots + 7) / 8;
  const long long cap = 4LL * device_sm_count();
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  ep_expand_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), w, static_cast<const __nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(out),
      dw, slots, k, cols);
  check(cudaGetLastError(), "ep_expand launch");
}

}  // namespace pb

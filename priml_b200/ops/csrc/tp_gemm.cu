// Tensor-parallel GEMMs fused with their collectives (sequence-parallel Megatron
// layout: activations sharded by rows, i.e. tokens, across the TP ranks).
//
//   tp_ag_gemm   C[M, N] = AllGather_rows(A_shard) @ B^T
//     One cooperative launch (every CTA resident). Besides the TMA producer,
//     the MMA issuer and four epilogue warps, each CTA runs two copy warps.
//     The peers' shards are cut into 16-row pieces (contiguous bytes); the
//     copy warps of all CTAs pull them over NVLink (16-byte peer loads, 16 in
//     flight per lane) into a local gather buffer in consumption order and
//     count each finished piece on its 128-row chunk (then copy this rank's
//     own rows, so the gathered buffer is complete for the weight gradient). Tiles are visited own
//     shard first, then the peers' shards in copy order; the producer loads
//     a peer tile only once its chunk is complete (bounded wait), so the copy
//     overlaps the GEMM tile by tile. A rank announces its shard on every
//     peer at kernel start, and the copy warps finish by counting themselves
//     on every source rank, which may then overwrite its shard buffer.
//   tp_gemm_rs   C_shard = ReduceScatter_rows(A @ B^T)
//     The epilogue stages each 64-column slice of its partial rows in shared
//     memory and every lane bulk-stores its row (128 contiguous bytes) into
//     the owner rank's receive slot for this rank over NVLink; each CTA then
//     counts itself on every rank. tp_rs_reduce waits for all ranks' stores
//     and sums the slots in rank order (fp32), then frees the slots for the
//     next call with a counter on every peer.
// B is K-major ([N, K]) or N-major ([K, N]); A is K-major. Every cross-rank
// wait is bounded by globaltimer and reports kTimeoutPeer.
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int TBM = 128, TBN = 256, TBK = 64, TSTAGES = 4;
constexpr int kTpABytes = TBM * TBK * 2, kTpBBytes = TBN * TBK * 2, kTpStage = kTpABytes + kTpBBytes;
constexpr int kOutCols = 64;                         // columns per staged epilogue slice
constexpr int kOutPitch = kOutCols * 2 + 16;         // padded row pitch of the staging buffer (bytes)
constexpr int kOutWarpBytes = 32 * kOutPitch;        // one epilogue warp's 32 rows
constexpr int kPieceRows = 16;                       // rows per all-gather copy piece
constexpr int kPiecesPerChunk = TBM / kPieceRows;
constexpr int kTpSmem = TSTAGES * kTpStage + 1024 + 256 + 4 * kOutWarpBytes;

__device__ __forceinline__ void red_add_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename F>
__device__ bool bounded_until(F ready, long long timeout_ns, int* status) {
  const unsigned long long t0 = globaltimer();
  while (!ready()) {
    if (static_cast<long long>(globaltimer() - t0) > timeout_ns) {
      record_error(status, kTimeoutPeer);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Virtual m-block vm -> real m-block: own shard first, then rank+1, rank+2, ...
__device__ __forceinline__ int real_mblock(int vm, int bps, int rank, int world) {
  const int s = (rank + vm / bps) % world;
  return s * bps + vm % bps;
}

template <bool B_MN, int MODE>  // MODE 0 = all-gather -> GEMM, 1 = GEMM -> reduce-scatter
__global__ void __launch_bounds__(MODE == 0 ? 256 : 192, 1)
    tp_gemm_kernel(const __grid_constant__ CUtensorMap tmA_own, const __grid_constant__ CUtensorMap tmA_full,
                   const __grid_constant__ CUtensorMap tmB, const TpGemmParams p) {
  constexpr int S = TSTAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + S * kTpABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kTpStage);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* stage_out = smem + S * kTpStage + 256;  // [4 warps][32 rows][kOutPitch]

  const int warp = warp_id(), lane = lane_id();
  const int bps = p.m_shard / TBM;               // 128-row blocks per shard
  const int num_m = bps * p.world;
  const int num_n = (p.N + TBN - 1) / TBN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + TBK - 1) / TBK;

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
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
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
      // n fastest within groups of 16 virtual m-blocks (L2 reuse of B)
      const int group = 16 * num_n;
      const int g = tile / group, first = g * 16, gm = min(num_m - first, 16), r = tile - g * group;
      const int vm = first + r % gm, nb = r / gm;
      const int mb = real_mblock(vm, bps, p.rank, p.world);
      const bool own = MODE == 1 || vm < bps;
      if (MODE == 0 && !own) {
        const unsigned int* flag = p.chunk_flags + (vm - bps);  // pieces copied (reset before the launch)
        if (!bounded_until([&] { return ld_acquire_gpu_u32(flag) >= static_cast<unsigned int>(kPiecesPerChunk) ||
                                        *abort_flag; },
                           p.timeout_ns, p.status) || *abort_flag) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        // the chunk was written by generic stores of other CTAs; the TMA (async proxy) reads it next
        asm volatile("fence.proxy.async.global;" ::: "memory");
      }
      const int n0 = nb * TBN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], kTpStage);
        uint8_t* a_dst = smA + stage * kTpABytes;
        uint8_t* b_dst = smB + stage * kTpBBytes;
        const int k0 = kb * TBK;
        if (MODE == 0 && own) {
          tma_load_2d(a_dst, &tmA_own, &full[stage], k0, (mb - p.rank * bps) * TBM);
        } else {
          tma_load_2d(a_dst, &tmA_full, &full[stage], k0, mb * TBM);
        }
        if constexpr (B_MN) {
#pragma unroll
          for (int j = 0; j < TBN / 64; ++j) tma_load_2d(b_dst + j * (TBK * 128), &tmB, &full[stage], n0 + 64 * j, k0);
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
    constexpr uint32_t idesc = make_idesc_bf16(TBM, TBN, false, B_MN);
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
      const uint32_t d_tmem = tmem_base + b * TBN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smA + stage * kTpABytes);
        const uint32_t b_base = smem_u32(smB + stage * kTpBBytes);
#pragma unroll
        for (int kk = 0; kk < TBK / 16; ++kk) {
          const uint64_t ad = make_sw128_desc(a_base + kk * 32, 16, 1024);
          const uint64_t bd = B_MN ? make_sw128_desc(b_base + kk * 2048, TBK * 128, 1024)
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
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    int local = 0;
    if (MODE == 1 && p.epoch > 1) {
      // the owners must have reduced the previous call's slots before they are overwritten
      const unsigned long long target = static_cast<unsigned long long>(p.epoch - 1) * p.world * p.reduce_grid;
      const unsigned long long* freed = reinterpret_cast<const unsigned long long*>(p.signal[p.rank]) + kTpSigRsFree;
      if (!bounded_until([&] { return ld_acquire_sys_u64(freed) >= target || *abort_flag; }, p.timeout_ns,
                         p.status))
        *abort_flag = 1;
    }
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int group = 16 * num_n;
      const int g = tile / group, first = g * 16, gm = min(num_m - first, 16), r = tile - g * group;
      const int vm = first + r % gm, nb = r / gm;
      const int mb = real_mblock(vm, bps, p.rank, p.world);
      const int b = local & 1;
      if (!mbar_wait_warp(&tfull[b], (local >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int row = mb * TBM + wq * 32 + lane;  // < M always (M = world * m_shard, m_shard % 128 == 0)
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16) + b * TBN;
      if constexpr (MODE == 0) {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.C) + static_cast<long long>(row) * p.ldc;
#pragma unroll 1
        for (int c = 0; c < TBN; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c, v);
          tmem_wait_ld();
          const int col = nb * TBN + c;
          if (col >= p.N || *abort_flag) continue;
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          if (col + 32 <= p.N) {
            uint4* o4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
            for (int q = 0; q < 4; ++q) o4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          } else {
            const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(pk);
            for (int j = 0; j < 32 && col + j < p.N; ++j) dst[col + j] = hb[j];
          }
        }
      } else {
        // Partial row -> the owner's slot for this rank: stage 64 columns, then one
        // 128-byte bulk store per lane (each lane only touches its own staged row).
        const int owner = row / p.m_shard, lr = row - owner * p.m_shard;
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.slots[owner]) +
                             (static_cast<long long>(p.rank) * p.m_shard + lr) * p.N;
        uint8_t* my_row = stage_out + wq * kOutWarpBytes + lane * kOutPitch;
#pragma unroll 1
        for (int c = 0; c < TBN; c += kOutCols) {
          uint32_t v[64];
          tmem_ld_32x32b_x32(t_row + c, *reinterpret_cast<uint32_t(*)[32]>(v));
          tmem_ld_32x32b_x32(t_row + c + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          tmem_wait_ld();
          const int col = nb * TBN + c;
          if (col >= p.N || *abort_flag) continue;
          tma_store_wait_read();  // the previous slice has left the staging row
          uint4* s4 = reinterpret_cast<uint4*>(my_row);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            s4[q] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * q]), __uint_as_float(v[8 * q + 1])),
                               pack_bf16x2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3])),
                               pack_bf16x2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5])),
                               pack_bf16x2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7])));
          fence_proxy_async_smem();
          bulk_store(dst + col, my_row, static_cast<uint32_t>(min(kOutCols, p.N - col)) * 2u);  // N % 8 == 0
          tma_store_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (MODE == 1) {
      // this thread's bulk stores are complete, then ordered before the CTA counts itself done
      tma_store_wait_all();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
    }
  } else if (MODE == 0 && warp >= 6) {
    // ------------------------------------------------------------ copy warps (all-gather)
    const int cw = warp - 6;
    const int pieces = (p.world - 1) * bps * kPiecesPerChunk;  // in consumption order: chunk j, piece q
    const long long piece_u4 = static_cast<long long>(kPieceRows) * p.K / 8;  // 16-byte words per piece
    if (blockIdx.x == 0 && cw == 0 && lane == 0) {
      // This rank's shard for this epoch is in place (stream order): tell every peer.
      __threadfence_system();
      for (int q = 0; q < p.world; ++q)
        st_release_sys_u64(reinterpret_cast<unsigned long long*>(p.signal[q]) + kTpSigAgReady + p.rank,
                           static_cast<unsigned long long>(p.epoch));
    }
    const unsigned long long* ready = reinterpret_cast<const unsigned long long*>(p.signal[p.rank]) + kTpSigAgReady;
    int ready_rank = p.rank;  // the source whose announcement this warp has already seen (own shard: in place)
    // Pieces [0, pieces) come from the peers and gate GEMM tiles; the last bps * kPiecesPerChunk
    // fill in this rank's own rows of the gathered output (read by the caller, not by the GEMM).
    const int total = pieces + bps * kPiecesPerChunk;
    for (int w = cw * gridDim.x + blockIdx.x; w < total; w += 2 * gridDim.x) {
      const bool own = w >= pieces;
      const int j = own ? -1 : w / kPiecesPerChunk;
      const int piece = own ? (w - pieces) % kPiecesPerChunk : w - j * kPiecesPerChunk;
      const int mb = own ? p.rank * bps + (w - pieces) / kPiecesPerChunk : real_mblock(bps + j, bps, p.rank, p.world);
      const int src_rank = mb / bps;
      if (src_rank != ready_rank) {
        bool ok = true;
        if (lane == 0)
          ok = bounded_until([&] { return ld_acquire_sys_u64(ready + src_rank) >= static_cast<unsigned long long>(p.epoch) ||
                                          *abort_flag; },
                             p.timeout_ns, p.status) && !*abort_flag;
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          *abort_flag = 1;
          break;
        }
        ready_rank = src_rank;
      }
      const long long row0 = static_cast<long long>(mb - src_rank * bps) * TBM + piece * kPieceRows;
      const uint4* src = reinterpret_cast<const uint4*>(p.peer_a[src_rank]) + row0 * (p.K / 8);
      uint4* dst = reinterpret_cast<uint4*>(p.a_full) + (static_cast<long long>(mb) * TBM + piece * kPieceRows) * (p.K / 8);
      constexpr int U = 16;
      for (long long base = lane; base < piece_u4; base += 32 * U) {
        uint4 buf[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (base + 32 * u < piece_u4) buf[u] = __ldcg(src + base + 32 * u);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (base + 32 * u < piece_u4) dst[base + 32 * u] = buf[u];
      }
      if (own) continue;
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(p.chunk_flags + j, 1u);
    }
    // Done reading the peers' shards for this epoch: tell every rank.
    __threadfence_system();
    __syncwarp();
    if (lane == 0)
      for (int q = 0; q < p.world; ++q)
        if (q != p.rank) red_add_release_sys_u64(reinterpret_cast<unsigned long long*>(p.signal[q]) + kTpSigAgDone, 1ull);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (MODE == 1 && threadIdx.x == 0) {
    // All of this CTA's partial rows are stored: count it on every rank.
    __threadfence_system();
    for (int q = 0; q < p.world; ++q)
      red_add_release_sys_u64(reinterpret_cast<unsigned long long*>(p.signal[q]) + kTpSigRsDone, 1ull);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, 512);
  }
}

// C_shard[lr, :] = sum_s slots[s][lr, :] once every rank's GEMM has stored its partials.
__global__ void __launch_bounds__(256) tp_rs_reduce_kernel(const TpGemmParams p, __nv_bfloat16* __restrict__ out,
                                                            long long ldo, unsigned long long target) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned long long* done = reinterpret_cast<const unsigned long long*>(p.signal[p.rank]) + kTpSigRsDone;
    ok = bounded_until([&] { return ld_acquire_sys_u64(done) >= target; }, p.timeout_ns, p.status) ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    const __nv_bfloat16* slots = reinterpret_cast<const __nv_bfloat16*>(p.slots[p.rank]);
    const long long per = static_cast<long long>(p.m_shard) * p.N;
    const long long n8 = per / 8;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const long long e = i * 8;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s = 0; s < p.world; ++s) {
        const uint4 w = __ldcg(reinterpret_cast<const uint4*>(slots + s * per + e));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[q]));
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      const long long lr = e / p.N, col = e % p.N;
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(out + lr * ldo + col) = o;
    }
  }
  // The slots may be overwritten by the next call once every CTA here has read them.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q)
      red_add_release_sys_u64(reinterpret_cast<unsigned long long*>(p.signal[q]) + kTpSigRsFree, 1ull);
  }
}

// Before this rank overwrites its A shard: every peer's copy warps are done with the last epoch.
__global__ void tp_wait_kernel(const unsigned long long* counter, unsigned long long target, long long timeout_ns,
                               int* status) {
  if (threadIdx.x == 0) bounded_until([&] { return ld_acquire_sys_u64(counter) >= target; }, timeout_ns, status);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <bool B_MN, int MODE>
void launch_tp(const CUtensorMap& a_own, const CUtensorMap& a_full, const CUtensorMap& b, const TpGemmParams& p,
               int grid, cudaStream_t stream) {
  auto kern = tp_gemm_kernel<B_MN, MODE>;
  static bool configured = false;
  if (!configured) {
    check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTpSmem), "tp smem attribute");
    configured = true;
  }
  const int threads = MODE == 0 ? 256 : 192;
  if (MODE == 0) {
    // Chunks copied by one CTA are consumed by others: every CTA must be resident.
    void* args[] = {const_cast<CUtensorMap*>(&a_own), const_cast<CUtensorMap*>(&a_full), const_cast<CUtensorMap*>(&b),
                    const_cast<TpGemmParams*>(&p)};
    check(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kern), dim3(grid), dim3(threads), args, kTpSmem,
                                      stream),
          "tp_ag_gemm cooperative launch");
  } else {
    kern<<<grid, threads, kTpSmem, stream>>>(a_own, a_full, b, p);
    check(cudaGetLastError(), "tp_gemm_rs launch");
  }
}

}  // namespace

int tp_gemm_grid(int M, int N) {
  const int tiles = (M / TBM) * ((N + TBN - 1) / TBN);
  const int sms = device_sm_count();
  return tiles < sms ? tiles : sms;
}

void tp_ag_gemm(const TpGemmParams& p, const void* a_shard, const void* B, long long ldb, bool b_mn, int grid,
                cudaStream_t stream) {
  if (p.m_shard % TBM != 0 || p.K % 8 != 0) throw std::invalid_argument("tp_ag_gemm: m_shard % 128 and K % 8");
  const int chunks = (p.world - 1) * (p.m_shard / TBM);
  if (chunks > 0) check(cudaMemsetAsync(p.chunk_flags, 0, sizeof(unsigned int) * chunks, stream), "tp chunk flags reset");
  const long long M = static_cast<long long>(p.m_shard) * p.world;
  CUtensorMap a_own, a_full, tb;
  make_tmap_2d_bf16(&a_own, a_shard, p.K, p.m_shard, p.K, 64, TBM);
  make_tmap_2d_bf16(&a_full, p.a_full, p.K, M, p.K, 64, TBM);
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, p.N, p.K, ldb, 64, TBK);
    launch_tp<true, 0>(a_own, a_full, tb, p, grid, stream);
  } else {
    make_tmap_2d_bf16(&tb, B, p.K, p.N, ldb, 64, TBN);
    launch_tp<false, 0>(a_own, a_full, tb, p, grid, stream);
  }
}

void tp_gemm_rs(const TpGemmParams& p, const void* A, long long lda, const void* B, long long ldb, bool b_mn, void* out,
                long long ldo, int grid, int reduce_grid, unsigned long long done_target, cudaStream_t stream) {
  if (p.m_shard % TBM != 0 || p.N % 8 != 0) throw std::invalid_argument("tp_gemm_rs: m_shard % 128 and N % 8");
  const long long M = static_cast<long long>(p.m_shard) * p.world;
  CUtensorMap ta, tb;
  make_tmap_2d_bf16(&ta, A, p.K, M, lda, 64, TBM);
  if (b_mn) {
    make_tmap_2d_bf16(&tb, B, p.N, p.K, ldb, 64, TBK);
    launch_tp<true, 1>(ta, ta, tb, p, grid, stream);
  } else {
    make_tmap_2d_bf16(&tb, B, p.K, p.N, ldb, 64, TBN);
    launch_tp<false, 1>(ta, ta, tb, p, grid, stream);
  }
  tp_rs_reduce_kernel<<<reduce_grid, 256, 0, stream>>>(p, static_cast<__nv_bfloat16*>(out), ldo, done_target);
  check(cudaGetLastError(), "tp_rs_reduce launch");
}

void tp_wait(const void* signal_local, int word, unsigned long long target, long long timeout_ns, int* status,
             cudaStream_t stream) {
  tp_wait_kernel<<<1, 32, 0, stream>>>(static_cast<const unsigned long long*>(signal_local) + word, target, timeout_ns,
                                       status);
  check(cudaGetLastError(), "tp_wait launch");
}

}  // namespace pb

// Expert-parallel token exchange over NVLink peer memory.
//
// Every rank owns a few experts and a symmetric receive buffer per direction
// (rows of `C` bf16 channels plus one int32 of metadata per row). A transfer
// writes rows straight into the destination rank's buffer at rows computed on
// the device (the dispatch plan lays out 128-aligned per-expert segments), so
// no host learns how many rows go where.
//
//   ep_scatter   row i of `src` (or src[gather[i]]) -> buffer of rank
//                dest_rank[i] at row dest_row[i] (16-byte peer stores, one warp
//                per row), optional metadata word. Before writing epoch e the
//                CTAs wait (bounded) until every rank has consumed epoch e-1 of
//                that buffer; the last CTA to finish counts this rank as done on
//                every destination.
//   ep_collect   after the owner has seen all ranks done (tp_wait on the done
//                counter): copy the first `bound` rows (a device value) of its
//                own buffer into a private tensor, zeroing segment padding and
//                writing -1 metadata for it.
//   ep_signal    count this rank on a signal word of every rank (buffer freed).
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace {

__device__ __forceinline__ void red_add_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool wait_at_least(const unsigned long long* word, unsigned long long target, long long timeout_ns,
                              int* status) {
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(word) < target) {
    if (static_cast<long long>(globaltimer() - t0) > timeout_ns) {
      record_error(status, kTimeoutPeer);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

__global__ void __launch_bounds__(256) ep_scatter_kernel(const EpScatterParams p) {
  __shared__ int go;
  if (threadIdx.x == 0) {
    const unsigned long long* freed = reinterpret_cast<const unsigned long long*>(p.signal[p.rank]) + p.free_word;
    go = wait_at_least(freed, static_cast<unsigned long long>(p.epoch - 1) * p.world, p.timeout_ns, p.status) ? 1 : 0;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int words = p.cols / 8;  // 16-byte words per row
  if (go) {
    for (long long i = static_cast<long long>(blockIdx.x) * 8 + warp; i < p.rows; i += static_cast<long long>(gridDim.x) * 8) {
      const int dr = p.dest_rank[i];
      if (dr < 0) continue;
      const long long srow = p.gather != nullptr ? p.gather[i] : i;
      const long long drow = p.dest_row[i];
      if (dr >= p.world || drow < 0 || drow >= p.dest_cap) {  // never write outside a peer's buffer
        if (lane == 0) record_error(p.status, kBadIndex);
        continue;
      }
      const uint4* s = reinterpret_cast<const uint4*>(p.src + srow * p.ld_src);
      uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.buf[dr]) + drow * p.cols);
      for (int w = lane; w < words; w += 32) d[w] = __ldg(s + w);
      if (p.meta != nullptr && lane == 0) reinterpret_cast<int*>(p.meta_buf[dr])[drow] = p.meta[i];
    }
  }
  // Count this CTA; the last one publishes "this rank is done" on every destination.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(p.block_counter, 1u);
    if (prev == gridDim.x - 1) {
      *p.block_counter = 0;  // reset for the next launch (stream-ordered)
      __threadfence_system();
      for (int q = 0; q < p.world; ++q)
        red_add_release_sys(reinterpret_cast<unsigned long long*>(p.signal[q]) + p.done_word, 1ull);
    }
  }
}

// dst[r] = pad(r) ? 0 : buf[r] for r < bound = seg_start[segs]; meta likewise (-1 for padding).
__global__ void __launch_bounds__(256) ep_collect_kernel(const __nv_bfloat16* __restrict__ buf, const int* __restrict__ meta,
                                                         __nv_bfloat16* __restrict__ dst, int* __restrict__ meta_dst,
                                                         const int* __restrict__ seg_start, const int* __restrict__ totals,
                                                         int segs, int cols, long long cap) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long bound = seg_start[segs];
  const int words = cols / 8;
  for (long long r = static_cast<long long>(blockIdx.x) * 8 + warp; r < bound && r < cap;
       r += static_cast<long long>(gridDim.x) * 8) {
    int lo = 0, hi = segs;  // segment of row r: largest s with seg_start[s] <= r
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (seg_start[mid] <= r) lo = mid; else hi = mid;
    }
    const bool pad = r - seg_start[lo] >= totals[lo];
    uint4* d = reinterpret_cast<uint4*>(dst + r * cols);
    const uint4* s = reinterpret_cast<const uint4*>(buf + r * cols);
    for (int w = lane; w < words; w += 32) d[w] = pad ? make_uint4(0u, 0u, 0u, 0u) : __ldcg(s + w);
    if (meta_dst != nullptr && lane == 0) meta_dst[r] = pad ? -1 : __ldcg(meta + r);
  }
}

__global__ void ep_signal_kernel(EpSignalParams p) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.world; ++q)
      red_add_release_sys(reinterpret_cast<unsigned long long*>(p.signal[q]) + p.word, 1ull);
  }
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

void ep_scatter(const EpScatterParams& p, cudaStream_t stream) {
  if (p.cols % 8 != 0) throw std::invalid_argument("ep_scatter: channels must be a multiple of 8");
  long long blocks = (p.rows + 7) / 8;
  const long long cap = 4LL * device_sm_count();
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  ep_scatter_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(p);
  check(cudaGetLastError(), "ep_scatter launch");
}

void ep_collect(const void* buf, const int* meta, void* dst, int* meta_dst, const int* seg_start, const int* totals,
                int segs, int cols, long long cap, cudaStream_t stream) {
  if (cols % 8 != 0) throw std::invalid_argument("ep_collect: channels must be a multiple of 8");
  const int blocks = 4 * device_sm_count();
  ep_collect_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(buf), meta,
                                                static_cast<__nv_bfloat16*>(dst), meta_dst, seg_start, totals, segs,
                                                cols, cap);
  check(cudaGetLastError(), "ep_collect launch");
}

void ep_signal(const EpSignalParams& p, cudaStream_t stream) {
  ep_signal_kernel<<<1, 32, 0, stream>>>(p);
  check(cudaGetLastError(), "ep_signal launch");
}

}  // namespace pb

// Collectives fused with the optimizer step, over NVLink peer memory.
//
// Sharded data parallelism with resident bf16 weights (the FSDP train step of
// `priml/train/parallelism.py` with an AdamW step, re-planned for 180 GB GPUs):
// every rank keeps the full bf16 weight copy and a full fp32 gradient buffer,
// both allocated with cudaMalloc and mapped into every peer by CUDA IPC; the
// fp32 master weights and Adam moments are sharded 1/R per rank.
//
//   rs_bucket_kernel       reduce-scatter of one gradient bucket: rank r sums
//                          slice r of the bucket over all R ranks' buffers
//                          (P2P loads, fixed rank order -> bitwise identical
//                          on every run), scales, writes its fp32 shard and
//                          per-CTA sums of squares. Launched on a side stream
//                          as soon as the bucket's gradients exist, so it
//                          overlaps the rest of the backward pass.
//   norm_exchange_kernel   global gradient norm: each rank publishes its sum of
//                          squares to every peer, sums the R values in rank
//                          order, and derives the clip coefficient on device.
//   adamw_scatter_kernel   clip + AdamW on the local shard, then the bf16 cast
//                          of the new weights stored straight into every rank's
//                          weight copy (P2P stores) -- the parameter all-gather
//                          happens inside the optimizer kernel.
//   peer_barrier_kernel    waits until every peer's scatter has landed here.
//   gather_shards          (sharded-weights mode) copies one bucket's bf16
//                          weight shards from every rank into a local window
//                          with one peer cudaMemcpyAsync per rank, i.e. on the
//                          copy engines, so the gather of the next block runs
//                          beside the current block's kernels without taking SMs.
//
// In the sharded-weights mode each rank keeps only its own bf16 shard; the
// optimizer kernel then stores the new weights into that shard alone
// (`local_only`), and the forward / backward gather each block ahead of use.
//
// Synchronization uses a small signal array per rank (also IPC-mapped):
// monotone epoch flags written with st.release.sys and read with
// ld.acquire.sys. Every wait is bounded by globaltimer; a wait that runs out
// records kTimeoutPeer in the status word and the kernel returns. Peer memory
// is read and written only with plain 16-byte global loads and stores.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace pb {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_add_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin until *flag >= target; false (after recording kTimeoutPeer) when the
// bound runs out first.
__device__ bool wait_flag_ge(const unsigned long long* flag, unsigned long long target, long long timeout_ns,
                             int* status) {
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(flag) < target) {
    if (static_cast<long long>(globaltimer() - t0) > timeout_ns) {
      record_error(status, kTimeoutPeer);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = 0.f;
  if (warp == 0) {
    r = lane < static_cast<int>(blockDim.x >> 5) ? scratch[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  }
  return r;  // valid in thread 0
}

__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  // torch.lerp: a + w (b - a) for w < 0.5, else b - (b - a)(1 - w)
  return w < 0.5f ? fmaf(w, b - a, a) : b - (b - a) * (1.f - w);
}

// W = world size (compile-time, so the peer loads are fully unrolled); each
// thread keeps U float4 chunks x W peers (16) independent 16-byte loads in flight:
// 48 CTAs then hold about 3 MB of reads in flight, the bandwidth-delay product of
// a peer link at ~1-2 us round trip.
template <int W>
__global__ void __launch_bounds__(256, 2) rs_bucket_kernel(PeerTable t, int rank, int bucket, long long bucket_off,
                                                         long long shard, float* __restrict__ out,
                                                         float* __restrict__ partial, unsigned long long epoch,
                                                         float scale, long long timeout_ns, int* status) {
  constexpr int U = W >= 16 ? 1 : 16 / W;
  __shared__ int ok;
  __shared__ float red[32];
  if (threadIdx.x == 0) {
    // This rank's gradients for the bucket are complete (stream order): say so
    // to every peer, then wait until every peer has said the same.
    __threadfence_system();
    for (int p = 0; p < W; ++p) {
      auto* sig = reinterpret_cast<unsigned long long*>(t.signal[p]);
      st_release_sys(sig + kSigReady + bucket * kMaxRanks + rank, epoch);
    }
    auto* mine = reinterpret_cast<const unsigned long long*>(t.signal[rank]);
    int good = 1;
    for (int p = 0; p < W && good; ++p)
      good = wait_flag_ge(mine + kSigReady + bucket * kMaxRanks + p, epoch, timeout_ns, status) ? 1 : 0;
    ok = good;
  }
  __syncthreads();
  float acc = 0.f;
  if (ok) {
    const long long base = bucket_off + static_cast<long long>(rank) * shard;
    const long long n4 = shard >> 2;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const float4* src[W];
#pragma unroll
    for (int p = 0; p < W; ++p) src[p] = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(t.grad[p]) + base);
    for (long long c0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c0 < n4; c0 += U * stride) {
      float4 v[U][W];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long c = c0 + u * stride;
        if (c < n4) {
#pragma unroll
          for (int p = 0; p < W; ++p) v[u][p] = __ldcg(src[p] + c);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long c = c0 + u * stride;
        if (c < n4) {
          float4 s = v[u][0];
#pragma unroll
          for (int p = 1; p < W; ++p) {
            s.x += v[u][p].x;
            s.y += v[u][p].y;
            s.z += v[u][p].z;
            s.w += v[u][p].w;
          }
          s.x *= scale;
          s.y *= scale;
          s.z *= scale;
          s.w *= scale;
          reinterpret_cast<float4*>(out)[c] = s;
          acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
        }
      }
    }
  }
  const float tot = block_sum(acc, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(256) norm_exchange_kernel(PeerTable t, int rank, int world,
                                                             const float* __restrict__ partial, int n_partial,
                                                             unsigned long long epoch, float max_norm,
                                                             float* __restrict__ norm_out, float* __restrict__ clip_out,
                                                             long long timeout_ns, int* status) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n_partial; i += blockDim.x) acc += partial[i];
  const float local = block_sum(acc, red);
  if (threadIdx.x != 0) return;
  const unsigned long long tag = (epoch & 0xffffffffull) << 32;
  const int slot = kSigNorm + static_cast<int>(epoch & 1ull) * kMaxRanks;
  const unsigned long long word = tag | __float_as_uint(local);
  for (int p = 0; p < world; ++p)
    st_release_sys(reinterpret_cast<unsigned long long*>(t.signal[p]) + slot + rank, word);
  auto* mine = reinterpret_cast<const unsigned long long*>(t.signal[rank]);
  float total = 0.f;
  bool good = true;
  const unsigned long long t0 = globaltimer();
  for (int p = 0; p < world && good; ++p) {
    unsigned long long w;
    while (((w = ld_acquire_sys(mine + slot + p)) & 0xffffffff00000000ull) != tag) {
      if (static_cast<long long>(globaltimer() - t0) > timeout_ns) {
        record_error(status, kTimeoutPeer);
        good = false;
        break;
      }
      __nanosleep(64);
    }
    if (good) total += __uint_as_float(static_cast<unsigned int>(w & 0xffffffffull));
  }
  const float norm = good ? sqrtf(total) : __int_as_float(0x7fc00000);
  norm_out[0] = norm;
  clip_out[0] = (good && max_norm > 0.f) ? fminf(1.f, max_norm / (norm + 1e-6f)) : (good ? 1.f : 0.f);
}

__global__ void __launch_bounds__(256) adamw_scatter_kernel(PeerTable t, int world, int local_rank,
                                                             const ShardSegment* __restrict__ segs,
                                                             int nseg, long long n_local, float* __restrict__ master,
                                                             float* __restrict__ m1, float* __restrict__ m2,
                                                             const float* __restrict__ grad,
                                                             const float* __restrict__ clip, AdamHyper hp) {
  const float gs = clip != nullptr ? clip[0] : 1.f;
  const long long n8 = n_local >> 3;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  int s = 0;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < n8; c += stride) {
    const long long e = c << 3;
    while (s + 1 < nseg && segs[s + 1].local_off <= e) ++s;
    const ShardSegment seg = segs[s];
    const int g = seg.group;
    const float lr = hp.lr[g], b1 = hp.beta1[g], b2 = hp.beta2[g], eps = hp.eps[g];
    const float decay = 1.f - lr * hp.wd[g];
    const float step_size = lr / hp.bias1[g];
    const float bias2 = hp.bias2[g];
    float p[8], mm[8], vv[8], gg[8];
    *reinterpret_cast<float4*>(p) = reinterpret_cast<const float4*>(master + e)[0];
    *reinterpret_cast<float4*>(p + 4) = reinterpret_cast<const float4*>(master + e)[1];
    *reinterpret_cast<float4*>(mm) = reinterpret_cast<const float4*>(m1 + e)[0];
    *reinterpret_cast<float4*>(mm + 4) = reinterpret_cast<const float4*>(m1 + e)[1];
    *reinterpret_cast<float4*>(vv) = reinterpret_cast<const float4*>(m2 + e)[0];
    *reinterpret_cast<float4*>(vv + 4) = reinterpret_cast<const float4*>(m2 + e)[1];
    *reinterpret_cast<float4*>(gg) = __ldcs(reinterpret_cast<const float4*>(grad + e));
    *reinterpret_cast<float4*>(gg + 4) = __ldcs(reinterpret_cast<const float4*>(grad + e) + 1);
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gj = gg[j] * gs;
      float pj = p[j] * decay;
      const float mj = lerp_t(mm[j], gj, 1.f - b1);
      const float vj = lerp_t(vv[j], gj * gj, 1.f - b2);
      pj -= mj / (sqrtf(vj / bias2) + eps) * step_size;
      p[j] = pj;
      mm[j] = mj;
      vv[j] = vj;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(p[2 * j], p[2 * j + 1]);
      packed[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    reinterpret_cast<float4*>(master + e)[0] = *reinterpret_cast<float4*>(p);
    reinterpret_cast<float4*>(master + e)[1] = *reinterpret_cast<float4*>(p + 4);
    reinterpret_cast<float4*>(m1 + e)[0] = *reinterpret_cast<float4*>(mm);
    reinterpret_cast<float4*>(m1 + e)[1] = *reinterpret_cast<float4*>(mm + 4);
    reinterpret_cast<float4*>(m2 + e)[0] = *reinterpret_cast<float4*>(vv);
    reinterpret_cast<float4*>(m2 + e)[1] = *reinterpret_cast<float4*>(vv + 4);
    const long long dst = seg.gathered_off + (e - seg.local_off);
    const uint4 val = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if (local_rank >= 0) {  // sharded weights: this rank's shard only
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(t.param[local_rank]) + dst)[0] = val;
    } else {
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)
        if (q < world) reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(t.param[q]) + dst)[0] = val;
    }
  }
  // Publish: this CTA's stores are visible system-wide, then count it on every peer.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int q = 0; q < world; ++q)
      red_add_release_sys(reinterpret_cast<unsigned long long*>(t.signal[q]) + kSigDone, 1ull);
}

__global__ void peer_barrier_kernel(const unsigned long long* __restrict__ done, unsigned long long target,
                                    long long timeout_ns, int* status) {
  if (threadIdx.x == 0) wait_flag_ge(done, target, timeout_ns, status);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

// ------------------------------------------------------------------ host side
void* sym_alloc(size_t bytes) {
  void* p = nullptr;
  check(cudaMalloc(&p, bytes), "cudaMalloc (peer-shared buffer)");
  check(cudaMemset(p, 0, bytes), "cudaMemset (peer-shared buffer)");
  return p;
}

void sym_free(void* p) {
  if (p != nullptr) cudaFree(p);
}

void ipc_handle(void* p, char out[64]) {
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(out, &h, 64);
}

void* ipc_open(const char handle[64]) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, 64);
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

void ipc_close(void* p) {
  if (p != nullptr) cudaIpcCloseMemHandle(p);
}

void rs_bucket(const PeerTable& t, int rank, int world, int bucket, long long bucket_off, long long shard, float* out,
               float* partial, int blocks, unsigned long long epoch, float scale, long long timeout_ns, int* status,
               cudaStream_t stream) {
  if (world > kMaxRanks || bucket >= kMaxBuckets || (shard & 3) != 0)
    throw std::invalid_argument("rs_bucket: world / bucket / shard alignment out of range");
#define PB_RS_CASE(W)                                                                                  \
  case W:                                                                                              \
    rs_bucket_kernel<W><<<blocks, 256, 0, stream>>>(t, rank, bucket, bucket_off, shard, out, partial, epoch, scale, \
                                                    timeout_ns, status);                               \
    break;
  switch (world) {
    PB_RS_CASE(1)
    PB_RS_CASE(2)
    PB_RS_CASE(3)
    PB_RS_CASE(4)
    PB_RS_CASE(5)
    PB_RS_CASE(6)
    PB_RS_CASE(7)
    PB_RS_CASE(8)
    default:
      throw std::invalid_argument("rs_bucket: world size must be 1..8");
  }
#undef PB_RS_CASE
  check(cudaGetLastError(), "rs_bucket launch");
}

void norm_exchange(const PeerTable& t, int rank, int world, const float* partial, int n_partial,
                   unsigned long long epoch, float max_norm, float* norm_out, float* clip_out, long long timeout_ns,
                   int* status, cudaStream_t stream) {
  norm_exchange_kernel<<<1, 256, 0, stream>>>(t, rank, world, partial, n_partial, epoch, max_norm, norm_out, clip_out,
                                              timeout_ns, status);
  check(cudaGetLastError(), "norm_exchange launch");
}

void adamw_scatter(const PeerTable& t, int world, const ShardSegment* segs, int nseg, long long n_local, float* master,
                   float* m1, float* m2, const float* grad, const float* clip, const AdamHyper& hp, int blocks,
                   cudaStream_t stream, int local_rank) {
  if ((n_local & 7) != 0) throw std::invalid_argument("adamw_scatter: local shard must be a multiple of 8");
  adamw_scatter_kernel<<<blocks, 256, 0, stream>>>(t, world, local_rank, segs, nseg, n_local, master, m1, m2, grad,
                                                   clip, hp);
  check(cudaGetLastError(), "adamw_scatter launch");
}

void gather_shards(const PeerTable& t, int world, long long src_off, long long count, void* dst, cudaStream_t stream) {
  for (int r = 0; r < world; ++r) {
    const auto* src = reinterpret_cast<const __nv_bfloat16*>(t.param[r]) + src_off;
    auto* out = static_cast<__nv_bfloat16*>(dst) + static_cast<long long>(r) * count;
    check(cudaMemcpyAsync(out, src, static_cast<size_t>(count) * 2, cudaMemcpyDeviceToDevice, stream),
          "gather_shards copy");
  }
}

void peer_barrier(const unsigned long long* done, unsigned long long target, long long timeout_ns, int* status,
                  cudaStream_t stream) {
  peer_barrier_kernel<<<1, 32, 0, stream>>>(done, target, timeout_ns, status);
  check(cudaGetLastError(), "peer_barrier launch");
}

}  // namespace pb

// Decode attention: one new query token per sequence against a KV cache whose
// valid length is a per-sequence device value.
//
// Decoding reads every cached key and value once per token and does a handful of
// FLOPs per byte, so the kernel is built for HBM bandwidth, not the tensor
// cores. The rows of one (sequence, KV head) are contiguous in the cache, so a
// producer thread streams them in 64-row chunks with bulk copies into a ring of
// shared-memory stages (mbarrier completion) and four consumer warps read them
// from there: each CTA keeps several chunks of K and V in flight without spending
// registers on them. A split over the key axis spreads even one sequence with a
// few KV heads over all SMs. Lengths are read on the device, which keeps a whole
// decode step free of host synchronisation and capturable in one CUDA graph.
//
// Layout: q [B, H, D]; caches [B, Hkv, T, D] with contiguous rows (any batch and
// head strides); lengths int32 [B] = keys visible to the query (its own key
// included, already written). Query head h reads KV head h / (H / Hkv).
// A window w >= 0 hides keys older than position len - 1 - w.
//
// Per CTA: GT query heads of one KV head over one key split. In a consumer warp a
// key row is spread over D/8 lanes (8 channels each) and 32/(D/8) rows are scored
// per instruction; a lane group scores 4 rows before one running-max update, so
// the exp and rescale work is shared by the batch. Partial (max, sum, acc) per
// split go to a workspace that the combine kernel merges; with one split the
// kernel writes the output directly.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;

__device__ __forceinline__ void unpack8(const uint4& raw, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// exp2 of a difference whose larger side may be -inf (an empty partial): 0 then.
__device__ __forceinline__ float exp2_or_zero(float x, float m) { return m == -INFINITY ? 0.f : exp2f(x - m); }

template <int D>
struct DecCfg {
  static constexpr int kRows = 64;                       // keys per pipeline chunk
  static constexpr int kStages = D == 64 ? 4 : 3;
  static constexpr int kChunkBytes = kRows * D * 2;      // one chunk of K (or V): contiguous cache rows
  static constexpr int kSmem = kStages * 2 * kChunkBytes + 2 * kStages * 8 + 16;
};

// Warps 0..3 consume (16 keys of every 64-key chunk each); warp 4's lane 0 streams the chunks of K
// and V into a ring of shared-memory stages with bulk copies (the rows of one (sequence, KV head)
// are contiguous), so each CTA keeps up to kStages chunks in flight without holding them in
// registers. Every wait is bounded; a wait that runs out records kTimeoutProducer and the CTA
// stops early (its partial then only covers the chunks it finished).
template <int D, int GT>
__global__ void __launch_bounds__(kDecThreads + 32) decode_attn_kernel(DecodeAttnParams p) {
  using Cfg = DecCfg<D>;
  constexpr int LPK = D / 8;     // lanes per key row
  constexpr int GPW = 32 / LPK;  // key rows per warp instruction
  constexpr int kWarpRows = Cfg::kRows / kDecWarps;
  constexpr int kBatch = GT >= 8 ? 2 : 4;  // rows per lane group between running-max updates
  constexpr int kRounds = kWarpRows / (GPW * kBatch);
  static_assert(kWarpRows % (GPW * kBatch) == 0, "rows per warp must split into batches");
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ks = smem;
  uint8_t* vs = smem + S * Cfg::kChunkBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * S * Cfg::kChunkBytes);
  uint64_t* empty = full + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
  __shared__ float red[kDecWarps][GT][D + 2];  // per consumer warp: channels, then (max, sum)

  const int split = blockIdx.x;
  const int head0 = blockIdx.y * GT;
  const int b = blockIdx.z;
  const int hk = head0 / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int len = min(max(p.lengths[b], 0), p.T);
  int lo = split * p.chunk;
  const int hi = min(lo + p.chunk, len);
  if (p.window >= 0) lo = max(lo, len - 1 - p.window);
  const int nchunks = hi > lo ? (hi - lo + Cfg::kRows - 1) / Cfg::kRows : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kDecWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const __nv_bfloat16* kb = p.k + b * p.k_sb + hk * p.k_sh;
      const __nv_bfloat16* vb = p.v + b * p.v_sb + hk * p.v_sh;
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c % S;
        if (c >= S && !mbar_wait(&empty[st], ((c / S) - 1) & 1, p.status, kTimeoutProducer, abort_flag)) break;
        const int base = lo + c * Cfg::kRows;
        const uint32_t bytes = static_cast<uint32_t>(min(Cfg::kRows, hi - base)) * D * 2;
        mbar_arrive_expect_tx(&full[st], 2 * bytes);
        bulk_load(ks + st * Cfg::kChunkBytes, kb + static_cast<long long>(base) * D, bytes, &full[st]);
        bulk_load(vs + st * Cfg::kChunkBytes, vb + static_cast<long long>(base) * D, bytes, &full[st]);
        issued = c + 1;
      }
      // No copy may still be landing in shared memory when the CTA exits: wait (bounded) for the
      // last chunk issued on every stage. In a normal run the consumers already saw them all.
      for (int c = max(0, issued - S); c < issued; ++c) mbar_wait(&full[c % S], (c / S) & 1, p.status, kTimeoutDrain, nullptr);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int sub = lane % LPK;
    const int grp = lane / LPK;
    float qf[GT][8];
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      const uint4 raw =
          *reinterpret_cast<const uint4*>(p.q + (static_cast<long long>(b) * p.H + head0 + h) * D + sub * 8);
      unpack8(raw, qf[h]);
#pragma unroll
      for (int c = 0; c < 8; ++c) qf[h][c] *= p.scale_log2;
    }
    float m[GT], l[GT], acc[GT][8];
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[h][c] = 0.f;
    }
    for (int c = 0; c < nchunks; ++c) {
      const int st = c % S;
      if (!mbar_wait_warp(&full[st], (c / S) & 1, p.status, kTimeoutProducer, abort_flag)) break;
      const int valid = min(Cfg::kRows, hi - (lo + c * Cfg::kRows));  // rows of this chunk (all lanes agree)
      const uint8_t* kc = ks + st * Cfg::kChunkBytes;
      const uint8_t* vc = vs + st * Cfg::kChunkBytes;
#pragma unroll
      for (int rd = 0; rd < kRounds; ++rd) {
        float sc[kBatch][GT];
        int rows[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          rows[i] = warp * kWarpRows + (rd * kBatch + i) * GPW + grp;
          const uint4 kr = *reinterpret_cast<const uint4*>(kc + rows[i] * (D * 2) + sub * 16);
          float kf[8];
          unpack8(kr, kf);
#pragma unroll
          for (int h = 0; h < GT; ++h) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = fmaf(qf[h][e], kf[e], d);
            sc[i][h] = d;
          }
        }
#pragma unroll
        for (int off = LPK / 2; off > 0; off >>= 1) {
#pragma unroll
          for (int i = 0; i < kBatch; ++i)
#pragma unroll
            for (int h = 0; h < GT; ++h) sc[i][h] += __shfl_xor_sync(0xffffffffu, sc[i][h], off);
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (rows[i] >= valid) {
#pragma unroll
            for (int h = 0; h < GT; ++h) sc[i][h] = -INFINITY;
          }
        }
#pragma unroll
        for (int h = 0; h < GT; ++h) {
          float mx = sc[0][h];
#pragma unroll
          for (int i = 1; i < kBatch; ++i) mx = fmaxf(mx, sc[i][h]);
          const float mn = fmaxf(m[h], mx);  // -inf while this lane group has seen no valid row
          const float corr = exp2_or_zero(m[h], mn);
          l[h] *= corr;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[h][e] *= corr;
          m[h] = mn;
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          // rows past the end of a partial chunk hold whatever the stage held before (possibly NaN
          // bit patterns): their weight is 0, and so must their values be
          float vf[8];
          unpack8(rows[i] < valid ? *reinterpret_cast<const uint4*>(vc + rows[i] * (D * 2) + sub * 16)
                                  : make_uint4(0u, 0u, 0u, 0u),
                  vf);
#pragma unroll
          for (int h = 0; h < GT; ++h) {
            const float pr = exp2_or_zero(sc[i][h], m[h]);  // 0 for a row past the end (-inf)
            l[h] += pr;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[h][e] = fmaf(pr, vf[e], acc[h][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // Merge the key groups of a warp (lanes with the same channel slice).
#pragma unroll
    for (int off = LPK; off < 32; off <<= 1) {
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m[h], off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l[h], off);
        const float mn = fmaxf(m[h], m2);
        const float c1 = exp2_or_zero(m[h], mn), c2 = exp2_or_zero(m2, mn);
        l[h] = l[h] * c1 + l2 * c2;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a2 = __shfl_xor_sync(0xffffffffu, acc[h][e], off);
          acc[h][e] = acc[h][e] * c1 + a2 * c2;
        }
        m[h] = mn;
      }
    }
    if (lane < LPK) {
#pragma unroll
      for (int h = 0; h < GT; ++h) {
#pragma unroll
        for (int e = 0; e < 8; ++e) red[warp][h][sub * 8 + e] = acc[h][e];
        if (sub == 0) {
          red[warp][h][D] = m[h];
          red[warp][h][D + 1] = l[h];
        }
      }
    }
  }
  __syncthreads();

  // Merge the four consumer warps: thread t owns 8 channels of one head.
  const int t = threadIdx.x;
  if (t >= GT * LPK) return;
  const int h = t / LPK, sl = t % LPK;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, red[w][h][D]);
  float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) {
    const float c = exp2_or_zero(red[w][h][D], M);
    L += red[w][h][D + 1] * c;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] += red[w][h][sl * 8 + e] * c;
  }
  const long long row = static_cast<long long>(b) * p.H + head0 + h;
  if (p.splits == 1) {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    uint4 raw;
    raw.x = pack2(o[0] * inv, o[1] * inv);
    raw.y = pack2(o[2] * inv, o[3] * inv);
    raw.z = pack2(o[4] * inv, o[5] * inv);
    raw.w = pack2(o[6] * inv, o[7] * inv);
    *reinterpret_cast<uint4*>(p.out + row * D + sl * 8) = raw;
  } else {
    float* pa = p.part_acc + (row * p.splits + split) * D + sl * 8;
    reinterpret_cast<float4*>(pa)[0] = make_float4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<float4*>(pa)[1] = make_float4(o[4], o[5], o[6], o[7]);
    if (sl == 0) {
      p.part_ml[(row * p.splits + split) * 2] = M;
      p.part_ml[(row * p.splits + split) * 2 + 1] = L;
    }
  }
}

// One warp per (sequence, head) merges the splits' partials. The lanes split the work two ways:
// LPK lanes cover the D channels (8 each) and 32 / LPK lane groups take every (32 / LPK)-th
// split, so the split loop is short and its loads independent; the groups then combine
// their (max, sum, acc) with shuffles.
template <int D>
__global__ void decode_combine_kernel(DecodeAttnParams p, int rows) {
  constexpr int LPK = D / 8;
  constexpr int G = 32 / LPK;  // split groups per warp
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps leave together
  const int sl = lane % LPK, grp = lane / LPK;
  const float* ml = p.part_ml + static_cast<long long>(row) * p.splits * 2;
  float M = -INFINITY;
  for (int s = grp; s < p.splits; s += G) M = fmaxf(M, ml[2 * s]);
  float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = grp; s < p.splits; s += G) {
    const float c = exp2_or_zero(ml[2 * s], M);
    L += ml[2 * s + 1] * c;
    const float4* pa =
        reinterpret_cast<const float4*>(p.part_acc + (static_cast<long long>(row) * p.splits + s) * D + sl * 8);
    const float4 a = pa[0], bb = pa[1];
    o[0] = fmaf(a.x, c, o[0]);
    o[1] = fmaf(a.y, c, o[1]);
    o[2] = fmaf(a.z, c, o[2]);
    o[3] = fmaf(a.w, c, o[3]);
    o[4] = fmaf(bb.x, c, o[4]);
    o[5] = fmaf(bb.y, c, o[5]);
    o[6] = fmaf(bb.z, c, o[6]);
    o[7] = fmaf(bb.w, c, o[7]);
  }
#pragma unroll
  for (int off = LPK; off < 32; off <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, M, off);
    const float l2 = __shfl_xor_sync(0xffffffffu, L, off);
    const float mn = fmaxf(M, m2);
    const float c1 = exp2_or_zero(M, mn), c2 = exp2_or_zero(m2, mn);
    L = L * c1 + l2 * c2;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = o[e] * c1 + __shfl_xor_sync(0xffffffffu, o[e], off) * c2;
    M = mn;
  }
  if (grp != 0) return;
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint4 raw;
  raw.x = pack2(o[0] * inv, o[1] * inv);
  raw.y = pack2(o[2] * inv, o[3] * inv);
  raw.z = pack2(o[4] * inv, o[5] * inv);
  raw.w = pack2(o[6] * inv, o[7] * inv);
  *reinterpret_cast<uint4*>(p.out + static_cast<long long>(row) * D + sl * 8) = raw;
}

template <int D, int GT>
void launch_decode(const DecodeAttnParams& p, int B, cudaStream_t stream) {
  const dim3 grid(p.splits, p.H / GT, B);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(decode_attn_kernel<D, GT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecCfg<D>::kSmem);
    configured = true;
  }
  decode_attn_kernel<D, GT><<<grid, kDecThreads + 32, DecCfg<D>::kSmem, stream>>>(p);
  if (p.splits > 1) {
    const int rows = B * p.H;
    decode_combine_kernel<D><<<(rows + 3) / 4, 128, 0, stream>>>(p, rows);
  }
}

template <int D>
void dispatch_group(const DecodeAttnParams& p, int B, int gt, cudaStream_t stream) {
  switch (gt) {
    case 8: launch_decode<D, 8>(p, B, stream); break;
    case 4: launch_decode<D, 4>(p, B, stream); break;
    case 2: launch_decode<D, 2>(p, B, stream); break;
    default: launch_decode<D, 1>(p, B, stream); break;
  }
}

}  // namespace

int decode_attn_heads_per_cta(int group) {
  for (int gt : {8, 4, 2}) {
    if (group % gt == 0) return gt;
  }
  return 1;
}

int decode_attn_splits(int B, int H, int group, int T, int sm_count) {
  const int ctas = B * (H / decode_attn_heads_per_cta(group));
  const int want = (2 * sm_count + ctas - 1) / ctas;  // about two CTAs per SM
  const int most = (T + 255) / 256;                    // at least four 64-key chunks per split (a full ring)
  return want < 1 ? 1 : (want < most ? want : (most < 1 ? 1 : most));
}

void decode_attn(const DecodeAttnParams& p, int B, int D, cudaStream_t stream) {
  const int gt = decode_attn_heads_per_cta(p.group);
  if (D == 64) {
    dispatch_group<64>(p, B, gt, stream);
  } else {
    dispatch_group<128>(p, B, gt, stream);
  }
}

}  // namespace pb

// Decode attention: one new query token per sequence against a KV cache whose
// valid length is a per-sequence device value.
//
// Decoding reads every cached key and value once per token and does a handful of
// FLOPs per byte, so the kernel is built for HBM bandwidth, not the tensor
// cores: 16-byte row loads, several keys in flight per lane, and a split over
// the key axis so that even one sequence with a few KV heads spreads over all
// SMs. Lengths are read on the device, which keeps a whole decode step free of
// host synchronisation and capturable in one CUDA graph.
//
// Layout: q [B, H, D]; caches [B, Hkv, T, D] with contiguous rows (any batch and
// head strides); lengths int32 [B] = keys visible to the query (its own key
// included, already written). Query head h reads KV head h / (H / Hkv).
// A window w >= 0 hides keys older than position len - 1 - w.
//
// Per CTA: GT query heads of one KV head over one key split. A key row is spread
// over D/8 lanes (8 channels each); a warp covers 32/(D/8) rows per load. Each
// lane group scores a batch of rows (4, or 2 at eight heads per CTA) before one
// running-max update, so the exp and rescale work is shared by the batch. Partial (max, sum, acc) per split go to a
// workspace that the combine kernel merges; with one split the kernel writes the
// output directly.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

template <int D, int GT>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(DecodeAttnParams p) {
  constexpr int LPK = D / 8;       // lanes per key row
  constexpr int GPW = 32 / LPK;    // key rows per warp load
  constexpr int NG = kDecWarps * GPW;
  constexpr int kBatch = GT >= 8 ? 2 : 4;  // rows per lane between max updates (register bound at 8 heads)
  const int split = blockIdx.x;
  const int head0 = blockIdx.y * GT;  // first query head of this CTA
  const int b = blockIdx.z;
  const int hk = head0 / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % LPK;
  const int grp = warp * GPW + lane / LPK;

  const int len = min(max(p.lengths[b], 0), p.T);
  int lo = split * p.chunk;
  const int hi = min(lo + p.chunk, len);
  if (p.window >= 0) lo = max(lo, len - 1 - p.window);

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

  const __nv_bfloat16* kb = p.k + b * p.k_sb + hk * p.k_sh + sub * 8;
  const __nv_bfloat16* vb = p.v + b * p.v_sb + hk * p.v_sh + sub * 8;
  // The loop bound is the same for every lane: the row shuffles below name the whole warp, so
  // no lane may leave the loop while others still run it (a lane group whose rows are all past
  // `hi` scores -inf and adds nothing).
  for (int base = lo; base < hi; base += NG * kBatch) {
    const int j0 = base + grp;
    uint4 kr[kBatch], vr[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int j = j0 + i * NG;
      if (j < hi) {
        kr[i] = __ldg(reinterpret_cast<const uint4*>(kb + static_cast<long long>(j) * D));
        vr[i] = __ldg(reinterpret_cast<const uint4*>(vb + static_cast<long long>(j) * D));
      } else {
        kr[i] = make_uint4(0, 0, 0, 0);
        vr[i] = make_uint4(0, 0, 0, 0);
      }
    }
    float s[kBatch][GT];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      float kf[8];
      unpack8(kr[i], kf);
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) d = fmaf(qf[h][c], kf[c], d);
        s[i][h] = d;
      }
    }
#pragma unroll
    for (int off = LPK / 2; off > 0; off >>= 1) {
#pragma unroll
      for (int i = 0; i < kBatch; ++i)
#pragma unroll
        for (int h = 0; h < GT; ++h) s[i][h] += __shfl_xor_sync(0xffffffffu, s[i][h], off);
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (j0 + i * NG >= hi) {
#pragma unroll
        for (int h = 0; h < GT; ++h) s[i][h] = -INFINITY;
      }
    }
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      float mx = s[0][h];
#pragma unroll
      for (int i = 1; i < kBatch; ++i) mx = fmaxf(mx, s[i][h]);
      const float mn = fmaxf(m[h], mx);  // -inf while this lane group has seen no valid row
      const float corr = exp2_or_zero(m[h], mn);
      l[h] *= corr;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[h][c] *= corr;
      m[h] = mn;
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      float vf[8];
      unpack8(vr[i], vf);
#pragma unroll
      for (int h = 0; h < GT; ++h) {
        const float pr = exp2_or_zero(s[i][h], m[h]);  // 0 for an invalid row (-inf)
        l[h] += pr;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[h][c] = fmaf(pr, vf[c], acc[h][c]);
      }
    }
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
      for (int c = 0; c < 8; ++c) {
        const float a2 = __shfl_xor_sync(0xffffffffu, acc[h][c], off);
        acc[h][c] = acc[h][c] * c1 + a2 * c2;
      }
      m[h] = mn;
    }
  }

  // Merge the warps through shared memory: [warp][head][D channels + (max, sum)].
  __shared__ float red[kDecWarps][GT][D + 2];
  if (lane < LPK) {
#pragma unroll
    for (int h = 0; h < GT; ++h) {
#pragma unroll
      for (int c = 0; c < 8; ++c) red[warp][h][sub * 8 + c] = acc[h][c];
      if (sub == 0) {
        red[warp][h][D] = m[h];
        red[warp][h][D + 1] = l[h];
      }
    }
  }
  __syncthreads();
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
    for (int k = 0; k < 8; ++k) o[k] += red[w][h][sl * 8 + k] * c;
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

// One warp per (sequence, head): merge the splits' partials into the output row.
template <int D>
__global__ void decode_combine_kernel(DecodeAttnParams p, int rows) {
  constexpr int LPK = D / 8;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows || lane >= LPK) return;
  const float* ml = p.part_ml + static_cast<long long>(row) * p.splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, ml[2 * s]);
  float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < p.splits; ++s) {
    const float c = exp2_or_zero(ml[2 * s], M);
    if (c == 0.f) continue;
    L += ml[2 * s + 1] * c;
    const float4* pa = reinterpret_cast<const float4*>(p.part_acc + (static_cast<long long>(row) * p.splits + s) * D +
                                                       lane * 8);
    const float4 a = pa[0], bb = pa[1];
    o[0] += a.x * c;
    o[1] += a.y * c;
    o[2] += a.z * c;
    o[3] += a.w * c;
    o[4] += bb.x * c;
    o[5] += bb.y * c;
    o[6] += bb.z * c;
    o[7] += bb.w * c;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint4 raw;
  raw.x = pack2(o[0] * inv, o[1] * inv);
  raw.y = pack2(o[2] * inv, o[3] * inv);
  raw.z = pack2(o[4] * inv, o[5] * inv);
  raw.w = pack2(o[6] * inv, o[7] * inv);
  *reinterpret_cast<uint4*>(p.out + static_cast<long long>(row) * D + lane * 8) = raw;
}

template <int D, int GT>
void launch_decode(const DecodeAttnParams& p, int B, cudaStream_t stream) {
  const dim3 grid(p.splits, p.H / GT, B);
  decode_attn_kernel<D, GT><<<grid, kDecThreads, 0, stream>>>(p);
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
  const int want = (4 * sm_count + ctas - 1) / ctas;  // about four CTAs per SM
  const int most = (T + 63) / 64;                      // at least 64 keys per split
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

// Shared pieces of the flash-attention kernels (forward and backward).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace attn {

constexpr int kTile = 128;          // rows per Q / K / V tile
constexpr int kChunkBytes = 128 * 128;  // one [128 rows][64 bf16] swizzled chunk = 16 KB
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Packed fp32 pairs (sm_100 f32x2 arithmetic): two lanes of work per FMA-pipe instruction.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AttnParams {
  int B, S, T, H, Hkv, D;  // D: query / key head dim
  int Dv;                   // value head dim (== D except for MLA's 192 / 128)
  float scale_log2;  // softmax scale * log2(e)
  float scale;
  int causal;
  int window;  // < 0: none
  // outputs / extra inputs
  void* o;           // fwd: O out; bwd: O in
  long long o_sb, o_ss, o_sh;
  float* lse;        // [B, H, S]
  float* delta;      // [B, H, S]
  float* nlse2;      // optional [B, H, S] output of the delta kernel: -lse * log2(e)
  int vec_s;         // row stride of delta / nlse2 per (b, h): S, or S rounded up to 4 for 16-byte bulk reads
  const void* dout;  // [B, S, H, D]
  long long do_sb, do_ss, do_sh;
  void* dq;  // [B, S, H, D] bf16 out
  long long dq_sb, dq_ss, dq_sh;
  void* dk;  // [B, T, Hkv, D] bf16 out
  void* dv;
  long long dk_sb, dk_ss, dk_sh;
  long long dv_sb, dv_ss, dv_sh;
  int* status;
  int* trace;  // optional progress record, 8 ints per CTA (stage, SM, producer / MMA / softmax tile), for diagnosis
};

__device__ __forceinline__ void trace_put(const AttnParams& p, int slot, int value) {
  if (p.trace != nullptr) {
    reinterpret_cast<volatile int*>(p.trace)[blockIdx.x * 8 + slot] = value;
    __threadfence_system();
  }
}

__device__ __forceinline__ int sm_id() {
  int id;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
  return id;
}

// Inclusive key range [lo, hi] visible to query rows [q0, q0 + rows).
__device__ __forceinline__ void key_range(const AttnParams& p, int q0, int rows, int& lo, int& hi) {
  const int off = p.T - p.S;
  hi = p.T - 1;
  lo = 0;
  if (p.causal) hi = min(hi, off + q0 + rows - 1);
  if (p.window >= 0) lo = max(0, off + q0 - p.window);
}

// Is key `k` visible to query `q` (absolute indices within the sequence)?
__device__ __forceinline__ bool visible(const AttnParams& p, int q, int k) {
  if (k >= p.T || q >= p.S) return false;
  const int pos = p.T - p.S + q;
  if (p.causal && k > pos) return false;
  if (p.window >= 0 && k < pos - p.window) return false;
  return true;
}

// K-major operand descriptor for chunked [128][D] tiles: MMA step kk covers
// d in [16 kk, 16 kk + 16).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_base, int kk, int chunk_bytes = kChunkBytes) {
  return make_sw128_desc(tile_base + (kk >> 2) * chunk_bytes + (kk & 3) * 32, 16, 1024);
}

// MN-major operand descriptor for a [128 rows = K][D = N] tile (N contiguous in
// 64-element chunks): MMA step kk covers rows [16 kk, 16 kk + 16).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_base, int kk, int chunk_bytes = kChunkBytes) {
  return make_sw128_desc(tile_base + kk * 2048, chunk_bytes, 1024);
}

__device__ __forceinline__ void load_tile(void* dst, const CUtensorMap* map, uint64_t* bar, int head_col, int row0,
                                          int b, int D, int chunk_bytes = kChunkBytes) {
  for (int c = 0; c < D / 64; ++c)
    tma_load_3d(static_cast<uint8_t*>(dst) + c * chunk_bytes, map, bar, head_col + 64 * c, row0, b);
}


inline void make_bshd_map(CUtensorMap* m, const AttnTensor& t, int heads, int D, int rows = kTile) {
  // [B, S, heads*D] view with the tensor's own token and batch strides.
  make_tmap_3d_bf16(m, t.ptr, static_cast<long long>(heads) * D, t.seq, t.batch, t.s_seq, t.s_batch, 64, rows,
                    true);
}

template <typename K>
inline void set_smem(K kern, int bytes) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Forward with two query tiles per CTA (attention_fwd3.cu): Q / K / V maps with 128-row boxes.
void attn_fwd3_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& p,
                      int D, cudaStream_t stream);

// Fused backward for head dim 64 (attention_bwd_d64.cu): Q / dO / K / V maps with 128-row
// boxes, dQ accumulator map [B*H*S, 64] fp32 with 32 x 32 boxes and 128-byte swizzle.
void attn_bwd_d64_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                         const CUtensorMap& mdq, const AttnParams& p, int grid, cudaStream_t stream);


}  // namespace attn
}  // namespace pb

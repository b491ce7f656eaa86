// Multi-head latent attention decode in latent space (the "absorbed" order), sm_100a.
//
// One new query token per sequence. With W_UK folded into the query, every head h
// scores the cached latent row c_kv[t] (512 wide) plus the shared rotary key
// k_pe[t] (64 wide) with one 576-wide query q[h] = [q_abs | q_pe], and the value
// is the latent row itself:
//
//   s[h, t]  = scale * (q[h] . [c_kv[t] | k_pe[t]])
//   lat[h]   = sum_t softmax_t(s[h, :]) * c_kv[t]              (512 wide)
//
// All heads share one key row, so a 128-key tile is one tensor-core problem with
// the keys on the M axis (tcgen05 needs M >= 64; there are only 16-32 heads):
//
//   S^T [128 keys, NH]   = K_tile [128, 576] . Q^T          (A K-major, B K-major)
//   O^T [512 lat, NH]   += C_tile^T [512, 128] . P^T [128, NH]
//                          (A = the same c_kv rows read M-major, B = P K-major)
//
// S^T and the four 128-row blocks of O^T live in TMEM. Per tile the softmax warps
// (one key row per thread) take the per-head maximum and sum across the 128 rows,
// write P in bf16 to shared memory in the 128-byte-swizzled K-major layout the
// MMA reads, and rescale O^T in TMEM when a head's maximum moved. The producer
// streams each tile into a ring of 32 KB stages with TMA: four stages of c_kv
// column pairs and one of k_pe. The MMA warp frees the k_pe stage after S^T and
// keeps the four c_kv stages for O^T (the same bytes, read M-major), so every
// cache row is read from HBM once; the spare stages load the next tile. A split of the
// keys over CTAs spreads a few sequences over all SMs; partial (max, sum, O)
// per split are merged by a combine kernel. Heads beyond 32 run in groups of 32,
// one CTA per group. Every mbarrier wait is bounded and reports through `status`.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int kLat = 512, kQK = 576;
constexpr int kKeys = 128;       // keys per tile (the MMA's M)
constexpr int kStageBytes = 32768;  // two 64-column blocks of 128 rows

template <int NH>
struct MlaCfg {
  static constexpr int kRing = NH == 16 ? 6 : 5;  // a tile takes five stages; the rest load ahead
  static constexpr int kQBytes = 9 * NH * 128;  // nine K-major 64-column blocks of NH rows
  static constexpr int kPBytes = 2 * NH * 128;  // P: two K-major blocks of 64 keys
  static constexpr int kRedBytes = 2 * 4 * NH * 4;
  static constexpr int kSmem = 1024 + kRing * kStageBytes + kQBytes + kPBytes + kRedBytes + 256;
  static_assert(kSmem <= 232448, "shared memory per CTA");
  static constexpr int kTmemCols = 5 * NH <= 128 ? 128 : 256;
  static_assert(kQBytes % 1024 == 0 && kPBytes % 1024 == 0, "operand blocks stay 1024-byte aligned");
};

__device__ __forceinline__ void bar_sync_softmax() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// AND of `v` over the four softmax warps (named barrier 1): they leave the tile loop together,
// so none of them is left waiting at a barrier that the others skipped.
__device__ __forceinline__ bool softmax_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n"
      ".reg .pred p, q;\n"
      "setp.ne.u32 p, %1, 0;\n"
      "bar.red.and.pred q, 1, 128, p;\n"
      "selp.u32 %0, 1, 0, q;\n"
      "}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

template <int NH>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float (&v)[NH]) {
  uint32_t r[NH];
  if constexpr (NH == 16) {
    tmem_ld_32x32b_x16(taddr, r);
  } else {
    tmem_ld_32x32b_x32(taddr, r);
  }
  tmem_wait_ld();
#pragma unroll
  for (int h = 0; h < NH; ++h) v[h] = __uint_as_float(r[h]);
}

template <int NH>
__device__ __forceinline__ void tmem_st_row(uint32_t taddr, const float (&v)[NH]) {
  uint32_t r[NH];
#pragma unroll
  for (int h = 0; h < NH; ++h) r[h] = __float_as_uint(v[h]);
  if constexpr (NH == 16) {
    tmem_st_32x32b_x16(taddr, r);
  } else {
    tmem_st_32x32b_x32(taddr, r);
  }
}

template <int NH>
__global__ void __launch_bounds__(192, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmC,
                      const __grid_constant__ CUtensorMap tmR, const MlaDecodeParams p) {
  using Cfg = MlaCfg<NH>;
  constexpr int kRing = Cfg::kRing;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* qs = ring + kRing * kStageBytes;
  uint8_t* ps = qs + Cfg::kQBytes;
  float* red_max = reinterpret_cast<float*>(ps + Cfg::kPBytes);  // [4 warps][NH]
  float* red_sum = red_max + 4 * NH;
  uint64_t* full = reinterpret_cast<uint64_t*>(red_sum + 4 * NH);
  uint64_t* empty = full + kRing;
  uint64_t* q_full = empty + kRing;
  uint64_t* s_full = q_full + 1;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int hg = blockIdx.x % p.head_groups;
  const int split = (blockIdx.x / p.head_groups) % p.splits;
  const int b = blockIdx.x / (p.head_groups * p.splits);
  const int len = p.lengths != nullptr ? min(max(p.lengths[b], 0), p.T) : p.T;
  const int key_lo = split * p.tiles_per_split * kKeys;
  const int key_hi = min(len, key_lo + p.tiles_per_split * kKeys);
  const int ntiles = key_hi > key_lo ? (key_hi - key_lo + kKeys - 1) / kKeys : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t s_col = 0, o_col = NH;  // S^T in columns [0, NH), O^T block m in [NH + m*NH, ...)

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    if (ntiles > 0) {
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
      for (int kb = 0; kb < 9; ++kb) tma_load_2d(qs + kb * NH * 128, &tmQ, q_full, kb * 64, b * p.H + hg * NH);
    }
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int key0 = key_lo + t * kKeys;
      for (int j = 0; j < 5; ++j) {  // 4 latent column pairs, then the rotary block
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kTimeoutProducer, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* st = ring + stage * kStageBytes;
        if (j == 4) {
          mbar_arrive_expect_tx(&full[stage], kStageBytes / 2);
          tma_load_3d(st, &tmR, &full[stage], 0, key0, b);
        } else {
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_3d(st, &tmC, &full[stage], j * 128, key0, b);
          tma_load_3d(st + kStageBytes / 2, &tmC, &full[stage], j * 128 + 64, key0, b);
        }
        ++issued;
        if (++stage == kRing) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      for (int i = 0; i < min(issued, kRing); ++i) {
        if (--stage < 0) {
          stage = kRing - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16(kKeys, NH, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(kKeys, NH, true, false);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = ntiles == 0 || mbar_wait(q_full, 0, p.status, kTimeoutMma, abort_flag);
    const uint32_t q_base = smem_u32(qs), p_base = smem_u32(ps);
    for (int t = 0; t < ntiles && ok; ++t) {
      int held[4];  // this tile's c_kv stages, kept for O^T
      for (int j = 0; j < 5 && ok; ++j) {
        if (!mbar_wait(&full[stage], phase, p.status, kTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (j < 4) held[j] = stage;
        const uint32_t st = smem_u32(ring + stage * kStageBytes);
        const int blocks = j == 4 ? 1 : 2;
        for (int hb = 0; hb < blocks; ++hb) {
          const int kb = j == 4 ? 8 : 2 * j + hb;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_sw128_desc(st + hb * (kStageBytes / 2) + kk * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(q_base + kb * NH * 128 + kk * 32, 16, 1024);
            umma_f16(tmem_base + s_col, ad, bd, idesc_s, (kb | kk) != 0 ? 1u : 0u);
          }
        }
        if (j == 4) umma_commit(&empty[stage]);  // the rotary block is done with; c_kv stays
        if (++stage == kRing) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(s_full);
      if (!mbar_wait_sleep(p_full, t & 1, p.status, kTimeoutMma, abort_flag)) break;
      tc_fence_after();
      for (int m = 0; m < 4; ++m) {
        const uint32_t st = smem_u32(ring + held[m] * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          // A: 128 latent rows (two 64-wide chunks 16 KB apart) x 16 keys, M-major
          const uint64_t ad = make_sw128_desc(st + kk * 2048, kStageBytes / 2, 1024);
          const uint64_t bd = make_sw128_desc(p_base + (kk >> 2) * NH * 128 + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem_base + o_col + m * NH, ad, bd, idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[held[m]]);
      }
      umma_commit(o_done);
    }
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax / epilogue (one key row per thread)
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
    float m[NH], l[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
    }
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      if (!softmax_all(mbar_wait_warp(s_full, t & 1, p.status, kTimeoutEpilogue, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[NH];
      tmem_ld_row<NH>(t_row + s_col, s);
      const bool valid = key_lo + t * kKeys + row < key_hi;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        float v = valid ? s[h] * p.scale_log2 : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red_max[wq * NH + h] = v;
        s[h] = valid ? s[h] * p.scale_log2 : -INFINITY;
      }
      bar_sync_softmax();
      float alpha[NH];
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const float tmax = fmaxf(fmaxf(red_max[h], red_max[NH + h]), fmaxf(red_max[2 * NH + h], red_max[3 * NH + h]));
        const float mn = fmaxf(m[h], tmax);
        alpha[h] = m[h] == -INFINITY ? 0.f : exp2f(m[h] - mn);
        m[h] = mn;
        const float pv = s[h] == -INFINITY ? 0.f : exp2f(s[h] - mn);
        s[h] = pv;
        float sum = pv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red_sum[wq * NH + h] = sum;
      }
      // P (bf16) in the K-major 128-byte-swizzled layout: head h = operand row, key = K index
      uint8_t* pblk = ps + (row >> 6) * (NH * 128);
      const int kc = (row & 63) >> 3, kw = (row & 7) * 2;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const __nv_bfloat16 pb = __float2bfloat16_rn(s[h]);
        *reinterpret_cast<__nv_bfloat16*>(pblk + (h >> 3) * 1024 + (h & 7) * 128 + ((kc ^ (h & 7)) << 4) + kw) = pb;
      }
      fence_proxy_async_smem();  // generic-proxy writes of P, read next by the MMA (async proxy)
      bar_sync_softmax();
#pragma unroll
      for (int h = 0; h < NH; ++h)
        l[h] = l[h] * alpha[h] + (red_sum[h] + red_sum[NH + h] + red_sum[2 * NH + h] + red_sum[3 * NH + h]);
      // Every thread holds the same maxima, so this test is uniform across the four warps. When no
      // head's maximum moved, O^T stays as it is and the wait on the previous tile's MMAs is skipped.
      bool moved = false;
#pragma unroll
      for (int h = 0; h < NH; ++h) moved |= alpha[h] != 1.f;
      if (t > 0 && moved) {
        // the previous tile's O^T MMAs must have finished before O^T is rescaled
        if (!softmax_all(mbar_wait_warp(o_done, (t - 1) & 1, p.status, kTimeoutEpilogue, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int mb = 0; mb < 4; ++mb) {
          float o[NH];
          tmem_ld_row<NH>(t_row + o_col + mb * NH, o);
#pragma unroll
          for (int h = 0; h < NH; ++h) o[h] *= alpha[h];
          tmem_st_row<NH>(t_row + o_col + mb * NH, o);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && ntiles > 0) ok = mbar_wait_warp(o_done, (ntiles - 1) & 1, p.status, kTimeoutEpilogue, abort_flag);
    if (ok && ntiles > 0) tc_fence_after();
    const int h_base = hg * NH;
    const long long part = (static_cast<long long>(b) * p.splits + split) * p.H;
#pragma unroll 1
    for (int mb = 0; mb < 4; ++mb) {
      float o[NH];
      if (ok && ntiles > 0) {
        tmem_ld_row<NH>(t_row + o_col + mb * NH, o);
      } else {
#pragma unroll
        for (int h = 0; h < NH; ++h) o[h] = 0.f;
      }
      const int lat = mb * kKeys + row;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        if (h_base + h >= p.H) continue;
        if (p.splits == 1) {
          const float v = l[h] > 0.f ? o[h] / l[h] : 0.f;
          p.out[(static_cast<long long>(b) * p.H + h_base + h) * kLat + lat] = __float2bfloat16_rn(v);
        } else {
          p.part_o[(part + h_base + h) * kLat + lat] = o[h];
        }
      }
    }
    if (p.splits > 1 && warp == 2 && lane == 0) {
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        if (h_base + h >= p.H) continue;
        p.part_ml[(part + h_base + h) * 2] = ntiles > 0 ? m[h] : -INFINITY;
        p.part_ml[(part + h_base + h) * 2 + 1] = l[h];
      }
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

// out[b, h, :] = sum_s w_s O_s / sum_s w_s l_s with w_s = 2^(m_s - max_s m_s); empty splits (m = -inf) skipped.
__global__ void __launch_bounds__(128) mla_decode_combine_kernel(const MlaDecodeParams p) {
  const long long bh = blockIdx.x;  // b * H + h
  const long long b = bh / p.H, h = bh % p.H;
  float mx = -INFINITY;
  for (int s = 0; s < p.splits; ++s) mx = fmaxf(mx, p.part_ml[((b * p.splits + s) * p.H + h) * 2]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float den = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const long long idx = (b * p.splits + s) * p.H + h;
    const float ms = p.part_ml[idx * 2];
    if (ms == -INFINITY) continue;
    const float w = exp2f(ms - mx);
    den += w * p.part_ml[idx * 2 + 1];
    const float4 o = reinterpret_cast<const float4*>(p.part_o + idx * kLat)[threadIdx.x];
    acc[0] += w * o.x;
    acc[1] += w * o.y;
    acc[2] += w * o.z;
    acc[3] += w * o.w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  __nv_bfloat16* dst = p.out + bh * kLat + threadIdx.x * 4;
  dst[0] = __float2bfloat16_rn(acc[0] * inv);
  dst[1] = __float2bfloat16_rn(acc[1] * inv);
  dst[2] = __float2bfloat16_rn(acc[2] * inv);
  dst[3] = __float2bfloat16_rn(acc[3] * inv);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <int NH>
void launch_mla(const CUtensorMap& q, const CUtensorMap& c, const CUtensorMap& r, const MlaDecodeParams& p, int grid,
                cudaStream_t stream) {
  auto kern = mla_decode_kernel<NH>;
  static bool configured = false;
  if (!configured) {
    check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MlaCfg<NH>::kSmem),
          "mla decode smem attribute");
    configured = true;
  }
  kern<<<grid, 192, MlaCfg<NH>::kSmem, stream>>>(q, c, r, p);
  check(cudaGetLastError(), "mla decode launch");
}

}  // namespace

int mla_decode_head_tile(int H) { return H <= 16 ? 16 : 32; }

void mla_decode_plan(int B, int H, int T, int sm_count, int* splits, int* tiles_per_split) {
  const int tiles = (T + kKeys - 1) / kKeys;
  const int groups = (H + mla_decode_head_tile(H) - 1) / mla_decode_head_tile(H);
  // One CTA fits an SM (the ring takes most of the shared memory): as many key splits as keep the
  // grid within one wave, so no SM runs a second, partial wave while the others idle.
  const int ctas = B * groups;
  int s = sm_count / ctas;
  if (s > tiles) s = tiles;
  if (s < 1) s = 1;
  const int per = (tiles + s - 1) / s;
  *tiles_per_split = per < 1 ? 1 : per;
  *splits = tiles > 0 ? (tiles + *tiles_per_split - 1) / *tiles_per_split : 1;
}

void mla_decode(const MlaDecodeParams& p, const void* q, const void* ckv, long long c_sb, long long c_st, const void* kpe,
                long long r_sb, long long r_st, cudaStream_t stream) {
  if (p.H < 1 || p.T < 1 || p.B < 1) throw std::invalid_argument("mla_decode: empty problem");
  const int nh = mla_decode_head_tile(p.H);
  if (p.head_groups != (p.H + nh - 1) / nh) throw std::invalid_argument("mla_decode: head groups");
  CUtensorMap tq, tc, tr;
  make_tmap_2d_bf16(&tq, q, kQK, static_cast<long long>(p.B) * p.H, kQK, 64, nh);
  make_tmap_3d_bf16(&tc, ckv, kLat, p.T, p.B, c_st, c_sb, 64, kKeys, true);
  make_tmap_3d_bf16(&tr, kpe, 64, p.T, p.B, r_st, r_sb, 64, kKeys, true);
  const int grid = p.B * p.splits * p.head_groups;
  if (nh == 16) launch_mla<16>(tq, tc, tr, p, grid, stream);
  else launch_mla<32>(tq, tc, tr, p, grid, stream);
  if (p.splits > 1) {
    mla_decode_combine_kernel<<<p.B * p.H, 128, 0, stream>>>(p);
    check(cudaGetLastError(), "mla decode combine launch");
  }
}

}  // namespace pb

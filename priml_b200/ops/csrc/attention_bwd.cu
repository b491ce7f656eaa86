// Flash-attention backward for sm_100a (layouts as in attention_fwd.cu).
//
// Two variants. With an fp32 dQ scratch and D = 64: the delta kernel, one fused
// dK/dV/dQ kernel (attention_bwd_d64.cu) and a dQ conversion kernel.
// Otherwise three kernels, no atomics:
//   delta : delta = rowsum(dO * O)
//   dkdv  : one CTA per (b, kv head, 128-key tile) loops over every query head
//           of its group and every 64-query tile: S^T = K Q^T and dP^T = V dO^T
//           into one of two TMEM buffer pairs (so the next pair is computed while
//           the softmax warps turn the current one into P^T / dS^T), then
//           dV += P^T dO and dK += dS^T Q with A read from TMEM.
//   dq    : one CTA per (b, h, 128-query tile) loops over 64-key tiles:
//           S = Q K^T, dP = dO V^T (double buffered), dS = P (dP - delta),
//           dQ += dS K.
// The softmax scale is applied to dK and dQ in the epilogue.
#include <algorithm>

#include "attention_common.cuh"

namespace pb {

namespace {

using namespace attn;

constexpr int kLT = 64;             // rows per loop tile (queries for dkdv, keys for dq)
constexpr int kLChunk = kLT * 128;  // one [64 rows][64 d] swizzled chunk = 8 KB

// ============================================================================ delta
__global__ void attn_delta_kernel(const AttnParams p) {
  // D / 8 threads per (b, q, h) row, one 16-byte load of O and dO each: delta = sum_d dO * O.
  const int tpr = p.Dv / 8;  // delta = rowsum(dO * O) over the value width
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = t / tpr;
  const int part = static_cast<int>(t % tpr);
  const long long total = static_cast<long long>(p.B) * p.S * p.H;
  float acc = 0.f;
  int b = 0, q = 0, h = 0;
  if (row < total) {
    h = static_cast<int>(row % p.H);
    const long long bq = row / p.H;
    q = static_cast<int>(bq % p.S);
    b = static_cast<int>(bq / p.S);
    const uint4 a = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.o) + b * p.o_sb + q * p.o_ss +
                                                    h * p.o_sh + part * 8);
    const uint4 c = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.dout) + b * p.do_sb +
                                                    q * p.do_ss + h * p.do_sh + part * 8);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&aw[j]));
      const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&cw[j]));
      acc += x.x * y.x + x.y * y.y;
    }
  }
  for (int s = tpr / 2; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (row < total && part == 0) {
    const long long bh = static_cast<long long>(b) * p.H + h;
    const long long vidx = bh * p.vec_s + q;
    p.delta[vidx] = acc;
    if (p.nlse2 != nullptr) p.nlse2[vidx] = -p.lse[bh * p.S + q] * kLog2e;
  }
}

// ============================================================================ dK dV
// D: query / key head dim, DV: value head dim. When dK and dV together are too wide for two
// score buffers in TMEM (MLA: 192 + 128), the S^T / dP^T buffers are single (NB = 1) and the
// next step's scores wait until this step's dV / dK MMAs have read P^T / dS^T.
template <int D, int DV>
struct KVSmem {
  static constexpr int kStages = 3;
  static constexpr int NB = 256 + D + DV <= 512 ? 2 : 1;  // score buffers
  static constexpr int kKBytes = (D / 64) * kChunkBytes;   // [128 keys][D]
  static constexpr int kVBytes = (DV / 64) * kChunkBytes;  // [128 keys][DV]
  static constexpr int kQBytes = (D / 64) * kLChunk;       // [64 q][D]
  static constexpr int kDOBytes = (DV / 64) * kLChunk;     // [64 q][DV]
  static constexpr int kBytes = kKBytes + kVBytes + kStages * (kQBytes + kDOBytes + 2 * kLT * 4) + 1024 + 256;
};

template <int D, int DV>
__global__ void __launch_bounds__(320, 1)
    attn_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     const AttnParams p) {
  using SM = KVSmem<D, DV>;
  constexpr int NS = SM::kStages;
  constexpr int NB = SM::NB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + SM::kKBytes;
  uint8_t* sQ = sV + SM::kVBytes;        // [NS]
  uint8_t* sDO = sQ + NS * SM::kQBytes;  // [NS]
  float* sVec = reinterpret_cast<float*>(sDO + NS * SM::kDOBytes);  // [NS][lse 64 | delta 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sVec + NS * 2 * kLT);
  uint64_t* kv_full = bars;
  uint64_t* in_full = kv_full + 1;    // [NS]
  uint64_t* in_empty = in_full + NS;  // [NS]
  uint64_t* s_full = in_empty + NS;   // [2]
  uint64_t* p_ready = s_full + 2;     // [2]
  uint64_t* mm_done = p_ready + 2;
  uint64_t* acc_final = mm_done + 1;
  uint64_t* drain = acc_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int bhk = blockIdx.x % (p.B * p.Hkv);
  const int kt = blockIdx.x / (p.B * p.Hkv);  // key tile 0 (seen by the most queries) first
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int g = p.H / p.Hkv;
  const int k0 = kt * kTile;
  const int off = p.T - p.S;
  int qlo = 0, qhi = p.S - 1;
  if (p.causal) qlo = max(0, k0 - off);
  if (p.window >= 0) qhi = min(qhi, k0 + kTile - 1 + p.window - off);
  const int qt_lo = qlo / kLT;
  const int qt_hi = qhi < qlo ? qt_lo - 1 : qhi / kLT;
  const int nq = qt_hi >= qt_lo ? qt_hi - qt_lo + 1 : 0;
  const int n_steps = nq * g;  // (query head, 64-query tile) pairs
  const bool bulk_vec = (p.vec_s & 3) == 0;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 8);
    }
    mbar_init(mm_done, 1);
    mbar_init(acc_final, 1);
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
  const uint32_t tmem = *tmem_slot;
  // cols: S^T buffers [0, 64 NB); dP^T buffers [64 NB, 128 NB); dV [128 NB, 128 NB + DV); dK after dV
  const uint32_t tPT = tmem + 64 * NB;  // dP^T buffers
  const uint32_t tdV = tmem + 128 * NB;
  const uint32_t tdK = tdV + DV;

  if (warp == 0 && lane == 0) {
    bool ok = true;
    mbar_arrive_expect_tx(kv_full, SM::kKBytes + SM::kVBytes);
    load_tile(sK, &tmK, kv_full, hk * D, k0, b, D);
    load_tile(sV, &tmV, kv_full, hk * DV, k0, b, DV);
    for (int i = 0; i < n_steps && ok; ++i) {
      const int st = i % NS;
      const uint32_t ph = static_cast<uint32_t>((i / NS) & 1);
      const int h = hk * g + i / nq;
      const int q0 = (qt_lo + i % nq) * kLT;
      if (!mbar_wait(&in_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; break; }
      float* vec = sVec + st * 2 * kLT;
      const long long row = (static_cast<long long>(b) * p.H + h) * p.S + q0;
      if (bulk_vec) {
        // 256-byte bulk copies; lse / delta carry 128 floats of tail padding and
        // entries past S belong to masked queries.
        mbar_arrive_expect_tx(&in_full[st], SM::kQBytes + SM::kDOBytes + 2 * kLT * 4);
        bulk_load(vec, p.lse + row, kLT * 4, &in_full[st]);
        bulk_load(vec + kLT, p.delta + row, kLT * 4, &in_full[st]);
      } else {
        for (int r = 0; r < kLT; ++r) {
          const bool in = q0 + r < p.S;
          vec[r] = in ? p.lse[row + r] : 0.f;
          vec[kLT + r] = in ? p.delta[row + r] : 0.f;
        }
        mbar_arrive_expect_tx(&in_full[st], SM::kQBytes + SM::kDOBytes);
      }
      load_tile(sQ + st * SM::kQBytes, &tmQ, &in_full[st], h * D, q0, b, D, kLChunk);
      load_tile(sDO + st * SM::kDOBytes, &tmDO, &in_full[st], h * DV, q0, b, DV, kLChunk);
    }
    if (!ok) mbar_wait(kv_full, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc_ss = make_idesc_bf16(128, kLT, false, false);  // [128 keys x 64 q]
    constexpr uint32_t idesc_dv = make_idesc_bf16(128, DV, false, true);   // [128 keys x DV]
    constexpr uint32_t idesc_dk = make_idesc_bf16(128, D, false, true);    // [128 keys x D]
    bool ok = mbar_wait(kv_full, 0, p.status, kTimeoutMma, abort_flag);
    tc_fence_after();
    const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
    auto issue_scores = [&](int i) -> bool {
      const int st = i % NS;
      if (!mbar_wait(&in_full[st], (i / NS) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      const uint32_t q_base = smem_u32(sQ + st * SM::kQBytes);
      const uint32_t do_base = smem_u32(sDO + st * SM::kDOBytes);
      const uint32_t tS = tmem + (i % NB) * kLT;
      const uint32_t tP = tPT + (i % NB) * kLT;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        umma_f16(tS, kmajor_desc(k_base, kk), kmajor_desc(q_base, kk, kLChunk), idesc_ss, kk > 0);
#pragma unroll
      for (int kk = 0; kk < DV / 16; ++kk)
        umma_f16(tP, kmajor_desc(v_base, kk), kmajor_desc(do_base, kk, kLChunk), idesc_ss, kk > 0);
      umma_commit(&s_full[i % NB]);
      return true;
    };
    if (ok && n_steps > 0) ok = issue_scores(0);
    for (int i = 0; i < n_steps && ok; ++i) {
      if (NB == 2 && i + 1 < n_steps && !(ok = issue_scores(i + 1))) break;
      if (!mbar_wait(&p_ready[i % NB], (i / NB) & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int st = i % NS;
      const uint32_t q_base = smem_u32(sQ + st * SM::kQBytes);
      const uint32_t do_base = smem_u32(sDO + st * SM::kDOBytes);
      const uint32_t tS = tmem + (i % NB) * kLT;
      const uint32_t tP = tPT + (i % NB) * kLT;
#pragma unroll
      for (int kk = 0; kk < kLT / 16; ++kk)
        umma_f16_tmem_a(tdV, tS + (kk >> 1) * 32 + (kk & 1) * 8, mnmajor_desc(do_base, kk, kLChunk), idesc_dv, (i | kk) != 0);
#pragma unroll
      for (int kk = 0; kk < kLT / 16; ++kk)
        umma_f16_tmem_a(tdK, tP + (kk >> 1) * 32 + (kk & 1) * 8, mnmajor_desc(q_base, kk, kLChunk), idesc_dk, (i | kk) != 0);
      umma_commit(&in_empty[st]);
      umma_commit(mm_done);
      // The buffer of step i is rewritten by the scores of step i + NB: wait for these reads.
      if (!mbar_wait(mm_done, i & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; break; }
      if (NB == 1 && i + 1 < n_steps && !(ok = issue_scores(i + 1))) break;
    }
    umma_commit(acc_final);
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // 8 compute warps: warp w owns TMEM lane quarter w % 4 (32 key rows) and one
    // 32-column half of each 64-query step (no row reductions are needed here).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int kr = quarter * 32 + lane;  // key row
    const int key = k0 + kr;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int c0 = half * 32;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int i = 0; i < n_steps; ++i) {
      const int st = i % NS;
      const int q0 = (qt_lo + i % nq) * kLT;
      // Acquire the lse / delta vectors (bulk copies or the producer's plain stores).
      if (!mbar_wait_warp(&in_full[st], (i / NS) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      if (!mbar_wait_warp(&s_full[i % NB], (i / NB) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = tmem + lane_off + (i % NB) * kLT;
      const uint32_t tP = tPT + lane_off + (i % NB) * kLT;
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(tS + c0, sv);
      tmem_ld_32x32b_x32(tP + c0, dv);
      const float4* lse4 = reinterpret_cast<const float4*>(sVec + st * 2 * kLT + c0);
      const float4* dl4 = reinterpret_cast<const float4*>(sVec + st * 2 * kLT + kLT + c0);
      float nl[32], dl[32];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float4 a = lse4[t], d = dl4[t];
        nl[4 * t] = -a.x * kLog2e;
        nl[4 * t + 1] = -a.y * kLog2e;
        nl[4 * t + 2] = -a.z * kLog2e;
        nl[4 * t + 3] = -a.w * kLog2e;
        dl[4 * t] = d.x;
        dl[4 * t + 1] = d.y;
        dl[4 * t + 2] = d.z;
        dl[4 * t + 3] = d.w;
      }
      tmem_wait_ld();
      const bool need_mask = (p.causal && k0 + kTile - 1 > off + q0 + c0) || (k0 + kTile > p.T) ||
                             (q0 + c0 + 32 > p.S) || (p.window >= 0 && k0 < off + q0 + c0 + 31 - p.window);
      uint32_t pk[16], dk[16];
      if (!need_mask) {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(sv[2 * t]), sl2, nl[2 * t]));
          const float p1 = fast_exp2(fmaf(__uint_as_float(sv[2 * t + 1]), sl2, nl[2 * t + 1]));
          pk[t] = pack_bf16x2(p0, p1);
          dk[t] = pack_bf16x2(p0 * (__uint_as_float(dv[2 * t]) - dl[2 * t]),
                              p1 * (__uint_as_float(dv[2 * t + 1]) - dl[2 * t + 1]));
        }
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          float pr[2], ds[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int qi = 2 * t + e;
            // Masked entries are exactly zero even when padded lse / delta hold garbage.
            const bool vis = visible(p, q0 + c0 + qi, key);
            const float pv = vis ? fast_exp2(fmaf(__uint_as_float(sv[qi]), sl2, nl[qi])) : 0.f;
            pr[e] = pv;
            ds[e] = vis ? pv * (__uint_as_float(dv[qi]) - dl[qi]) : 0.f;
          }
          pk[t] = pack_bf16x2(pr[0], pr[1]);
          dk[t] = pack_bf16x2(ds[0], ds[1]);
        }
      }
      tmem_st_32x32b_x16(tS + c0, pk);  // inside this half's own S columns
      tmem_st_32x32b_x16(tP + c0, dk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[i % NB]);
    }
    if (ok && n_steps > 0) ok = mbar_wait_warp(acc_final, 0, p.status, kTimeoutEpilogue, abort_flag);
    tc_fence_after();
    // TMEM loads are warp-collective: every lane executes them; only stores are predicated.
    const bool row_ok = key < p.T;
    const long long krow = row_ok ? key : 0;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      __nv_bfloat16* dst = which == 0
                               ? static_cast<__nv_bfloat16*>(p.dv) + b * p.dv_sb + krow * p.dv_ss + hk * p.dv_sh
                               : static_cast<__nv_bfloat16*>(p.dk) + b * p.dk_sb + krow * p.dk_ss + hk * p.dk_sh;
      const uint32_t src = (which == 0 ? tdV : tdK) + lane_off;
      const float f = which == 0 ? 1.f : p.scale;
      const int width = which == 0 ? DV : D;
#pragma unroll
      for (int cc = 0; cc < (D > DV ? D : DV) / 64; ++cc) {
        if (cc >= width / 64) break;
        const int c = half * (width / 2) + cc * 32;
        uint32_t v[32];
        if (ok && n_steps > 0) {
          tmem_ld_32x32b_x32(src + c, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) v[t] = 0u;
        }
        if (row_ok) {
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) pk[t] = pack_bf16x2(__uint_as_float(v[2 * t]) * f, __uint_as_float(v[2 * t + 1]) * f);
          uint4* o4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int t = 0; t < 4; ++t) o4[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ dQ
template <int D, int DV>
struct QSmem {
  static constexpr int kStages = 3;
  static constexpr int kQBytes = (D / 64) * kChunkBytes;    // [128 q][D]
  static constexpr int kDOBytes = (DV / 64) * kChunkBytes;  // [128 q][DV]
  static constexpr int kKBytes = (D / 64) * kLChunk;        // [64 keys][D]
  static constexpr int kVBytes = (DV / 64) * kLChunk;       // [64 keys][DV]
  static constexpr int kBytes = kQBytes + kDOBytes + kStages * (kKBytes + kVBytes) + 1024 + 256;
};

template <int D, int DV>
__global__ void __launch_bounds__(320, 1)
    attn_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const AttnParams p) {
  using SM = QSmem<D, DV>;
  constexpr int NS = SM::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + SM::kQBytes;
  uint8_t* sK = sDO + SM::kDOBytes;     // [NS]
  uint8_t* sV = sK + NS * SM::kKBytes;  // [NS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NS * SM::kVBytes);
  uint64_t* qd_full = bars;
  uint64_t* kv_full = qd_full + 1;    // [NS]
  uint64_t* kv_empty = kv_full + NS;  // [NS]
  uint64_t* s_full = kv_empty + NS;   // [2]
  uint64_t* p_ready = s_full + 2;     // [2]
  uint64_t* mm_done = p_ready + 2;
  uint64_t* acc_final = mm_done + 1;
  uint64_t* drain = acc_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int num_q = (p.S + kTile - 1) / kTile;
  const int bh = blockIdx.x % (p.B * p.H);
  const int qt = num_q - 1 - blockIdx.x / (p.B * p.H);
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int q0 = qt * kTile;
  int klo, khi;
  key_range(p, q0, kTile, klo, khi);
  const int kt_lo = klo / kLT;
  const int kt_hi = khi < klo ? kt_lo - 1 : khi / kLT;
  const int n_tiles = kt_hi - kt_lo + 1;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 8);
    }
    mbar_init(mm_done, 1);
    mbar_init(acc_final, 1);
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
  const uint32_t tmem = *tmem_slot;
  // cols: S buffers [0,64) [64,128); dP buffers [128,192) [192,256); dQ [256, 256 + D)
  const uint32_t tdQ = tmem + 256;

  if (warp == 0 && lane == 0) {
    bool ok = true;
    mbar_arrive_expect_tx(qd_full, SM::kQBytes + SM::kDOBytes);
    load_tile(sQ, &tmQ, qd_full, h * D, q0, b, D);
    load_tile(sDO, &tmDO, qd_full, h * DV, q0, b, DV);
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j % NS;
      const int k0 = (kt_lo + j) * kLT;
      if (!mbar_wait(&kv_empty[st], ((j / NS) & 1) ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; break; }
      mbar_arrive_expect_tx(&kv_full[st], SM::kKBytes + SM::kVBytes);
      load_tile(sK + st * SM::kKBytes, &tmK, &kv_full[st], hk * D, k0, b, D, kLChunk);
      load_tile(sV + st * SM::kVBytes, &tmV, &kv_full[st], hk * DV, k0, b, DV, kLChunk);
    }
    if (!ok) mbar_wait(qd_full, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc_ss = make_idesc_bf16(128, kLT, false, false);
    constexpr uint32_t idesc_dq = make_idesc_bf16(128, D, false, true);
    bool ok = mbar_wait(qd_full, 0, p.status, kTimeoutMma, abort_flag);
    tc_fence_after();
    const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sDO);
    auto issue_scores = [&](int j) -> bool {
      const int st = j % NS;
      if (!mbar_wait(&kv_full[st], (j / NS) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      const uint32_t k_base = smem_u32(sK + st * SM::kKBytes);
      const uint32_t v_base = smem_u32(sV + st * SM::kVBytes);
      const uint32_t tS = tmem + (j & 1) * kLT;
      const uint32_t tP = tmem + 128 + (j & 1) * kLT;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        umma_f16(tS, kmajor_desc(q_base, kk), kmajor_desc(k_base, kk, kLChunk), idesc_ss, kk > 0);
#pragma unroll
      for (int kk = 0; kk < DV / 16; ++kk)
        umma_f16(tP, kmajor_desc(do_base, kk), kmajor_desc(v_base, kk, kLChunk), idesc_ss, kk > 0);
      umma_commit(&s_full[j & 1]);
      return true;
    };
    if (ok && n_tiles > 0) ok = issue_scores(0);
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (j + 1 < n_tiles && !(ok = issue_scores(j + 1))) break;
      if (!mbar_wait(&p_ready[j & 1], (j >> 1) & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int st = j % NS;
      const uint32_t k_base = smem_u32(sK + st * SM::kKBytes);
      const uint32_t tS = tmem + (j & 1) * kLT;
#pragma unroll
      for (int kk = 0; kk < kLT / 16; ++kk)
        umma_f16_tmem_a(tdQ, tS + (kk >> 1) * 32 + (kk & 1) * 8, mnmajor_desc(k_base, kk, kLChunk), idesc_dq, (j | kk) != 0);
      umma_commit(&kv_empty[st]);
      umma_commit(mm_done);
      if (!mbar_wait(mm_done, j & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; break; }
    }
    umma_commit(acc_final);
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // 8 compute warps: lane quarter w % 4 (32 query rows), one 32-key half per tile.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int c0 = half * 32;
    const long long vidx = (static_cast<long long>(b) * p.H + h) * p.S + q;
    const float neg_lse2 = q < p.S ? -p.lse[vidx] * kLog2e : 0.f;
    const float dl = q < p.S ? p.delta[vidx] : 0.f;
    const float sl2 = p.scale_log2;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int k0 = (kt_lo + j) * kLT + c0;  // first key of this warp's half
      if (!mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = tmem + lane_off + (j & 1) * kLT;
      const uint32_t tP = tmem + lane_off + 128 + (j & 1) * kLT;
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(tS + c0, sv);
      tmem_ld_32x32b_x32(tP + c0, dv);
      tmem_wait_ld();
      const bool need_mask = (p.causal && k0 + 31 > p.T - p.S + q0) || (k0 + 32 > p.T) ||
                             (p.window >= 0 && k0 < p.T - p.S + q0 + kTile - 1 - p.window) || (q0 + kTile > p.S);
      uint32_t dk[16];
      if (!need_mask) {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(sv[2 * t]), sl2, neg_lse2));
          const float p1 = fast_exp2(fmaf(__uint_as_float(sv[2 * t + 1]), sl2, neg_lse2));
          dk[t] = pack_bf16x2(p0 * (__uint_as_float(dv[2 * t]) - dl), p1 * (__uint_as_float(dv[2 * t + 1]) - dl));
        }
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          float ds[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int ki = 2 * t + e;
            const bool vis = visible(p, q, k0 + ki);
            const float pv = fast_exp2(fmaf(__uint_as_float(sv[ki]), sl2, neg_lse2));
            ds[e] = vis ? pv * (__uint_as_float(dv[ki]) - dl) : 0.f;
          }
          dk[t] = pack_bf16x2(ds[0], ds[1]);
        }
      }
      tmem_st_32x32b_x16(tS + c0, dk);  // inside this half's own S columns
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[j & 1]);
    }
    if (ok && n_tiles > 0) ok = mbar_wait_warp(acc_final, 0, p.status, kTimeoutEpilogue, abort_flag);
    tc_fence_after();
    __nv_bfloat16* dqr = static_cast<__nv_bfloat16*>(p.dq) + b * p.dq_sb + static_cast<long long>(q) * p.dq_ss + h * p.dq_sh;
#pragma unroll
    for (int cc = 0; cc < D / 64; ++cc) {
      const int c = half * (D / 2) + cc * 32;
      uint32_t v[32];
      if (ok && n_tiles > 0) {
        tmem_ld_32x32b_x32(tdQ + lane_off + c, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int t = 0; t < 32; ++t) v[t] = 0u;
      }
      if (q < p.S) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t)
          pk[t] = pack_bf16x2(__uint_as_float(v[2 * t]) * p.scale, __uint_as_float(v[2 * t + 1]) * p.scale);
        uint4* o4 = reinterpret_cast<uint4*>(dqr + c);
#pragma unroll
        for (int t = 0; t < 4; ++t) o4[t] = make_uint4(pk[4 * t], pk[4 * t + 1], pk[4 * t + 2], pk[4 * t + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}


// dq[b, s, h, :] = bf16(scale * dq_acc[b, h, s, :]), 8 elements per thread.
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int B, int S,
                                       int H, int D, long long dq_sb, long long dq_ss, float scale) {
  const long long n8 = static_cast<long long>(B) * H * S * D / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 8;
    const int d = static_cast<int>(e % D);
    const long long r = e / D;  // (b * H + h) * S + s
    const int s = static_cast<int>(r % S);
    const long long bh = r / S;
    const int h = static_cast<int>(bh % H);
    const int b = static_cast<int>(bh / H);
    const float4 a = reinterpret_cast<const float4*>(acc + e)[0];
    const float4 c = reinterpret_cast<const float4*>(acc + e)[1];
    uint4 o;
    o.x = pack_bf16x2(a.x * scale, a.y * scale);
    o.y = pack_bf16x2(a.z * scale, a.w * scale);
    o.z = pack_bf16x2(c.x * scale, c.y * scale);
    o.w = pack_bf16x2(c.z * scale, c.w * scale);
    *reinterpret_cast<uint4*>(dq + b * dq_sb + s * dq_ss + static_cast<long long>(h) * D + d) = o;
  }
}
}  // namespace

void attn_bwd(const AttnTensor& q, const AttnTensor& k, const AttnTensor& v, const AttnTensor& o,
              const AttnTensor& dout, const float* lse, float* delta, const AttnTensor& dq, const AttnTensor& dk,
              const AttnTensor& dv, int H, int Hkv, int D, float scale, bool causal, int window, int* status,
              cudaStream_t stream, float* dq_acc, int Dv) {
  if (Dv <= 0) Dv = D;
  AttnParams p{};
  p.B = q.batch;
  p.S = q.seq;
  p.T = k.seq;
  p.H = H;
  p.Hkv = Hkv;
  p.D = D;
  p.Dv = Dv;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.window = window;
  p.o = o.ptr;
  p.o_sb = o.s_batch;
  p.o_ss = o.s_seq;
  p.o_sh = Dv;
  p.lse = const_cast<float*>(lse);
  p.delta = delta;
  p.dout = dout.ptr;
  p.do_sb = dout.s_batch;
  p.do_ss = dout.s_seq;
  p.do_sh = Dv;
  p.dq = dq.ptr;
  p.dq_sb = dq.s_batch;
  p.dq_ss = dq.s_seq;
  p.dq_sh = D;
  p.dk = dk.ptr;
  p.dv = dv.ptr;
  p.dk_sb = dk.s_batch;
  p.dk_ss = dk.s_seq;
  p.dk_sh = D;
  p.dv_sb = dv.s_batch;
  p.dv_ss = dv.s_seq;
  p.dv_sh = Dv;
  p.status = status;
  const bool fused = D == 64 && Dv == 64 && dq_acc != nullptr;
  {
    const long long rows = static_cast<long long>(p.B) * p.S * p.H;
    // The fused kernel reads delta and -lse * log2(e) in 128-row bulk copies, so their rows are
    // padded to a multiple of 4 floats (16 bytes); delta holds 2 * (B * H * vec_s + 128) floats,
    // zeroed when padding rows exist so that the padded queries read finite values.
    p.vec_s = fused ? (p.S + 3) / 4 * 4 : p.S;
    const long long n_vec = static_cast<long long>(p.B) * p.H * p.vec_s;
    p.nlse2 = fused ? delta + n_vec + 128 : nullptr;
    if (fused && p.vec_s != p.S) cudaMemsetAsync(delta, 0, 2 * (n_vec + 128) * sizeof(float), stream);
    const long long threads = rows * (Dv / 8);
    attn_delta_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(p);
  }
  CUtensorMap mq128, mdo128, mq64, mdo64, mk128, mv128, mk64, mv64;
  make_bshd_map(&mq128, q, H, D, kTile);
  make_bshd_map(&mdo128, dout, H, Dv, kTile);
  make_bshd_map(&mq64, q, H, D, kLT);
  make_bshd_map(&mdo64, dout, H, Dv, kLT);
  make_bshd_map(&mk128, k, Hkv, D, kTile);
  make_bshd_map(&mv128, v, Hkv, Dv, kTile);
  make_bshd_map(&mk64, k, Hkv, D, kLT);
  make_bshd_map(&mv64, v, Hkv, Dv, kLT);
  const int grid_kv = ((p.T + kTile - 1) / kTile) * p.B * p.Hkv;
  const int grid_q = ((p.S + kTile - 1) / kTile) * p.B * p.H;
  if (fused) {
    const long long n_acc = static_cast<long long>(p.B) * p.H * p.S * D;
    cudaMemsetAsync(dq_acc, 0, n_acc * sizeof(float), stream);
    CUtensorMap mdq;
    make_tmap_2d_f32_sw128(&mdq, dq_acc, D, static_cast<long long>(p.B) * p.H * p.S, D, 32, 32);
    attn_bwd_d64_launch(mq128, mk128, mv128, mdo128, mdq, p, grid_kv, stream);
    const long long n8 = n_acc / 8;
    const int blocks = static_cast<int>(std::min<long long>((n8 + 255) / 256, 148LL * 16));
    attn_dq_convert_kernel<<<blocks, 256, 0, stream>>>(dq_acc, static_cast<__nv_bfloat16*>(p.dq), p.B, p.S, p.H, D,
                                                       p.dq_sb, p.dq_ss, scale);
    return;
  }
  auto run = [&](auto dkdv, int kv_bytes, auto dqk, int q_bytes) {
    set_smem(dkdv, kv_bytes);
    set_smem(dqk, q_bytes);
    dkdv<<<grid_kv, 320, kv_bytes, stream>>>(mq64, mk128, mv128, mdo64, p);
    dqk<<<grid_q, 320, q_bytes, stream>>>(mq128, mk64, mv64, mdo128, p);
  };
  if (D == 64 && Dv == 64) {
    run(attn_dkdv_kernel<64, 64>, KVSmem<64, 64>::kBytes, attn_dq_kernel<64, 64>, QSmem<64, 64>::kBytes);
  } else if (D == 128 && Dv == 128) {
    run(attn_dkdv_kernel<128, 128>, KVSmem<128, 128>::kBytes, attn_dq_kernel<128, 128>, QSmem<128, 128>::kBytes);
  } else {  // multi-head latent attention: 128 + 64 rotary query / key channels, 128 value channels
    run(attn_dkdv_kernel<192, 128>, KVSmem<192, 128>::kBytes, attn_dq_kernel<192, 128>, QSmem<192, 128>::kBytes);
  }
}

}  // namespace pb

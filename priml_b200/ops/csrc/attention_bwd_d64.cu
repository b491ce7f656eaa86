// Flash-attention backward for head dim 64 on sm_100a: one kernel computes
// dK, dV and (through an fp32 accumulator in global memory) dQ.
//
// One CTA per (batch, KV head, 128-key tile); it walks every (query head of the
// group, 128-query tile) pair -- a "step" -- and keeps dK and dV in TMEM.
//
// Per step, with Kt = this CTA's keys, Qi / dOi the step's queries:
//   MMA A(i):   S^T  = Kt Qi^T   and   dP^T = Vt dOi^T      (M 128 keys, N 128 queries,
//               K = 64; K and V are A operands read from TMEM)
//   softmax(i): P^T  = exp2(S^T * scale*log2e - lse*log2e)
//               dS^T = P^T * (dP^T - delta), both packed to bf16 in shared memory
//   MMA B(i):   dV += P^T dOi,  dK += dS^T Qi     (N 64, K 128 queries)
//               dQi = dS Kt                        (A = dS^T read M-major from shared memory)
//   dQ(i):      the softmax warps move dQi from TMEM to shared memory and reduce-add it
//               (bulk tensor reduce, fp32, performed in L2) into dq_acc [B, H, S, 64];
//               a later kernel scales and converts it.
//
// The softmax warps release the S^T / dP^T TMEM columns as soon as they have
// loaded them, so the MMA warp queues A(i+1) while the tensor cores still run
// B(i-1) and the softmax works on step i (issue order A(0), then A(i+1), B(i)).
//
// TMEM columns: S^T [0,128) dP^T [128,256) dV [256,320) dK [320,384)
//               dQ [384,448) K [448,480) V [480,512) (K, V as bf16 pairs).
// Warps: 0 TMA producer, 1 MMA issuer, 2-17 softmax, 18-21 dQ flush.
//   Softmax warp w covers TMEM lane quarter (w & 3) -- 32 keys -- and query quarter
//   (w - 2) >> 2 -- 32 queries -- of a step: sixteen warps keep enough work in flight
//   to hide the latency of the TMEM loads, the exponentials and the shared-memory
//   stores; the score arithmetic runs on packed fp32 pairs (f32x2).
//   dQ warp w moves the 32 query rows of lane quarter (w & 3) out of TMEM, so that
//   work never sits on the softmax warps' path.
#include "attention_common.cuh"

namespace pb {

namespace {

using namespace attn;

constexpr int kSoftmaxWarps = 16;
constexpr int kDqWarps = 4;
constexpr int kThreads = 32 * (2 + kSoftmaxWarps + kDqWarps);

struct BwdD64Smem {
  static constexpr int kStages = 3;
  static constexpr int kTileBytes = kChunkBytes;           // [128 rows][64 bf16], 128B-swizzled
  static constexpr int kPairBytes = 2 * kChunkBytes;       // [128 keys][128 queries] as two 64-query chunks
  static constexpr int kDQWarpBytes = 2 * 32 * 128;        // [32 queries][64 fp32] as two 128B-swizzled boxes
  static constexpr int kVecBytes = 2 * kTile * 4;          // -lse*log2e and delta of 128 queries
  static constexpr int kOffK = 0;
  static constexpr int kOffQ = kOffK + kTileBytes;
  static constexpr int kOffDO = kOffQ + kStages * kTileBytes;
  static constexpr int kOffPT = kOffDO + kStages * kTileBytes;  // also stages V before it moves to TMEM
  static constexpr int kOffDST = kOffPT + kPairBytes;
  static constexpr int kOffDQ = kOffDST + kPairBytes;
  static constexpr int kOffVec = kOffDQ + kDqWarps * kDQWarpBytes;
  static constexpr int kOffBars = kOffVec + kStages * kVecBytes;
  static constexpr int kBytes = kOffBars + 256 + 1024;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_d64_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmDQ, const AttnParams p) {
  constexpr int D = 64;
  using SM = BwdD64Smem;
  constexpr int NS = SM::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + SM::kOffK;
  uint8_t* sQ = smem + SM::kOffQ;
  uint8_t* sDO = smem + SM::kOffDO;
  uint8_t* sPT = smem + SM::kOffPT;
  uint8_t* sV = sPT;
  uint8_t* sDST = smem + SM::kOffDST;
  uint8_t* sDQ = smem + SM::kOffDQ;
  float* sVec = reinterpret_cast<float*>(smem + SM::kOffVec);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kOffBars);
  uint64_t* kv_full = bars;
  uint64_t* kv_tmem = bars + 1;
  uint64_t* in_full = bars + 2;        // [NS]
  uint64_t* in_empty = in_full + NS;   // [NS]
  uint64_t* s_full = in_empty + NS;
  uint64_t* st_free = s_full + 1;
  uint64_t* ds_ready = st_free + 1;
  uint64_t* ds_free = ds_ready + 1;
  uint64_t* dq_full = ds_free + 1;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* acc_final = dq_free + 1;
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
  const int qt_lo = qlo / kTile;
  const int qt_hi = qhi < qlo ? qt_lo - 1 : qhi / kTile;
  const int nq = qt_hi >= qt_lo ? qt_hi - qt_lo + 1 : 0;
  const int n_steps = nq * g;  // (query head, 128-query tile) pairs
  const bool bulk_vec = (p.vec_s & 3) == 0;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_tmem, kSoftmaxWarps);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(st_free, kSoftmaxWarps);
    mbar_init(ds_ready, kSoftmaxWarps);
    mbar_init(ds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kDqWarps);
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
  const uint32_t tS = tmem, tP = tmem + 128;
  const uint32_t tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384;
  const uint32_t tK = tmem + 448, tV = tmem + 480;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ producer
    bool ok = true;
    mbar_arrive_expect_tx(kv_full, 2 * SM::kTileBytes);
    load_tile(sK, &tmK, kv_full, hk * D, k0, b, D);
    load_tile(sV, &tmV, kv_full, hk * D, k0, b, D);
    for (int i = 0; i < n_steps && ok; ++i) {
      const int st = i % NS;
      const uint32_t ph = static_cast<uint32_t>((i / NS) & 1);
      const int h = hk * g + i / nq;
      const int q0 = (qt_lo + i % nq) * kTile;
      if (!mbar_wait(&in_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; break; }
      float* vec = sVec + st * 2 * kTile;
      const long long row = (static_cast<long long>(b) * p.H + h) * p.vec_s + q0;
      if (bulk_vec) {
        mbar_arrive_expect_tx(&in_full[st], 2 * SM::kTileBytes + SM::kVecBytes);
        bulk_load(vec, p.nlse2 + row, kTile * 4, &in_full[st]);
        bulk_load(vec + kTile, p.delta + row, kTile * 4, &in_full[st]);
      } else {
        for (int r = 0; r < kTile; ++r) {
          const bool in = q0 + r < p.S;
          vec[r] = in ? p.nlse2[row + r] : 0.f;
          vec[kTile + r] = in ? p.delta[row + r] : 0.f;
        }
        mbar_arrive_expect_tx(&in_full[st], 2 * SM::kTileBytes);
      }
      load_tile(sQ + st * SM::kTileBytes, &tmQ, &in_full[st], h * D, q0, b, D);
      load_tile(sDO + st * SM::kTileBytes, &tmDO, &in_full[st], h * D, q0, b, D);
    }
    if (!ok) mbar_wait(kv_full, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);   // [128 keys x 128 q]
    constexpr uint32_t idesc_acc = make_idesc_bf16(128, D, false, true);    // [128 keys x 64 d]
    constexpr uint32_t idesc_dq = make_idesc_bf16(128, D, true, true);      // [128 q x 64 d]
    bool ok = mbar_wait(kv_full, 0, p.status, kTimeoutMma, abort_flag) &&
              mbar_wait(kv_tmem, 0, p.status, kTimeoutMma, abort_flag);
    tc_fence_after();
    const uint32_t k_base = smem_u32(sK);
    const uint32_t pt_base = smem_u32(sPT), dst_base = smem_u32(sDST);
    auto issue_scores = [&](int i) -> bool {
      const int st = i % NS;
      if (!mbar_wait(&in_full[st], (i / NS) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      // the softmax warps have loaded S^T / dP^T of step i-1 out of TMEM
      if (i > 0 && !mbar_wait(st_free, (i - 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      const uint32_t q_base = smem_u32(sQ + st * SM::kTileBytes);
      const uint32_t do_base = smem_u32(sDO + st * SM::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        umma_f16_tmem_a(tS, tK + kk * 8, kmajor_desc(q_base, kk), idesc_s, kk > 0);
        umma_f16_tmem_a(tP, tV + kk * 8, kmajor_desc(do_base, kk), idesc_s, kk > 0);
      }
      umma_commit(s_full);
      return true;
    };
    auto issue_grads = [&](int i) -> bool {
      const int st = i % NS;
      if (!mbar_wait(ds_ready, i & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      const uint32_t q_base = smem_u32(sQ + st * SM::kTileBytes);
      const uint32_t do_base = smem_u32(sDO + st * SM::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        umma_f16(tdV, kmajor_desc(pt_base, kk), mnmajor_desc(do_base, kk), idesc_acc, (i | kk) != 0);
        umma_f16(tdK, kmajor_desc(dst_base, kk), mnmajor_desc(q_base, kk), idesc_acc, (i | kk) != 0);
      }
      // dQ of step i-1 must have left TMEM before dQ of step i overwrites it
      if (i > 0 && !mbar_wait(dq_free, (i - 1) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk)
        umma_f16(tdQ, mnmajor_desc(dst_base, kk), mnmajor_desc(k_base, kk), idesc_dq, kk > 0);
      umma_commit(&in_empty[st]);
      umma_commit(ds_free);
      umma_commit(dq_full);
      return true;
    };
    if (ok && n_steps > 0) ok = issue_scores(0);
    for (int i = 0; i < n_steps && ok; ++i) {
      if (i + 1 < n_steps && !(ok = issue_scores(i + 1))) break;
      ok = issue_grads(i);
    }
    umma_commit(acc_final);
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2 + kSoftmaxWarps) {
    // ------------------------------------------------------------------ dQ flush
    // Query rows 32 quarter .. of dQ_j, all 64 columns: TMEM -> two 128B-swizzled staging boxes
    // [32 rows][32 fp32] -> bulk tensor reduce-add (fp32, in L2) into dq_acc.
    const int quarter = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* stage = sDQ + (warp - 2 - kSoftmaxWarps) * SM::kDQWarpBytes;
    int h = hk * g, qt = qt_lo;  // (query head, query tile) of step j, advanced without divisions
    bool ok = true;
    for (int j = 0; j < n_steps && ok; ++j) {
      if (!mbar_wait_warp(dq_full, j & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) tma_store_wait_read();  // the previous reduces no longer read the staging rows
      __syncwarp();
#pragma unroll
      for (int box = 0; box < 2; ++box) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tdQ + lane_off + 32 * box, v);
        tmem_wait_ld();
        if (box == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dq_free);
        }
        uint8_t* row = stage + box * (32 * 128) + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(row + ((c ^ (lane & 7)) << 4)) =
              make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int y = static_cast<int>((static_cast<long long>(b) * p.H + h) * p.S + qt * kTile + quarter * 32);
        tma_reduce_add_2d(&tmDQ, stage, 0, y);
        tma_reduce_add_2d(&tmDQ, stage + 32 * 128, 32, y);
        tma_store_commit();
      }
      if (++qt > qt_hi) {
        qt = qt_lo;
        ++h;
      }
    }
    if (lane == 0) tma_store_wait_all();
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ softmax, final epilogue
    const int quarter = warp & 3;          // TMEM lanes: keys of S^T, dP^T, dK, dV
    const int part = (warp - 2) >> 2;      // 32-query slice of a step
    const int kr = quarter * 32 + lane;    // key row of this thread
    const int key = k0 + kr;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint64_t sl2x2 = f2_pack(p.scale_log2, p.scale_log2);
    bool ok = mbar_wait_warp(kv_full, 0, p.status, kTimeoutEpilogue, abort_flag);
    if (ok && part < 2) {
      // Key row kr of K (part 0) or V (part 1) into TMEM: eight swizzled 16-byte chunks -> 32 columns.
      const uint8_t* src = (part == 0 ? sK : sV) + kr * 128;
      uint32_t w[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 x = *reinterpret_cast<const uint4*>(src + ((c ^ (kr & 7)) << 4));
        w[4 * c] = x.x;
        w[4 * c + 1] = x.y;
        w[4 * c + 2] = x.z;
        w[4 * c + 3] = x.w;
      }
      tmem_st_32x32b_x32((part == 0 ? tK : tV) + lane_off, w);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(kv_tmem);

    uint8_t* prow = sPT + (part >> 1) * kChunkBytes + kr * 128;
    uint8_t* drow = sDST + (part >> 1) * kChunkBytes + kr * 128;
    const int piece0 = (part & 1) * 4;  // this warp's four 16-byte pieces of the 128-byte row
    int qt = qt_lo;                     // query tile of step i, advanced without divisions
    for (int i = 0; i < n_steps && ok; ++i) {
      const int st = i % NS;
      const int qa = qt * kTile + part * 32;  // first query of this warp's 32 columns
      if (++qt > qt_hi) qt = qt_lo;
      if (!mbar_wait_warp(&in_full[st], (i / NS) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      if (!mbar_wait_warp(s_full, i & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const ulonglong2* nl2 = reinterpret_cast<const ulonglong2*>(sVec + st * 2 * kTile + part * 32);
      const ulonglong2* dl2 = reinterpret_cast<const ulonglong2*>(sVec + st * 2 * kTile + kTile + part * 32);
      const bool need_mask = (p.causal && k0 + kTile - 1 > off + qa) || (k0 + kTile > p.T) || (qa + 32 > p.S) ||
                             (p.window >= 0 && k0 < off + qa + 31 - p.window);
      uint32_t pk[16], dk[16];
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {  // two 16-column passes keep the register footprint small
        uint32_t sv[16], dv[16];
        tmem_ld_32x32b_x16(tS + lane_off + part * 32 + pass * 16, sv);
        tmem_ld_32x32b_x16(tP + lane_off + part * 32 + pass * 16, dv);
        tmem_wait_ld();
        if (pass == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(st_free);  // the MMA warp may now write the next step's scores
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const ulonglong2 nl = nl2[pass * 4 + t], dl = dl2[pass * 4 + t];
          const uint64_t nls[2] = {nl.x, nl.y}, dls[2] = {dl.x, dl.y};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = 4 * t + 2 * e;           // within this pass
            const int qc = pass * 16 + col;          // within the warp's 32 queries
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[col]), __uint_as_float(sv[col + 1])), sl2x2, nls[e]), x0, x1);
            const uint64_t pr = f2_pack(fast_exp2(x0), fast_exp2(x1));
            const uint64_t d2 = f2_pack(__uint_as_float(dv[col]), __uint_as_float(dv[col + 1]));
            float p0, p1, g0, g1;
            f2_unpack(pr, p0, p1);
            f2_unpack(f2_mul(pr, f2_sub(d2, dls[e])), g0, g1);
            if (need_mask) {
              // diagonal, ragged or windowed tile: invisible entries are exact zeros (they may
              // read padding rows of the per-query vectors)
              const bool v0 = visible(p, qa + qc, key), v1 = visible(p, qa + qc + 1, key);
              p0 = v0 ? p0 : 0.f;
              g0 = v0 ? g0 : 0.f;
              p1 = v1 ? p1 : 0.f;
              g1 = v1 ? g1 : 0.f;
            }
            pk[qc >> 1] = pack_bf16x2(p0, p1);
            dk[qc >> 1] = pack_bf16x2(g0, g1);
          }
        }
      }
      // B(i-1) has finished reading the previous P^T / dS^T.
      if (i > 0 && !mbar_wait_warp(ds_free, (i - 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pos = ((piece0 + j) ^ (kr & 7)) << 4;
        *reinterpret_cast<uint4*>(prow + pos) = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4*>(drow + pos) = make_uint4(dk[4 * j], dk[4 * j + 1], dk[4 * j + 2], dk[4 * j + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
    }

    // dV (parts 0, 1) and dK scaled by the softmax scale (parts 2, 3): TMEM lanes = keys.
    if (ok && n_steps > 0) ok = mbar_wait_warp(acc_final, 0, p.status, kTimeoutEpilogue, abort_flag);
    tc_fence_after();
    const bool row_ok = key < p.T;
    const long long row_off = b * p.dk_sb + static_cast<long long>(row_ok ? key : 0) * p.dk_ss + hk * p.dk_sh;
    const bool is_dk = part >= 2;
    const int col = (part & 1) * 32;
    __nv_bfloat16* dst = (is_dk ? static_cast<__nv_bfloat16*>(p.dk) : static_cast<__nv_bfloat16*>(p.dv)) + row_off;
    const float f = is_dk ? p.scale : 1.f;
    uint32_t v[32];
    if (ok && n_steps > 0) {
      tmem_ld_32x32b_x32((is_dk ? tdK : tdV) + lane_off + col, v);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int t = 0; t < 32; ++t) v[t] = 0u;
    }
    if (row_ok) {
      uint32_t o[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) o[t] = pack_bf16x2(__uint_as_float(v[2 * t]) * f, __uint_as_float(v[2 * t + 1]) * f);
      uint4* o4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
      for (int t = 0; t < 4; ++t) o4[t] = make_uint4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
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

}  // namespace

namespace attn {

void attn_bwd_d64_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                         const CUtensorMap& mdq, const AttnParams& p, int grid, cudaStream_t stream) {
  set_smem(attn_bwd_d64_kernel, BwdD64Smem::kBytes);
  attn_bwd_d64_kernel<<<grid, kThreads, BwdD64Smem::kBytes, stream>>>(mq, mk, mv, mdo, mdq, p);
}

}  // namespace attn
}  // namespace pb

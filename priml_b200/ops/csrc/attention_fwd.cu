// Flash-attention forward for sm_100a: tcgen05 MMAs with TMEM accumulators,
// TMA-fed tiles, grouped KV heads read in place (no K/V expansion), causal and
// sliding-window masks, fp32 log-sum-exp output for the backward pass.
//
// Layouts: q/o [B, S, H, D], k/v [B, T, Hkv, D] (any token / batch strides,
// heads x D contiguous), lse [B, H, S] fp32. Causal masks are aligned
// bottom-right: query i (absolute position T - S + i) sees keys <= T - S + i; a
// window w additionally requires key >= position - w.
//
// One CTA per (b, h, 128-query tile), two CTAs per SM (256 TMEM columns each):
//   warp 0     TMA: Q once, then 64-key K / V tiles through a ring.
//   warp 1     MMA: S_j = Q K_j^T into one of two TMEM score buffers, so S_{j+1}
//              is computed while the softmax works on S_j; O += P_j V_j reads
//              P_j (bf16, written over S_j) straight from TMEM.
//   warps 2-5  softmax: one query row per thread (64 scores per tile), one FFMA
//              + ex2 per score, P packed to bf16 and stored back to TMEM. The
//              running max only moves (and O is rescaled) when it grows by more
//              than 2^8; epilogue divides by the row sum, writes bf16 O and the
//              natural-log LSE.
#include "attention_common.cuh"

namespace pb {

namespace {

using namespace attn;

constexpr int kKT = 64;                   // keys per tile
constexpr int kKChunk = kKT * 128;        // one [64 keys][64 d] swizzled chunk = 8 KB

template <int D>
struct Fwd2Smem {
  static constexpr int kStages = D == 64 ? 3 : 2;
  static constexpr int kQBytes = (D / 64) * kChunkBytes;
  static constexpr int kKVBytes = (D / 64) * kKChunk;
  static constexpr int kBytes = kQBytes + 2 * kStages * kKVBytes + 1024 + 256;
};

template <int D>
__global__ void __launch_bounds__(192, 2)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using SM = Fwd2Smem<D>;
  constexpr int NS = SM::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + SM::kQBytes;
  uint8_t* sV = sK + NS * SM::kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NS * SM::kKVBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2]
  uint64_t* p_ready = s_full + 2;   // [2]
  uint64_t* pv_done = p_ready + 2;
  uint64_t* o_final = pv_done + 1;
  uint64_t* drain = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int num_q = (p.S + kTile - 1) / kTile;
  const int bh = blockIdx.x % (p.B * p.H);
  const int qt = num_q - 1 - blockIdx.x / (p.B * p.H);  // heaviest (latest) query tiles first
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int q0 = qt * kTile;
  int klo, khi;
  key_range(p, q0, kTile, klo, khi);
  const int kt_lo = klo / kKT;
  const int kt_hi = khi < klo ? kt_lo - 1 : khi / kKT;
  const int n_tiles = kt_hi - kt_lo + 1;  // may be 0 for a fully masked query tile

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    trace_put(p, 0, 1);
    trace_put(p, 1, sm_id());
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 4);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) trace_put(p, 0, 2);
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 2 * kKT;  // S buffers at cols [0, 64) and [64, 128); O at [128, 128 + D)

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- producer
    bool ok = true;
    mbar_arrive_expect_tx(q_full, SM::kQBytes);
    load_tile(sQ, &tmQ, q_full, h * D, q0, b, D);
    int st = 0;
    uint32_t ph = 0;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int k0 = (kt_lo + j) * kKT;
      if (!mbar_wait(&k_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; trace_put(p, 5, 1000 + j); break; }
      mbar_arrive_expect_tx(&k_full[st], SM::kKVBytes);
      load_tile(sK + st * SM::kKVBytes, &tmK, &k_full[st], hk * D, k0, b, D, kKChunk);
      if (!mbar_wait(&v_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; trace_put(p, 5, 2000 + j); break; }
      mbar_arrive_expect_tx(&v_full[st], SM::kKVBytes);
      load_tile(sV + st * SM::kKVBytes, &tmV, &v_full[st], hk * D, k0, b, D, kKChunk);
      if (++st == NS) { st = 0; ph ^= 1u; }
      trace_put(p, 2, j + 1);
    }
    if (!ok) mbar_wait(q_full, 0, p.status, kTimeoutDrain, nullptr);
    trace_put(p, 2, 100 + (ok ? 1 : 0));
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc_s = make_idesc_bf16(128, kKT, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(128, D, false, true);
    bool ok = mbar_wait(q_full, 0, p.status, kTimeoutMma, abort_flag);
    tc_fence_after();
    const uint32_t q_base = smem_u32(sQ);
    auto issue_s = [&](int j) -> bool {
      const int st = j % NS;
      const uint32_t ph = static_cast<uint32_t>((j / NS) & 1);
      if (!mbar_wait(&k_full[st], ph, p.status, kTimeoutMma, abort_flag)) { trace_put(p, 6, 1000 + j); return false; }
      tc_fence_after();
      const uint32_t k_base = smem_u32(sK + st * SM::kKVBytes);
      const uint32_t tS = tmem + (j & 1) * kKT;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        umma_f16(tS, kmajor_desc(q_base, kk), kmajor_desc(k_base, kk, kKChunk), idesc_s, kk > 0);
      umma_commit(&k_empty[st]);
      umma_commit(&s_full[j & 1]);
      return true;
    };
    if (ok && n_tiles > 0) ok = issue_s(0);
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (j + 1 < n_tiles && !(ok = issue_s(j + 1))) break;
      if (!mbar_wait(&p_ready[j & 1], (j >> 1) & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; trace_put(p, 6, 2000 + j); break; }
      tc_fence_after();
      const int st = j % NS;
      if (!mbar_wait(&v_full[st], (j / NS) & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; trace_put(p, 6, 3000 + j); break; }
      tc_fence_after();
      const uint32_t v_base = smem_u32(sV + st * SM::kKVBytes);
      const uint32_t tP = tmem + (j & 1) * kKT;
#pragma unroll
      for (int kk = 0; kk < kKT / 16; ++kk)
        umma_f16_tmem_a(tO, tP + kk * 8, mnmajor_desc(v_base, kk, kKChunk), idesc_o, (j | kk) != 0);
      umma_commit(&v_empty[st]);
      umma_commit(pv_done);
      // P_j sits in score buffer j&1, which S_{j+2} overwrites next iteration.
      if (!mbar_wait(pv_done, j & 1, p.status, kTimeoutMma, abort_flag)) { ok = false; trace_put(p, 6, 4000 + j); break; }
      trace_put(p, 3, j + 1);
    }
    trace_put(p, 3, 100 + (ok ? 1 : 0));
    umma_commit(o_final);
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m = -INFINITY;  // running max of scaled scores (log2 units), possibly stale by < 2^8
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int k0 = (kt_lo + j) * kKT;
      if (!mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; if (lane == 0) trace_put(p, 7, 1000 + 100 * warp + j); break; }
      tc_fence_after();
      const uint32_t tS = tmem + lane_off + (j & 1) * kKT;
      uint32_t v[64];
      tmem_ld_32x32b_x32(tS, *reinterpret_cast<uint32_t(*)[32]>(v));
      tmem_ld_32x32b_x32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_wait_ld();
      const bool need_mask = (p.causal && k0 + kKT - 1 > p.T - p.S + q0) || (k0 + kKT > p.T) ||
                             (p.window >= 0 && k0 < p.T - p.S + q0 + kTile - 1 - p.window) || (q0 + kTile > p.S);
      float mx = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (!visible(p, q, k0 + i)) v[i] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(v[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; i += 2) mx = fmaxf(mx, fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 1])));
      }
      const float mxs = mx * sl2;  // scale > 0: max commutes with scaling
      // Rows move their running max independently, but rescaling O uses warp-collective
      // tcgen05.ld / st: the warp rescales together whenever any of its rows must, each
      // row by its own factor (1 for rows whose max did not move).
      const bool grow = mxs > m + kRescaleThreshold;
      const bool scale_o = grow && j > 0 && m != -INFINITY;
      if (__any_sync(0xffffffffu, scale_o)) {
        // O holds P V of earlier tiles: wait until the last of them landed.
        if (!mbar_wait_warp(pv_done, (j - 1) & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; if (lane == 0) trace_put(p, 7, 2000 + 100 * warp + j); break; }
        tc_fence_after();
        const float f = scale_o ? fast_exp2(m - mxs) : 1.f;
        l *= f;
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld_32x32b_x16(tO + lane_off + c * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st_32x32b_x16(tO + lane_off + c * 16, o);
        }
      }
      if (grow) m = mxs;
      const float neg_mu = m == -INFINITY ? 0.f : -m;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = fast_exp2(fmaf(__uint_as_float(v[c * 32 + 2 * i]), sl2, neg_mu));
          const float e1 = fast_exp2(fmaf(__uint_as_float(v[c * 32 + 2 * i + 1]), sl2, neg_mu));
          rs0 += e0;
          rs1 += e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        tmem_st_32x32b_x16(tS + c * 16, pk);
      }
      l += rs0 + rs1;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[j & 1]);
      if (threadIdx.x == 64) trace_put(p, 4, j + 1);
    }
    if (threadIdx.x == 64) trace_put(p, 4, 100 + (ok ? 1 : 0));
    if (ok && n_tiles > 0) ok = mbar_wait_warp(o_final, 0, p.status, kTimeoutEpilogue, abort_flag);
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.o) + b * p.o_sb + static_cast<long long>(q) * p.o_ss + h * p.o_sh;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t v[32];
      if (ok && n_tiles > 0) {
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      if (q < p.S) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(v[2 * i]) * inv, __uint_as_float(v[2 * i + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
    if (q < p.S) {
      const float lse = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      p.lse[(static_cast<long long>(b) * p.H + h) * p.S + q] = lse;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) trace_put(p, 0, 3);
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
    if (lane == 0) trace_put(p, 0, 4);
  }
}

}  // namespace

void attn_fwd(const AttnTensor& q, const AttnTensor& k, const AttnTensor& v, const AttnTensor& o, float* lse, int H,
              int Hkv, int D, float scale, bool causal, int window, int* status, cudaStream_t stream, int* trace,
              int Dv) {
  if (Dv <= 0) Dv = D;
  AttnParams p{};
  p.trace = trace;
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
  p.lse = lse;
  p.status = status;
  CUtensorMap mq, mk, mv;
  make_bshd_map(&mq, q, H, D, kTile);
  if (trace == nullptr || Dv != D) {
    const int kt = D == 128 ? kTile : kKT;  // keys per tile of the two-tile kernel
    make_bshd_map(&mk, k, Hkv, D, kt);
    make_bshd_map(&mv, v, Hkv, Dv, kt);
    attn_fwd3_launch(mq, mk, mv, p, D, stream);
    return;
  }
  make_bshd_map(&mk, k, Hkv, D, kKT);
  make_bshd_map(&mv, v, Hkv, D, kKT);
  const int grid = ((p.S + kTile - 1) / kTile) * p.B * p.H;
  if (D == 64) {
    set_smem(attn_fwd2_kernel<64>, Fwd2Smem<64>::kBytes);
    attn_fwd2_kernel<64><<<grid, 192, Fwd2Smem<64>::kBytes, stream>>>(mq, mk, mv, p);
  } else {
    set_smem(attn_fwd2_kernel<128>, Fwd2Smem<128>::kBytes);
    attn_fwd2_kernel<128><<<grid, 192, Fwd2Smem<128>::kBytes, stream>>>(mq, mk, mv, p);
  }
}

}  // namespace pb

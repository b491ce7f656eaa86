// Flash-attention forward for sm_100a, two query tiles per CTA. Query / key head dim D and value
// head dim DV: (64, 64), (128, 128), and (192, 128) for multi-head latent attention.
//
// Layouts as in attention_fwd.cu: q/o [B, S, H, D], k/v [B, T, Hkv, D] (token and
// batch strides free, heads x D contiguous), lse [B, H, S] fp32 natural log.
// Causal masks are aligned bottom-right; a window w also requires key >= pos - w.
//
// One CTA per (b, h, pair of 128-query tiles), heaviest pairs first. Head dim 64 uses
// 64-key tiles and 256 TMEM columns, so two CTAs share an SM and their softmax warps
// overlap; head dim 128 uses 128-key tiles and one CTA per SM.
//   warp 0     TMA: Q of both tiles once, then K and V tiles through a ring.
//   warp 1     MMA: for each key tile j, S_t(j) = Q_t K_j^T (N = keys per tile) for the
//              two query tiles t, and O_t += P_t(j) V_j with P_t read from TMEM. The
//              issue order S_0(0) S_1(0), then per j: PV_0(j) S_0(j+1) PV_1(j) S_1(j+1)
//              lets group 1's softmax of tile j run while the tensor cores work on
//              group 0's next scores, and the other way round.
//   warps 2-5  softmax of query tile 0; warps 6-9 of query tile 1 (one row per
//              thread, one score per key of the tile). P is packed to bf16 and written
//              over the first half of the tile's own S columns in TMEM: tcgen05.mma of one
//              CTA execute in issue order, so S_t(j+1) overwrites P_t(j) only after
//              PV_t(j) has read it. The running max moves (and O is rescaled) only
//              when it grows by more than 2^8; the epilogue divides by the row sum
//              and writes bf16 O and the natural-log LSE.
// TMEM: S_0 [0,KT) S_1 [KT,2KT) O_0 [2KT, 2KT + DV) O_1 [2KT + DV, 2KT + 2DV), KT keys per tile.
#include "attention_common.cuh"

namespace pb {

namespace {

using namespace attn;

template <int D, int DV>
struct Fwd3Cfg {
  static constexpr int KT = D == 128 ? 128 : 64;              // keys per tile
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kTmemCols = 2 * KT + 2 * DV <= 256 ? 256 : 512;
  static constexpr int kStages = D == 64 ? 4 : (D == 128 ? 2 : 3);
  static constexpr int kQBytes = (D / 64) * kChunkBytes;      // [128 rows][D] in 64-column chunks
  static constexpr int kKVChunk = KT * 128;                   // [KT rows][64 columns] swizzled chunk
  static constexpr int kKBytes = (D / 64) * kKVChunk;
  static constexpr int kVBytes = (DV / 64) * kKVChunk;
  static constexpr int kOffQ = 0;                             // two query tiles
  static constexpr int kOffK = 2 * kQBytes;
  static constexpr int kOffV = kOffK + kStages * kKBytes;
  static constexpr int kOffBars = kOffV + kStages * kVBytes;
  static constexpr int kBytes = kOffBars + 256 + 1024;
};

template <int D, int DV>
__global__ void __launch_bounds__(320, Fwd3Cfg<D, DV>::kCtasPerSm)
    attn_fwd3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using SM = Fwd3Cfg<D, DV>;
  constexpr int NS = SM::kStages;
  constexpr int KT = SM::KT;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + SM::kOffQ;
  uint8_t* sK = smem + SM::kOffK;
  uint8_t* sV = smem + SM::kOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kOffBars);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;         // [NS]
  uint64_t* k_empty = k_full + NS;     // [NS]
  uint64_t* v_full = k_empty + NS;     // [NS]
  uint64_t* v_empty = v_full + NS;     // [NS]
  uint64_t* s_full = v_empty + NS;     // [2] one per query tile
  uint64_t* p_ready = s_full + 2;      // [2]
  uint64_t* o_final = p_ready + 2;     // [2]
  uint64_t* drain = o_final + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int num_q = (p.S + kTile - 1) / kTile;
  const int num_pairs = (num_q + 1) / 2;
  const int bh = blockIdx.x % (p.B * p.H);
  const int pair = num_pairs - 1 - blockIdx.x / (p.B * p.H);  // heaviest (latest) query tiles first
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  // Key tiles [lo_t, hi_t] seen by query tile t (empty when hi_t < lo_t); the CTA walks their union.
  int lo[2], hi[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int q0 = (2 * pair + t) * kTile;
    if (q0 >= p.S) {
      lo[t] = 0;
      hi[t] = -1;
      continue;
    }
    int klo, khi;
    key_range(p, q0, kTile, klo, khi);
    lo[t] = klo / KT;
    hi[t] = khi < klo ? lo[t] - 1 : khi / KT;
  }
  const bool has0 = hi[0] >= lo[0], has1 = hi[1] >= lo[1];
  const int j_lo = has0 && has1 ? min(lo[0], lo[1]) : (has0 ? lo[0] : lo[1]);
  const int j_hi = has0 && has1 ? max(hi[0], hi[1]) : (has0 ? hi[0] : hi[1]);
  const int n_tiles = (has0 || has1) ? j_hi - j_lo + 1 : 0;

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&o_final[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, SM::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------ producer
    bool ok = true;
    const uint32_t q_bytes = (has0 ? SM::kQBytes : 0) + (has1 ? SM::kQBytes : 0);
    mbar_arrive_expect_tx(q_full, q_bytes);
    if (has0) load_tile(sQ, &tmQ, q_full, h * D, (2 * pair) * kTile, b, D);
    if (has1) load_tile(sQ + SM::kQBytes, &tmQ, q_full, h * D, (2 * pair + 1) * kTile, b, D);
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j % NS;
      const uint32_t ph = static_cast<uint32_t>((j / NS) & 1);
      const int k0 = (j_lo + j) * KT;
      if (!mbar_wait(&k_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; break; }
      mbar_arrive_expect_tx(&k_full[st], SM::kKBytes);
      load_tile(sK + st * SM::kKBytes, &tmK, &k_full[st], hk * D, k0, b, D, SM::kKVChunk);
      if (!mbar_wait(&v_empty[st], ph ^ 1u, p.status, kTimeoutProducer, abort_flag)) { ok = false; break; }
      mbar_arrive_expect_tx(&v_full[st], SM::kVBytes);
      load_tile(sV + st * SM::kVBytes, &tmV, &v_full[st], hk * DV, k0, b, DV, SM::kKVChunk);
    }
    if (!ok) mbar_wait(q_full, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16(128, KT, false, false);     // [128 q x KT keys]
    constexpr uint32_t idesc_o = make_idesc_bf16(128, DV, false, true);      // [128 q x DV]
    bool ok = mbar_wait(q_full, 0, p.status, kTimeoutMma, abort_flag);
    tc_fence_after();
    int done0 = 0, done1 = 0;  // key tiles already accumulated into O_0 / O_1
    auto active = [&](int t, int j) {
      const int kt = j_lo + j;
      return t == 0 ? (lo[0] <= kt && kt <= hi[0]) : (lo[1] <= kt && kt <= hi[1]);
    };
    auto issue_s = [&](int t, int j) -> bool {
      const int st = j % NS;
      if (!mbar_wait(&k_full[st], (j / NS) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      if (active(t, j)) {
        const uint32_t q_base = smem_u32(sQ + t * SM::kQBytes);
        const uint32_t k_base = smem_u32(sK + st * SM::kKBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tmem + t * KT, kmajor_desc(q_base, kk), kmajor_desc(k_base, kk, SM::kKVChunk), idesc_s, kk > 0);
        umma_commit(&s_full[t]);
      }
      return true;
    };
    auto issue_pv = [&](int t, int j) -> bool {
      if (!active(t, j)) return true;
      int& done = t == 0 ? done0 : done1;
      if (!mbar_wait(&p_ready[t], done & 1, p.status, kTimeoutMma, abort_flag)) return false;
      const int st = j % NS;
      if (!mbar_wait(&v_full[st], (j / NS) & 1, p.status, kTimeoutMma, abort_flag)) return false;
      tc_fence_after();
      const uint32_t v_base = smem_u32(sV + st * SM::kVBytes);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)
        umma_f16_tmem_a(tmem + 2 * KT + t * DV, tmem + t * KT + kk * 8, mnmajor_desc(v_base, kk, SM::kKVChunk), idesc_o,
                        (done | kk) != 0);
      ++done;
      return true;
    };
    if (ok && n_tiles > 0) ok = issue_s(0, 0) && issue_s(1, 0);
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j % NS;
      if (!(ok = issue_pv(0, j))) break;
      if (j + 1 < n_tiles && !(ok = issue_s(0, j + 1))) break;
      if (!(ok = issue_pv(1, j))) break;
      umma_commit(&v_empty[st]);
      umma_commit(&k_empty[st]);  // both S of tile j were issued before PV_1(j)
      if (j + 1 < n_tiles && !(ok = issue_s(1, j + 1))) break;
    }
    umma_commit(&o_final[0]);
    umma_commit(&o_final[1]);
    umma_commit(drain);
    mbar_wait(drain, 0, p.status, kTimeoutDrain, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 2) >> 2;  // query tile of this warp's group
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q0 = (2 * pair + t) * kTile;
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + t * KT + lane_off;
    const uint32_t tO = tmem + 2 * KT + t * DV + lane_off;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = f2_pack(sl2, sl2);
    const int my_lo = t == 0 ? lo[0] : lo[1], my_hi = t == 0 ? hi[0] : hi[1];
    const bool has = my_hi >= my_lo;
    float m = -INFINITY;  // running max of scaled scores (log2 units), possibly stale by < 2^8
    float l = 0.f;
    bool ok = true;
    int n = 0;  // key tiles processed by this group
    for (int kt = my_lo; has && kt <= my_hi && ok; ++kt, ++n) {
      const int k0 = kt * KT;
      if (!mbar_wait_warp_sleep(&s_full[t], n & 1, p.status, kTimeoutEpilogue, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[KT];
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) tmem_ld_32x32b_x32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
      tmem_wait_ld();
      const bool need_mask = (p.causal && k0 + KT - 1 > p.T - p.S + q0) || (k0 + KT > p.T) ||
                             (p.window >= 0 && k0 < p.T - p.S + q0 + kTile - 1 - p.window) || (q0 + kTile > p.S);
      float mx = -INFINITY;
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < KT; ++i) {
          if (!visible(p, q, k0 + i)) v[i] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(v[i]));
        }
      } else {
        float a = -INFINITY, c2 = -INFINITY;
#pragma unroll
        for (int i = 0; i < KT; i += 2) {
          a = fmaxf(a, __uint_as_float(v[i]));
          c2 = fmaxf(c2, __uint_as_float(v[i + 1]));
        }
        mx = fmaxf(a, c2);
      }
      const float mxs = mx * sl2;  // scale > 0: max commutes with scaling
      // O is rescaled with warp-collective tcgen05.ld / st: the warp rescales together when any
      // of its rows must, each row by its own factor (1 when its max did not move). s_full for
      // this tile implies the previous PV of this tile completed (commits cover all earlier MMAs).
      const bool grow = mxs > m + kRescaleThreshold;
      const bool scale_o = grow && n > 0 && m != -INFINITY;
      if (__any_sync(0xffffffffu, scale_o)) {
        const float f = scale_o ? fast_exp2(m - mxs) : 1.f;
        l *= f;
#pragma unroll
        for (int c = 0; c < DV / 16; ++c) {
          uint32_t o[16];
          tmem_ld_32x32b_x16(tO + c * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st_32x32b_x16(tO + c * 16, o);
        }
      }
      if (grow) m = mxs;
      const float neg_mu = m == -INFINITY ? 0.f : -m;
      const uint64_t nm2 = f2_pack(neg_mu, neg_mu);
      uint64_t rs = f2_pack(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(v[32 * c + 2 * i]), __uint_as_float(v[32 * c + 2 * i + 1])),
                           sl2x2, nm2), x0, x1);
          const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
          const uint64_t e2 = f2_pack(e0, e1);
          asm("add.rn.f32x2 %0, %0, %1;" : "+l"(rs) : "l"(e2));
          pk[i] = pack_bf16x2(e0, e1);
        }
        tmem_st_32x32b_x16(tS + 16 * c, pk);  // P over the first 64 columns of S
      }
      float r0, r1;
      f2_unpack(rs, r0, r1);
      l += r0 + r1;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[t]);
    }
    if (ok && has) ok = mbar_wait_warp_sleep(&o_final[t], 0, p.status, kTimeoutEpilogue, abort_flag);
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const bool row_ok = q < p.S;
    __nv_bfloat16* orow =
        static_cast<__nv_bfloat16*>(p.o) + b * p.o_sb + static_cast<long long>(row_ok ? q : 0) * p.o_ss + h * p.o_sh;
#pragma unroll
    for (int c = 0; c < DV / 32; ++c) {
      uint32_t o[32];
      if (ok && has) {
        tmem_ld_32x32b_x32(tO + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (row_ok) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
    if (row_ok) {
      const float lse = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      p.lse[(static_cast<long long>(b) * p.H + h) * p.S + q] = lse;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, SM::kTmemCols);
  }
}

}  // namespace

namespace attn {

void attn_fwd3_launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& p,
                      int D, cudaStream_t stream) {
  const int num_q = (p.S + kTile - 1) / kTile;
  const int grid = ((num_q + 1) / 2) * p.B * p.H;
  auto run = [&](auto kern, int bytes) {
    set_smem(kern, bytes);
    kern<<<grid, 320, bytes, stream>>>(mq, mk, mv, p);
  };
  if (D == 64 && p.Dv == 64) {
    run(attn_fwd3_kernel<64, 64>, Fwd3Cfg<64, 64>::kBytes);
  } else if (D == 128 && p.Dv == 128) {
    run(attn_fwd3_kernel<128, 128>, Fwd3Cfg<128, 128>::kBytes);
  } else {
    run(attn_fwd3_kernel<192, 128>, Fwd3Cfg<192, 128>::kBytes);
  }
}

}  // namespace attn
}  // namespace pb

// Gated delta-rule recurrence across chunks (tcgen05), forward and backward.
//
// Counterpart of the chunk recurrence inside `chunk_gated_delta_rule` that
// `priml/model/gated_delta_net.py:172-193` calls (flash-linear-attention on CUDA,
// `_torch_chunk_gated_delta_rule` at `priml/model/gated_delta_net.py:207-280` on CPU).
//
// The chunk algebra is split in two. Everything that does not depend on the running
// state is chunk-parallel and runs as batched GEMMs in `priml_b200/ops/gated_delta.py`:
// per chunk of C = 128 tokens it produces
//   W   [C, dk]  = (I + A)^-1 (beta * gamma * K)     Ut [C, dv] = (I + A)^-1 (beta * V)   (fp32)
//   Qg  [C, dk]  = gamma * Q                          Kr [C, dk] = (gamma_C / gamma) * K
//   Mqk [C, C]   = tril(gamma_t / gamma_s * Q K^T)    gC          = gamma_C (chunk decay)
// What remains is a strictly sequential scan over the chunks of one (batch, head) with a
// [dk, dv] state H (H = S^T of the delta rule):
//   U   = Ut - W H                 (the chunk's corrected values)
//   O   = Qg H + Mqk U             (the chunk's output)
//   H'  = gC * H + Kr^T U          (the exit state)
// One CTA owns one (batch, head) and walks its chunks in order. Every product is a
// 128 x 128 x 128 tcgen05 MMA; the fp32 state lives in TMEM, its bf16 copy (the MMA
// operand) in shared memory, and the chunk operands arrive by TMA one chunk ahead.
//
// The backward walks the chunks in reverse with the state gradient dH' (fp32, TMEM):
//   dU  = Mqk^T dO + Kr dH'        dH = gC * dH' + Qg^T dO - W^T dU
// and writes dU and dH' per chunk; the remaining gradients are chunk-parallel batched
// GEMMs on the host side.
//
// Roles: four warps. Thread 0 issues the TMA copies and the MMAs; all four warps run
// the epilogues (warp w owns TMEM lanes 32w..32w+31, i.e. rows 32w..32w+31 of every
// accumulator). Every wait is bounded and reports through the status word.
#include "common.cuh"
#include "kernels.h"

namespace pb {
namespace {

constexpr int kC = 128;                  // tokens per chunk; also dk and dv
constexpr int kSlab = 128 * 128;         // one [128 rows][64 bf16] 128-byte-swizzled slab
constexpr int kTileB = 2 * kSlab;        // one [128][128] bf16 tile
constexpr uint32_t kIdescKK = make_idesc_bf16(128, 128, false, true);  // A K-major, B MN-major
constexpr uint32_t kIdescMM = make_idesc_bf16(128, 128, true, true);   // A MN-major, B MN-major

// [128 rows = M][128 = K] tile, K contiguous in two 64-element slabs: MMA step kk (K = 16).
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * kSlab + (kk & 3) * 32, 16, 1024);
}
// [128 rows = K][128 = M or N] tile, MN contiguous in two 64-element slabs: MMA step kk.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 2048, kSlab, 1024);
}

// Write 32 consecutive bf16 columns [col0, col0 + 32) of `row` into a swizzled [128][128] tile.
__device__ __forceinline__ void st_tile_row32(uint8_t* tile, int row, int col0, const uint32_t (&pk)[16]) {
  uint8_t* r = tile + (col0 >> 6) * kSlab + row * 128;
  const int piece0 = (col0 & 63) >> 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pos = ((piece0 + j) ^ (row & 7)) << 4;
    *reinterpret_cast<uint4*>(r + pos) = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  }
}

__device__ __forceinline__ void st_global_bf16x32(__nv_bfloat16* dst, const uint32_t (&pk)[16]) {
  uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
}

__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, long long row0) {
  tma_load_2d(dst, map, bar, 0, static_cast<int>(row0));
  tma_load_2d(dst + kSlab, map, bar, 64, static_cast<int>(row0));
}

// Bounded wait of thread 0 on a phase it started but nobody consumed (exit after an abort).
__device__ __forceinline__ void drain(uint64_t* bar, uint32_t parity, int* status) {
  mbar_wait(bar, parity, status, kTimeoutDrain, nullptr);
}

}  // namespace

// Forward scan. Shared memory: W, Qg (group A), Mqk, Kr (group B), the bf16 state Hb and
// the corrected values U, each a [128][128] bf16 tile. TMEM: X = W Hb (cols 0-127),
// O (128-255), fp32 state H (256-383).
__global__ void __launch_bounds__(128, 1)
    gdn_fwd_kernel(const __grid_constant__ CUtensorMap mW, const __grid_constant__ CUtensorMap mQ,
                   const __grid_constant__ CUtensorMap mM, const __grid_constant__ CUtensorMap mK, GdnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sQ = smem + kTileB;
  uint8_t* sM = smem + 2 * kTileB;
  uint8_t* sK = smem + 3 * kTileB;
  uint8_t* sH = smem + 4 * kTileB;
  uint8_t* sU = smem + 5 * kTileB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kTileB);
  uint64_t* ld_a = bars;      // W, Qg of a chunk landed
  uint64_t* ld_b = bars + 1;  // Mqk, Kr of a chunk landed
  uint64_t* mma1 = bars + 2;  // X and Qg Hb done
  uint64_t* mma2 = bars + 3;  // O += Mqk U and H += Kr^T U done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = warp * 32 + lane;  // TMEM lane = tile row owned by this thread
  const int n = p.n_chunks;
  const long long chunk0 = static_cast<long long>(blockIdx.x) * n;  // first chunk of this (batch, head)
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mW);
    prefetch_tmap(&mQ);
    prefetch_tmap(&mM);
    prefetch_tmap(&mK);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  for (int i = tid; i < kTileB / 16; i += 128) reinterpret_cast<uint4*>(sH)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tX = tbase, tO = tbase + 128, tH = tbase + 256;

  {  // zero state: fp32 in TMEM, and the saved entry state of chunk 0
    uint32_t z[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) z[j] = 0u;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) tmem_st_32x32b_x32(tH + lane_off + cb * 32, z);
    uint4* hs = reinterpret_cast<uint4*>(p.hs + (chunk0 * kC + row) * kC);
#pragma unroll
    for (int j = 0; j < 16; ++j) hs[j] = make_uint4(0, 0, 0, 0);
  }
  int pend_a = -1, pend_b = -1, pend_m1 = -1, pend_m2 = -1;  // thread 0: phases issued, not yet seen
  if (tid == 0) {
    mbar_arrive_expect_tx(ld_a, 2 * kTileB);
    load_tile(sW, &mW, ld_a, chunk0 * kC);
    load_tile(sQ, &mQ, ld_a, chunk0 * kC);
    mbar_arrive_expect_tx(ld_b, 2 * kTileB);
    load_tile(sM, &mM, ld_b, chunk0 * kC);
    load_tile(sK, &mK, ld_b, chunk0 * kC);
    pend_a = pend_b = 0;
  }
  tmem_wait_st();
  fence_proxy_async_smem();
  tc_fence_before();
  bool ok = __syncthreads_and(1);
  tc_fence_after();

  for (int c = 0; c < n && ok; ++c) {
    const long long r0 = (chunk0 + c) * kC;
    const uint32_t ph = c & 1;
    if (tid == 0) {
      if (mbar_wait(ld_a, ph, p.status, kTimeoutProducer, abort_flag)) {
        pend_a = -1;
        tc_fence_after();
        const uint32_t aw = smem_u32(sW), aq = smem_u32(sQ), bh = smem_u32(sH);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tX, desc_k(aw, kk), desc_mn(bh, kk), kIdescKK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tO, desc_k(aq, kk), desc_mn(bh, kk), kIdescKK, kk > 0);
        umma_commit(mma1);
        pend_m1 = c;
      }
    }
    __syncwarp();
    if (!mbar_wait_warp(mma1, ph, p.status, kTimeoutEpilogue, abort_flag)) ok = false;
    tc_fence_after();
    if (tid == 0 && ok) {
      pend_m1 = -1;
      if (c + 1 < n) {  // W and Qg are free: fetch the next chunk's
        mbar_arrive_expect_tx(ld_a, 2 * kTileB);
        load_tile(sW, &mW, ld_a, r0 + kC);
        load_tile(sQ, &mQ, ld_a, r0 + kC);
        pend_a = c + 1;
      }
    }
    if (ok) {  // U = Ut - X: bf16 into shared memory (operand of both next MMAs) and to global
      const float* ut = p.ut + (r0 + row) * kC;
      __nv_bfloat16* us = p.us + (r0 + row) * kC;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tX + lane_off + cb * 32, v);
        const float4* u4 = reinterpret_cast<const float4*>(ut + cb * 32);
        float uf[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 t = __ldg(u4 + j);
          uf[4 * j] = t.x;
          uf[4 * j + 1] = t.y;
          uf[4 * j + 2] = t.z;
          uf[4 * j + 3] = t.w;
        }
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          pk[j] = pack_bf16x2(uf[2 * j] - __uint_as_float(v[2 * j]), uf[2 * j + 1] - __uint_as_float(v[2 * j + 1]));
        st_tile_row32(sU, row, cb * 32, pk);
        st_global_bf16x32(us + cb * 32, pk);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) break;
    if (tid == 0) {
      if (mbar_wait(ld_b, ph, p.status, kTimeoutProducer, abort_flag)) {
        pend_b = -1;
        tc_fence_after();
        const uint32_t am = smem_u32(sM), ak = smem_u32(sK), bu = smem_u32(sU);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tO, desc_k(am, kk), desc_mn(bu, kk), kIdescKK, 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tH, desc_mn(ak, kk), desc_mn(bu, kk), kIdescMM, 1);
        umma_commit(mma2);
        pend_m2 = c;
      }
    }
    __syncwarp();
    if (!mbar_wait_warp(mma2, ph, p.status, kTimeoutEpilogue, abort_flag)) ok = false;
    tc_fence_after();
    if (tid == 0 && ok) {
      pend_m2 = -1;
      if (c + 1 < n) {
        mbar_arrive_expect_tx(ld_b, 2 * kTileB);
        load_tile(sM, &mM, ld_b, r0 + kC);
        load_tile(sK, &mK, ld_b, r0 + kC);
        pend_b = c + 1;
      }
    }
    if (ok) {
      __nv_bfloat16* o = p.o + (r0 + row) * kC;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tO + lane_off + cb * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        st_global_bf16x32(o + cb * 32, pk);
      }
      if (c + 1 < n) {  // exit state: bf16 operand copy, saved entry state of chunk c + 1, then H *= gC(c + 1)
        const float g = p.gc[chunk0 + c + 1];
        __nv_bfloat16* hs = p.hs + (r0 + kC + row) * kC;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tH + lane_off + cb * 32, v);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          st_tile_row32(sH, row, cb * 32, pk);
          st_global_bf16x32(hs + cb * 32, pk);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * g);
          tmem_st_32x32b_x32(tH + lane_off + cb * 32, v);
        }
        tmem_wait_st();
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }

  if (tid == 0) {  // after an abort: let issued copies and MMAs finish before the CTA leaves
    if (pend_a >= 0) drain(ld_a, pend_a & 1, p.status);
    if (pend_b >= 0) drain(ld_b, pend_b & 1, p.status);
    if (pend_m1 >= 0) drain(mma1, pend_m1 & 1, p.status);
    if (pend_m2 >= 0) drain(mma2, pend_m2 & 1, p.status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// Backward scan, chunks in reverse. Shared memory: Kr, Mqk, dO, Qg (group A, free after the
// first MMA group), W (group B), the bf16 state gradient dHb and -dU. TMEM: dU (cols 0-127),
// fp32 state gradient dH (128-255). First group: dU = Kr dHb + Mqk^T dO and dH += Qg^T dO
// (dH was scaled by gC beforehand); second group: dH += W^T (-dU).
__global__ void __launch_bounds__(128, 1)
    gdn_bwd_kernel(const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mM,
                   const __grid_constant__ CUtensorMap mDO, const __grid_constant__ CUtensorMap mQ,
                   const __grid_constant__ CUtensorMap mW, GdnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sM = smem + kTileB;
  uint8_t* sDO = smem + 2 * kTileB;
  uint8_t* sQ = smem + 3 * kTileB;
  uint8_t* sW = smem + 4 * kTileB;
  uint8_t* sDH = smem + 5 * kTileB;
  uint8_t* sNDU = smem + 6 * kTileB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTileB);
  uint64_t* ld_a = bars;      // Kr, Mqk, dO, Qg of a chunk landed
  uint64_t* ld_b = bars + 1;  // W of a chunk landed
  uint64_t* mma1 = bars + 2;
  uint64_t* mma2 = bars + 3;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = warp * 32 + lane;
  const int n = p.n_chunks;
  const long long chunk0 = static_cast<long long>(blockIdx.x) * n;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(bars + i, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&mK);
    prefetch_tmap(&mM);
    prefetch_tmap(&mDO);
    prefetch_tmap(&mQ);
    prefetch_tmap(&mW);
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  for (int i = tid; i < kTileB / 16; i += 128) reinterpret_cast<uint4*>(sDH)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tDU = tbase, tDH = tbase + 128;

  {  // no gradient reaches the last chunk's exit state
    uint32_t z[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) z[j] = 0u;
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) tmem_st_32x32b_x32(tDH + lane_off + cb * 32, z);
    float4* dhs = reinterpret_cast<float4*>(p.dhs + ((chunk0 + n - 1) * kC + row) * kC);
#pragma unroll
    for (int j = 0; j < 32; ++j) dhs[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int pend_a = -1, pend_b = -1, pend_m1 = -1, pend_m2 = -1;
  if (tid == 0) {
    const long long rl = (chunk0 + n - 1) * kC;
    mbar_arrive_expect_tx(ld_a, 4 * kTileB);
    load_tile(sK, &mK, ld_a, rl);
    load_tile(sM, &mM, ld_a, rl);
    load_tile(sDO, &mDO, ld_a, rl);
    load_tile(sQ, &mQ, ld_a, rl);
    mbar_arrive_expect_tx(ld_b, kTileB);
    load_tile(sW, &mW, ld_b, rl);
    pend_a = pend_b = 0;
  }
  tmem_wait_st();
  fence_proxy_async_smem();
  tc_fence_before();
  bool ok = __syncthreads_and(1);
  tc_fence_after();

  for (int i = 0; i < n && ok; ++i) {
    const int c = n - 1 - i;
    const long long r0 = (chunk0 + c) * kC;
    const uint32_t ph = i & 1;
    if (tid == 0) {
      if (mbar_wait(ld_a, ph, p.status, kTimeoutProducer, abort_flag)) {
        pend_a = -1;
        tc_fence_after();
        const uint32_t ak = smem_u32(sK), am = smem_u32(sM), bdo = smem_u32(sDO), aq = smem_u32(sQ),
                       bdh = smem_u32(sDH);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tDU, desc_k(ak, kk), desc_mn(bdh, kk), kIdescKK, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tDU, desc_mn(am, kk), desc_mn(bdo, kk), kIdescMM, 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tDH, desc_mn(aq, kk), desc_mn(bdo, kk), kIdescMM, 1);
        umma_commit(mma1);
        pend_m1 = i;
      }
    }
    __syncwarp();
    if (!mbar_wait_warp(mma1, ph, p.status, kTimeoutEpilogue, abort_flag)) ok = false;
    tc_fence_after();
    if (tid == 0 && ok) {
      pend_m1 = -1;
      if (c > 0) {
        const long long rn = r0 - kC;
        mbar_arrive_expect_tx(ld_a, 4 * kTileB);
        load_tile(sK, &mK, ld_a, rn);
        load_tile(sM, &mM, ld_a, rn);
        load_tile(sDO, &mDO, ld_a, rn);
        load_tile(sQ, &mQ, ld_a, rn);
        pend_a = i + 1;
      }
    }
    if (ok) {  // dU: fp32 to global, -dU as the bf16 operand of the second group
      float* du = p.du + (r0 + row) * kC;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tDU + lane_off + cb * 32, v);
        tmem_wait_ld();
        float4* d4 = reinterpret_cast<float4*>(du + cb * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          d4[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                              __uint_as_float(v[4 * j + 3]));
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(-__uint_as_float(v[2 * j]), -__uint_as_float(v[2 * j + 1]));
        st_tile_row32(sNDU, row, cb * 32, pk);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) break;
    if (tid == 0) {
      if (mbar_wait(ld_b, ph, p.status, kTimeoutProducer, abort_flag)) {
        pend_b = -1;
        tc_fence_after();
        const uint32_t aw = smem_u32(sW), bn = smem_u32(sNDU);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tDH, desc_mn(aw, kk), desc_mn(bn, kk), kIdescMM, 1);
        umma_commit(mma2);
        pend_m2 = i;
      }
    }
    __syncwarp();
    if (!mbar_wait_warp(mma2, ph, p.status, kTimeoutEpilogue, abort_flag)) ok = false;
    tc_fence_after();
    if (tid == 0 && ok) {
      pend_m2 = -1;
      if (c > 0) {
        mbar_arrive_expect_tx(ld_b, kTileB);
        load_tile(sW, &mW, ld_b, r0 - kC);
        pend_b = i + 1;
      }
    }
    if (ok && c > 0) {  // gradient of chunk c - 1's exit state: saved fp32, bf16 operand, then dH *= gC(c - 1)
      const float g = p.gc[chunk0 + c - 1];
      float* dhs = p.dhs + (r0 - kC + row) * kC;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tDH + lane_off + cb * 32, v);
        tmem_wait_ld();
        float4* d4 = reinterpret_cast<float4*>(dhs + cb * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          d4[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                              __uint_as_float(v[4 * j + 3]));
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        st_tile_row32(sDH, row, cb * 32, pk);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * g);
        tmem_st_32x32b_x32(tDH + lane_off + cb * 32, v);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }

  if (tid == 0) {
    if (pend_a >= 0) drain(ld_a, pend_a & 1, p.status);
    if (pend_b >= 0) drain(ld_b, pend_b & 1, p.status);
    if (pend_m1 >= 0) drain(mma1, pend_m1 & 1, p.status);
    if (pend_m2 >= 0) drain(mma2, pend_m2 & 1, p.status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

namespace {
constexpr int kFwdSmem = 6 * kTileB + 1024 + 64;
constexpr int kBwdSmem = 7 * kTileB + 1024 + 64;
}  // namespace

void gdn_chunk_fwd(const void* w, const void* qg, const void* mqk, const void* kr, const GdnParams& p,
                   cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.bh) * p.n_chunks * kC;
  CUtensorMap mW, mQ, mM, mK;
  make_tmap_2d_bf16(&mW, w, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mQ, qg, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mM, mqk, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mK, kr, kC, rows, kC, 64, kC);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gdn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
    attr = true;
  }
  gdn_fwd_kernel<<<p.bh, 128, kFwdSmem, stream>>>(mW, mQ, mM, mK, p);
}

void gdn_chunk_bwd(const void* kr, const void* mqk, const void* dout, const void* qg, const void* w,
                   const GdnParams& p, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.bh) * p.n_chunks * kC;
  CUtensorMap mK, mM, mDO, mQ, mW;
  make_tmap_2d_bf16(&mK, kr, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mM, mqk, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mDO, dout, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mQ, qg, kC, rows, kC, 64, kC);
  make_tmap_2d_bf16(&mW, w, kC, rows, kC, 64, kC);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gdn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
    attr = true;
  }
  gdn_bwd_kernel<<<p.bh, 128, kBwdSmem, stream>>>(mK, mM, mDO, mQ, mW, p);
}

}  // namespace pb

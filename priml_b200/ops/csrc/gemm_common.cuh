// Tile constants, parameters, tile order and the epilogue row store shared by
// the dense GEMM (gemm.cu) and the grouped expert GEMM (grouped_gemm.cu).
#pragma once

#include "common.cuh"

namespace pb {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int GROUP_M = 16;
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct GemmParams {
  int M, N, K;
  void* C;
  long long ldc;
  const void* aux;       // SwiGLU: unused; residual add: [M, ldc] bf16
  int* status;
  int num_n_half;        // fused SwiGLU: H (gate/up split point in B rows)
  int splits = 1;        // split-K factor (pair kernel, fp32 reduce-add epilogue only)
  float alpha = 1.f;     // epilogue 5: C = alpha * acc + beta * aux (aux bf16 with row stride ldc)
  float beta = 0.f;
  int batch = 1;         // pair kernel: independent products stacked along the outer (row) axis of every operand
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int group = GROUP_M * num_n;
  const int g = tile / group;
  const int first_m = g * GROUP_M;
  const int gm = min(num_m - first_m, GROUP_M);
  const int r = tile - g * group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// 1 / (1 + e^-x) with the hardware exponential and reciprocal approximations. Large negative
// x gives an infinite denominator and a zero result, never the slow path of an IEEE divide.
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Epilogue staging tiles are 32 rows of NCH 16-byte chunks (NCH = 4: 64-byte bf16 rows,
// NCH = 8: 128-byte fp32 rows) in the layout of the tensor maps' 64-byte / 128-byte swizzle:
// chunk k of row r sits at chunk position k ^ ((r >> 1) & 3) (NCH = 4) or k ^ (r & 7)
// (NCH = 8), i.e. address bits [4, 4 + log2 NCH) XOR bits [7, 7 + log2 NCH) of the offset.
// Eight lanes writing or reading their own rows in one 128-bit phase then hit distinct banks,
// and the data index stays a compile-time constant (only the address depends on the lane).
template <int NCH>
__device__ __forceinline__ int swz_chunk(int row, int k) {
  return NCH == 8 ? (k ^ (row & 7)) : (k ^ ((row >> 1) & 3));
}

template <int NCH>
__device__ __forceinline__ void stage_row(uint8_t* tile, int row, const uint32_t (&words)[4 * NCH]) {
  uint8_t* row_ptr = tile + row * (16 * NCH);
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    *reinterpret_cast<uint4*>(row_ptr + swz_chunk<NCH>(row, k) * 16) =
        make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
  }
}

template <int NCH>
__device__ __forceinline__ void load_row(const uint8_t* tile, int row, uint32_t (&words)[4 * NCH]) {
  const uint8_t* row_ptr = tile + row * (16 * NCH);
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const uint4 v = *reinterpret_cast<const uint4*>(row_ptr + swz_chunk<NCH>(row, k) * 16);
    words[4 * k] = v.x;
    words[4 * k + 1] = v.y;
    words[4 * k + 2] = v.z;
    words[4 * k + 3] = v.w;
  }
}

// Store one accumulator row slice (this thread's TMEM lane) of output tile column block `nb`,
// accumulator columns [c_lo, c_hi) (hidden units [c_lo, c_hi) of the tile for the SwiGLU
// epilogues 3 and 4; c_hi < 0 means the whole tile).
template <int BN, int EPI>
__device__ __forceinline__ void store_acc_row(const GemmParams& p, uint32_t t_row, int row, int nb, int c_lo = 0,
                                              int c_hi = -1) {
  const bool row_ok = row < p.M;
  if constexpr (EPI == 3) {
    const int H = p.num_n_half;
    const int h0 = nb * (BN / 2);
    __nv_bfloat16* hout = static_cast<__nv_bfloat16*>(p.C) + static_cast<long long>(row) * p.ldc;
    __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(p.aux)) +
                        static_cast<long long>(row) * (2LL * H);
    if (c_hi < 0) c_hi = BN / 2;
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(t_row + c, g);
      tmem_ld_32x32b_x32(t_row + BN / 2 + c, u);
      tmem_wait_ld();
      const int col = h0 + c;
      if (row_ok && col < H) {
        uint32_t hv[16], gv[16], uv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float g0 = __uint_as_float(g[2 * j]), g1 = __uint_as_float(g[2 * j + 1]);
          const float u0 = __uint_as_float(u[2 * j]), u1 = __uint_as_float(u[2 * j + 1]);
          // Round gate/up to bf16 first so forward and backward see the same values.
          const __nv_bfloat162 gb = __floats2bfloat162_rn(g0, g1);
          const __nv_bfloat162 ub = __floats2bfloat162_rn(u0, u1);
          const float2 gf = __bfloat1622float2(gb), uf = __bfloat1622float2(ub);
          const float s0 = gf.x * sigmoid_fast(gf.x), s1 = gf.y * sigmoid_fast(gf.y);
          hv[j] = pack_bf16x2(s0 * uf.x, s1 * uf.y);
          gv[j] = *reinterpret_cast<const uint32_t*>(&gb);
          uv[j] = *reinterpret_cast<const uint32_t*>(&ub);
        }
        if (col + 32 <= H) {
          uint4* hp = reinterpret_cast<uint4*>(hout + col);
          uint4* gp = reinterpret_cast<uint4*>(gu + col);
          uint4* up = reinterpret_cast<uint4*>(gu + H + col);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            hp[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
            gp[q] = make_uint4(gv[4 * q], gv[4 * q + 1], gv[4 * q + 2], gv[4 * q + 3]);
            up[q] = make_uint4(uv[4 * q], uv[4 * q + 1], uv[4 * q + 2], uv[4 * q + 3]);
          }
        } else {
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(hv);
          const __nv_bfloat16* gb2 = reinterpret_cast<const __nv_bfloat16*>(gv);
          const __nv_bfloat16* ub2 = reinterpret_cast<const __nv_bfloat16*>(uv);
          for (int j = 0; j < 32 && col + j < H; ++j) {
            hout[col + j] = hb[j];
            gu[col + j] = gb2[j];
            gu[H + col + j] = ub2[j];
          }
        }
      }
    }
  } else if constexpr (EPI == 4) {
    // Accumulator = dh (N = H); aux = saved [gate | up] pre-activation [M, 2H]; C = dgu [M, 2H].
    // dh is rounded to bf16 first, as the unfused path stores it.
    const int H = p.num_n_half;
    const __nv_bfloat16* gu = static_cast<const __nv_bfloat16*>(p.aux) + static_cast<long long>(row) * (2LL * H);
    __nv_bfloat16* dgu = static_cast<__nv_bfloat16*>(p.C) + static_cast<long long>(row) * p.ldc;
    if (c_hi < 0) c_hi = BN;
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c, v);
      tmem_wait_ld();
      const int col = nb * BN + c;
      if (!row_ok || col >= H) continue;
      const int n = min(32, H - col);
      uint32_t gw[16], uw[16], dg[16], du[16];
      if (n == 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 a = reinterpret_cast<const uint4*>(gu + col)[q];
          const uint4 b = reinterpret_cast<const uint4*>(gu + H + col)[q];
          gw[4 * q] = a.x, gw[4 * q + 1] = a.y, gw[4 * q + 2] = a.z, gw[4 * q + 3] = a.w;
          uw[4 * q] = b.x, uw[4 * q + 1] = b.y, uw[4 * q + 2] = b.z, uw[4 * q + 3] = b.w;
        }
      } else {
        const uint16_t* g16 = reinterpret_cast<const uint16_t*>(gu + col);
        const uint16_t* u16 = reinterpret_cast<const uint16_t*>(gu + H + col);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int a = 2 * j, b2 = 2 * j + 1;
          gw[j] = (a < n ? g16[a] : 0u) | ((b2 < n ? static_cast<uint32_t>(g16[b2]) : 0u) << 16);
          uw[j] = (a < n ? u16[a] : 0u) | ((b2 < n ? static_cast<uint32_t>(u16[b2]) : 0u) << 16);
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[j]));
        const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[j]));
        const float2 d = __bfloat1622float2(__floats2bfloat162_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])));
        const float s0 = sigmoid_fast(g.x), s1 = sigmoid_fast(g.y);
        du[j] = pack_bf16x2(d.x * (g.x * s0), d.y * (g.y * s1));
        dg[j] = pack_bf16x2(d.x * u.x * s0 * (1.f + g.x * (1.f - s0)), d.y * u.y * s1 * (1.f + g.y * (1.f - s1)));
      }
      if (n == 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          reinterpret_cast<uint4*>(dgu + col)[q] = make_uint4(dg[4 * q], dg[4 * q + 1], dg[4 * q + 2], dg[4 * q + 3]);
          reinterpret_cast<uint4*>(dgu + H + col)[q] = make_uint4(du[4 * q], du[4 * q + 1], du[4 * q + 2], du[4 * q + 3]);
        }
      } else {
        const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(dg);
        const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(du);
        for (int j = 0; j < n; ++j) {
          dgu[col + j] = gb[j];
          dgu[H + col + j] = ub[j];
        }
      }
    }
  } else {
    if (c_hi < 0) c_hi = BN;
#pragma unroll 1
    for (int c = c_lo; c < c_hi; c += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c, v);
      tmem_wait_ld();
      const int col = nb * BN + c;
      if (!row_ok || col >= p.N) continue;
      const bool full_chunk = col + 32 <= p.N;
      if constexpr (EPI == 0) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.C) + static_cast<long long>(row) * p.ldc + col;
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
          uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
          for (int q = 0; q < 4; ++q) o4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        } else {
          const __nv_bfloat16* pb16 = reinterpret_cast<const __nv_bfloat16*>(pk);
          for (int j = 0; j < 32 && col + j < p.N; ++j) out[j] = pb16[j];
        }
      } else {
        float* out = static_cast<float*>(p.C) + static_cast<long long>(row) * p.ldc + col;
        if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
          float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 a = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                   __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
            if constexpr (EPI == 2) {
              const float4 o = o4[q];
              a.x += o.x;
              a.y += o.y;
              a.z += o.z;
              a.w += o.w;
            }
            o4[q] = a;
          }
        } else {
          for (int j = 0; j < 32 && col + j < p.N; ++j) {
            const float a = __uint_as_float(v[j]);
            out[j] = EPI == 2 ? out[j] + a : a;
          }
        }
      }
    }
  }
}

}  // namespace
}  // namespace pb

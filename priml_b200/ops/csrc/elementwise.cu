// Memory-bound kernels: RMSNorm, RoPE, SwiGLU, cross-entropy, multi-tensor
// AdamW / grad-norm, casts. All statistics are accumulated in fp32; every
// kernel reads and writes with 16-byte vectors where the layout allows.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

namespace pb {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Load / store 8 consecutive elements as fp32 from bf16 or fp32 storage.
__device__ __forceinline__ void load8(const void* base, bool f32, long long idx, float (&v)[8]) {
  if (f32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + idx);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void store8(void* base, bool f32, long long idx, const float (&v)[8]) {
  if (f32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + idx);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 raw;
    raw.x = pack_bf16x2(v[0], v[1]);
    raw.y = pack_bf16x2(v[2], v[3]);
    raw.z = pack_bf16x2(v[4], v[5]);
    raw.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(base) + idx) = raw;
  }
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; C % 8 == 0.
//
// Residual form: with an addend d the kernel normalizes h = x + d and, when h
// is given, stores it (the next residual-stream value) in the same pass, so a
// pre-norm block needs no separate add kernel. A bf16 h is rounded before the
// statistics, so y is exactly the normalization of the stored h.
__device__ __forceinline__ void round_bf16_8(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
}

__global__ void rmsnorm_fwd_kernel(const void* __restrict__ x, bool x_f32, const void* __restrict__ d, bool d_f32,
                                   const float* __restrict__ w, void* __restrict__ h, bool h_f32,
                                   void* __restrict__ y, bool y_f32, float* __restrict__ rstd, int R, int C,
                                   float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const long long base = static_cast<long long>(row) * C;
  float ss = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
    float v[8];
    load8(x, x_f32, base + c, v);
    if (d != nullptr) {
      float a[8];
      load8(d, d_f32, base + c, a);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += a[j];
      if (h != nullptr) {
        if (!h_f32) round_bf16_8(v);
        store8(h, h_f32, base + c, v);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(C) + eps);
  if (lane == 0 && rstd != nullptr) rstd[row] = r;
  for (int c = lane * 8; c < C; c += 256) {
    float v[8];
    if (d != nullptr && h != nullptr) {
      load8(h, h_f32, base + c, v);  // this thread's own stores from the first pass
    } else {
      load8(x, x_f32, base + c, v);
      if (d != nullptr) {
        float a[8];
        load8(d, d_f32, base + c, a);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += a[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = v[j] * r * (w != nullptr ? w[c + j] : 1.f);
    store8(y, y_f32, base + c, v);
  }
}

// dx = dres + rstd * (w*dy - xhat * mean(w*dy*xhat)); dres is the gradient that
// reached the normalized input along the residual path (optional). dx2, when
// given, receives the same values in a second dtype: the gradient of the
// addend d, which shares h's gradient.
__global__ void rmsnorm_bwd_kernel(const void* __restrict__ dy, bool dy_f32, const void* __restrict__ x, bool x_f32,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   const void* __restrict__ dres, bool dres_f32, void* __restrict__ dx, bool dx_f32,
                                   void* __restrict__ dx2, bool dx2_f32, float* __restrict__ dw, int R, int C) {
  // dw: every warp sums its rows' dy * xhat into its own C-float slice of shared memory (each lane
  // owns fixed columns, so the adds need no atomics); the slices are summed once at the end.
  extern __shared__ float dw_acc[];  // warps * C floats when dw != nullptr
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  float* my_dw = dw_acc + (threadIdx.x >> 5) * C;
  if (dw != nullptr) {
    for (int c = threadIdx.x; c < warps * C; c += blockDim.x) dw_acc[c] = 0.f;
    __syncthreads();
  }
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < R; row += gridDim.x * warps) {
    const long long base = static_cast<long long>(row) * C;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = lane * 8; c < C; c += 256) {
      float g[8], v[8];
      load8(dy, dy_f32, base + c, g);
      load8(x, x_f32, base + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += g[j] * (w != nullptr ? w[c + j] : 1.f) * v[j] * r;
    }
    dot = warp_sum(dot) / static_cast<float>(C);
    for (int c = lane * 8; c < C; c += 256) {
      float g[8], v[8], o[8];
      load8(dy, dy_f32, base + c, g);
      load8(x, x_f32, base + c, v);
      if (dres != nullptr) {
        load8(dres, dres_f32, base + c, o);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = v[j] * r;
        const float wg = g[j] * (w != nullptr ? w[c + j] : 1.f);
        o[j] += r * (wg - xh * dot);
        if (dw != nullptr) my_dw[c + j] += g[j] * xh;
      }
      store8(dx, dx_f32, base + c, o);
      if (dx2 != nullptr) store8(dx2, dx2_f32, base + c, o);
    }
  }
  if (dw != nullptr) {
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float sum = 0.f;
      for (int q = 0; q < warps; ++q) sum += dw_acc[q * C + c];
      atomicAdd(&dw[c], sum);
    }
  }
}

// ------------------------------------------------------------------ RoPE
// One block per (b, s); threads over (head, pair). y is contiguous [B, S, H, D].
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, long long sb, long long ss, long long sh,
                            __nv_bfloat16* __restrict__ y, int S, int H, int D, const float* __restrict__ cosv,
                            const float* __restrict__ sinv, float sign) {
  const int bs = blockIdx.x;
  const int b = bs / S, s = bs - b * S;
  const int half = D / 2;
  const __nv_bfloat16* xr = x + b * sb + s * ss;
  __nv_bfloat16* yr = y + (static_cast<long long>(bs) * H) * D;
  const float* cr = cosv + static_cast<long long>(s) * half;
  const float* sr = sinv + static_cast<long long>(s) * half;
  // Two pairs per thread step (bf16x2 loads on each half).
  const int pairs2 = H * (half / 2);
  for (int t = threadIdx.x; t < pairs2; t += blockDim.x) {
    const int h = t / (half / 2);
    const int i = (t - h * (half / 2)) * 2;
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(xr + h * sh + i);
    const __nv_bfloat162 c = *reinterpret_cast<const __nv_bfloat162*>(xr + h * sh + i + half);
    const float2 x0 = __bfloat1622float2(a), x1 = __bfloat1622float2(c);
    const float c0 = cr[i], c1 = cr[i + 1];
    const float s0 = sign * sr[i], s1 = sign * sr[i + 1];
    // Separately rounded products (no FMA contraction) so the result matches the
    // fp32 reference x0*cos - x1*sin, x1*cos + x0*sin bit for bit.
    __nv_bfloat162 o0 = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(x0.x, c0), __fmul_rn(x1.x, s0)),
                                              __fsub_rn(__fmul_rn(x0.y, c1), __fmul_rn(x1.y, s1)));
    __nv_bfloat162 o1 = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(x1.x, c0), __fmul_rn(x0.x, s0)),
                                              __fadd_rn(__fmul_rn(x1.y, c1), __fmul_rn(x0.y, s1)));
    *reinterpret_cast<__nv_bfloat162*>(yr + h * D + i) = o0;
    *reinterpret_cast<__nv_bfloat162*>(yr + h * D + i + half) = o1;
  }
}

// ------------------------------------------------------------------ SwiGLU
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, long long R,
                                  int H) {
  const long long n8 = R * H / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 8;
    const long long r = e / H;
    const int c = static_cast<int>(e - r * H);
    float g[8], u[8], o[8];
    load8(gu, false, r * 2 * H + c, g);
    load8(gu, false, r * 2 * H + H + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    store8(h, false, e, o);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, long long R, int H) {
  const long long n8 = R * H / 8;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 8;
    const long long r = e / H;
    const int c = static_cast<int>(e - r * H);
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu, false, r * 2 * H + c, g);
    load8(gu, false, r * 2 * H + H + c, u);
    load8(dh, false, e, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-g[j]));
      const float silu = g[j] * sg;
      du[j] = d[j] * silu;
      dg[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
    }
    store8(dgu, false, r * 2 * H + c, dg);
    store8(dgu, false, r * 2 * H + H + c, du);
  }
}

// ------------------------------------------------------------------ cross-entropy
// One block (256 threads) per row; online max / sum-exp in one pass.
constexpr int kCeThreads = 256;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
  m = mm;
}

// Soft cap z = cap * tanh(x / cap) (Gemma 2's logit cap), evaluated on the fp32 value of each
// bf16 logit. tanh.approx.f32 is one MUFU operation with relative error below 2^-10.9, far under
// the bf16 rounding of the logit it is applied to; the row stays one read of HBM.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool kCap>
__device__ __forceinline__ float ce_logit(float x, float cap, float inv_cap) {
  if constexpr (kCap) return cap * tanh_approx(x * inv_cap);
  return x;
}

template <bool kCap>
__global__ void ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, const int64_t* __restrict__ tgt,
                              float* __restrict__ loss, float* __restrict__ lse_out, int V, long long ignore_index,
                              float cap) {
  const long long row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  const float inv_cap = kCap ? 1.f / cap : 0.f;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
    float v[8];
    if (c + 8 <= V) {
      load8(x, false, c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = ce_logit<kCap>(v[j], cap, inv_cap);
    } else {
      for (int j = 0; j < 8; ++j)
        v[j] = c + j < V ? ce_logit<kCap>(__bfloat162float(x[c + j]), cap, inv_cap) : -INFINITY;
    }
    float lm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, v[j]);
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ls += __expf(v[j] - lm);
    online_merge(m, s, lm, ls);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[kCeThreads / 32], ssum[kCeThreads / 32];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm[w] = m;
    ssum[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], Ssum = ssum[0];
    for (int i = 1; i < kCeThreads / 32; ++i) online_merge(M, Ssum, sm[i], ssum[i]);
    const float lse = M + __logf(Ssum);
    const int64_t t = tgt[row];
    lse_out[row] = lse;
    loss[row] = (t == ignore_index) ? 0.f : lse - ce_logit<kCap>(__bfloat162float(x[t]), cap, inv_cap);
  }
}

// d(loss)/d(x) = (softmax(z) - onehot(t)) * dz/dx, with dz/dx = 1 - tanh(x / cap)^2 under the cap.
template <bool kCap>
__device__ __forceinline__ float ce_grad(float x, float l, bool is_t, float scale, float cap, float inv_cap) {
  if constexpr (kCap) {
    const float th = tanh_approx(x * inv_cap);
    return (__expf(cap * th - l) - (is_t ? 1.f : 0.f)) * scale * (1.f - th * th);
  }
  return (__expf(x - l) - (is_t ? 1.f : 0.f)) * scale;
}

template <bool kCap>
__global__ void ce_bwd_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, const int64_t* __restrict__ tgt,
                              const float* __restrict__ lse, const float* __restrict__ g, long long g_stride,
                              __nv_bfloat16* __restrict__ dlogits, int V, long long ignore_index, float cap) {
  const long long row = blockIdx.x;
  const int64_t t = tgt[row];
  const float scale = (t == ignore_index) ? 0.f : g[row * g_stride];
  const float l = lse[row];
  const float inv_cap = kCap ? 1.f / cap : 0.f;
  const __nv_bfloat16* x = logits + row * ld;
  __nv_bfloat16* d = dlogits + row * ld;
  for (int c = threadIdx.x * 8; c < V; c += kCeThreads * 8) {
    if (c + 8 <= V) {
      float v[8];
      load8(x, false, c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = ce_grad<kCap>(v[j], l, c + j == t, scale, cap, inv_cap);
      store8(d, false, c, v);
    } else {
      for (int j = c; j < V; ++j) {
        d[j] = __float2bfloat16(ce_grad<kCap>(__bfloat162float(x[j]), l, j == t, scale, cap, inv_cap));
      }
    }
  }
}

// ------------------------------------------------------------------ AdamW
__device__ __forceinline__ float lerp_torch(float a, float b, float w) {
  // torch.lerp: a + w (b - a) for w < 0.5, else b - (b - a)(1 - w)
  return w < 0.5f ? fmaf(w, b - a, a) : b - (b - a) * (1.f - w);
}

__global__ void adamw_kernel(const AdamTensor* __restrict__ tensors, const int* __restrict__ chunk_tensor,
                             const long long* __restrict__ chunk_start, int chunk_elems, float lr, float beta1,
                             float beta2, float eps, float wd, float bias1, float bias2,
                             const float* __restrict__ grad_scale) {
  const AdamTensor t = tensors[chunk_tensor[blockIdx.x]];
  const long long start = chunk_start[blockIdx.x];
  const long long end = min(start + chunk_elems, t.n);
  const float gs = grad_scale != nullptr ? *grad_scale : 1.f;
  const float decay = 1.f - lr * wd;
  const float step_size = lr / bias1;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = (t.g_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(t.g)[i])
                              : static_cast<const float*>(t.g)[i]) *
                    gs;
    float p = t.p[i] * decay;
    const float m = lerp_torch(t.m[i], g, 1.f - beta1);
    const float v = lerp_torch(t.v[i], g * g, 1.f - beta2);
    const float denom = sqrtf(v / bias2) + eps;
    p -= m / denom * step_size;
    t.p[i] = p;
    t.m[i] = m;
    t.v[i] = v;
    if (t.shadow != nullptr) static_cast<__nv_bfloat16*>(t.shadow)[i] = __float2bfloat16(p);
  }
}

__global__ void sumsq_kernel(const AdamTensor* __restrict__ tensors, const int* __restrict__ chunk_tensor,
                             const long long* __restrict__ chunk_start, int chunk_elems, float* __restrict__ out) {
  const AdamTensor t = tensors[chunk_tensor[blockIdx.x]];
  const long long start = chunk_start[blockIdx.x];
  const long long end = min(start + chunk_elems, t.n);
  float acc = 0.f;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = t.g_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(t.g)[i])
                             : static_cast<const float*>(t.g)[i];
    acc += g * g;
  }
  acc = warp_sum(acc);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

__global__ void clip_kernel(const float* sumsq, float max_norm, float* clip, float* norm) {
  const float n = sqrtf(*sumsq);
  if (norm != nullptr) *norm = n;
  if (clip != nullptr) *clip = fminf(1.f, max_norm / (n + 1e-6f));
}

__global__ void cast_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}

int grid_for(long long work, int threads) {
  const long long blocks = (work + threads - 1) / threads;
  const long long cap = static_cast<long long>(device_sm_count()) * 16;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace

void rmsnorm_fwd(const void* x, bool x_f32, const float* w, void* y, bool y_f32, float* rstd, int R, int C, float eps,
                 cudaStream_t stream, const void* d, bool d_f32, void* h, bool h_f32) {
  const int warps = 8;
  rmsnorm_fwd_kernel<<<(R + warps - 1) / warps, warps * 32, 0, stream>>>(x, x_f32, d, d_f32, w, h, h_f32, y, y_f32,
                                                                          rstd, R, C, eps);
}

void rmsnorm_bwd(const void* dy, bool dy_f32, const void* x, bool x_f32, const float* w, const float* rstd, void* dx,
                 bool dx_f32, float* dw, int R, int C, cudaStream_t stream, const void* dres, bool dres_f32, void* dx2,
                 bool dx2_f32) {
  // With dw, each warp keeps a C-float slice in shared memory: at most 96 KB per block.
  int warps = 8;
  if (dw != nullptr) {
    const int fit = static_cast<int>((96 * 1024) / (static_cast<size_t>(C) * sizeof(float)));
    warps = fit < 1 ? 1 : (fit < 8 ? fit : 8);
  }
  int blocks = (R + warps - 1) / warps;
  const size_t smem = dw != nullptr ? static_cast<size_t>(warps) * C * sizeof(float) : 0;
  if (dw != nullptr) {
    const int per_sm = static_cast<int>((200 * 1024) / smem);  // resident blocks the shared slices allow
    const int cap = device_sm_count() * (per_sm < 1 ? 1 : (per_sm > 4 ? 4 : per_sm));
    blocks = blocks < cap ? blocks : cap;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  }
  rmsnorm_bwd_kernel<<<blocks, warps * 32, smem, stream>>>(dy, dy_f32, x, x_f32, w, rstd, dres, dres_f32, dx, dx_f32,
                                                            dx2, dx2_f32, dw, R, C);
}

void rope_apply(const void* x, long long sb, long long ss, long long sh, void* y, int B, int S, int H, int D,
                const float* cos, const float* sin, float sign, cudaStream_t stream) {
  const int threads = 128;
  rope_kernel<<<B * S, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), sb, ss, sh,
                                             static_cast<__nv_bfloat16*>(y), S, H, D, cos, sin, sign);
}

void swiglu_fwd(const void* gu, void* h, long long R, int H, cudaStream_t stream) {
  swiglu_fwd_kernel<<<grid_for(R * H / 8, 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(gu),
                                                                   static_cast<__nv_bfloat16*>(h), R, H);
}

void swiglu_bwd(const void* gu, const void* dh, void* dgu, long long R, int H, cudaStream_t stream) {
  swiglu_bwd_kernel<<<grid_for(R * H / 8, 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(dh),
      static_cast<__nv_bfloat16*>(dgu), R, H);
}

void ce_fwd(const void* logits, long long ld, const int64_t* targets, float* loss, float* lse, long long R, int V,
            long long ignore_index, float softcap, cudaStream_t stream) {
  auto* x = static_cast<const __nv_bfloat16*>(logits);
  if (softcap > 0.f)
    ce_fwd_kernel<true><<<static_cast<unsigned>(R), kCeThreads, 0, stream>>>(x, ld, targets, loss, lse, V,
                                                                             ignore_index, softcap);
  else
    ce_fwd_kernel<false><<<static_cast<unsigned>(R), kCeThreads, 0, stream>>>(x, ld, targets, loss, lse, V,
                                                                              ignore_index, 0.f);
}

void ce_bwd(const void* logits, long long ld, const int64_t* targets, const float* lse, const float* g,
            long long g_stride, void* dlogits, long long R, int V, long long ignore_index, float softcap,
            cudaStream_t stream) {
  auto* x = static_cast<const __nv_bfloat16*>(logits);
  auto* d = static_cast<__nv_bfloat16*>(dlogits);
  if (softcap > 0.f)
    ce_bwd_kernel<true><<<static_cast<unsigned>(R), kCeThreads, 0, stream>>>(x, ld, targets, lse, g, g_stride, d, V,
                                                                             ignore_index, softcap);
  else
    ce_bwd_kernel<false><<<static_cast<unsigned>(R), kCeThreads, 0, stream>>>(x, ld, targets, lse, g, g_stride, d,
                                                                              V, ignore_index, 0.f);
}

void adamw_multi(const AdamTensor* tensors, const int* chunk_tensor, const long long* chunk_start, int num_chunks,
                 int chunk_elems, float lr, float beta1, float beta2, float eps, float weight_decay, float bias1,
                 float bias2, const float* grad_scale, cudaStream_t stream) {
  if (num_chunks == 0) return;
  adamw_kernel<<<num_chunks, 512, 0, stream>>>(tensors, chunk_tensor, chunk_start, chunk_elems, lr, beta1, beta2, eps,
                                               weight_decay, bias1, bias2, grad_scale);
}

void multi_sumsq(const AdamTensor* tensors, const int* chunk_tensor, const long long* chunk_start, int num_chunks,
                 int chunk_elems, float* out, cudaStream_t stream) {
  if (num_chunks == 0) return;
  sumsq_kernel<<<num_chunks, 512, 0, stream>>>(tensors, chunk_tensor, chunk_start, chunk_elems, out);
}

void clip_coef(const float* sumsq, float max_norm, float* clip, float* norm, cudaStream_t stream) {
  clip_kernel<<<1, 1, 0, stream>>>(sumsq, max_norm, clip, norm);
}

void cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t stream) {
  cast_kernel<<<grid_for(n, 256), 256, 0, stream>>>(x, static_cast<__nv_bfloat16*>(y), n);
}

}  // namespace pb

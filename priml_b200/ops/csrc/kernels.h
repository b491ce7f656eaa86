// Host-side entry points of the sm_100a kernels (raw pointers, no torch types),
// so the .cu files build with nvcc alone and bindings.cpp stays the only
// translation unit that includes torch.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pb {

int device_sm_count();
// 2-D bf16 tensor map, 128-byte swizzle. `inner` is the contiguous extent,
// `row_stride` the stride (elements) between consecutive outer rows.
void make_tmap_2d_bf16(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                       int box_inner, int box_outer);
// 2-D maps for epilogue staging tiles: bf16 with 64-byte rows and 64-byte swizzle, fp32 with
// 128-byte rows and 128-byte swizzle.
void make_tmap_2d_bf16_sw64(CUtensorMap* map, const void* base, long long inner, long long outer,
                            long long row_stride, int box_inner, int box_outer);
void make_tmap_2d_f32_sw128(CUtensorMap* map, const void* base, long long inner, long long outer,
                            long long row_stride, int box_inner, int box_outer);
// 3-D bf16 tensor map (inner, mid, outer) with element strides for mid/outer.
// 2-D fp32 map without swizzle (bulk reduce targets).
void make_tmap_2d_f32(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                      int box_inner, int box_outer);
void make_tmap_2d_u8(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                     int box_inner, int box_outer);
void make_tmap_2d_u8_plain(CUtensorMap* map, const void* base, long long inner, long long outer, long long row_stride,
                           int box_inner, int box_outer);
void make_tmap_3d_bf16(CUtensorMap* map, const void* base, long long inner, long long mid, long long outer,
                       long long mid_stride, long long outer_stride, int box_inner, int box_mid, bool swizzle128);

// GEMM: C[M,N] (op)= sum_k A(m,k) B(n,k). epi: 0 bf16, 1 fp32, 2 fp32 +=, 3 fused SwiGLU,
// 4 SwiGLU backward, 5 bf16 C = alpha * acc + beta * aux (aux: bf16 rows of stride ldc).
void gemm_bf16(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C,
               long long ldc, int M, int N, int K, int epi, const void* aux, int swiglu_h, int* status,
               cudaStream_t stream, float alpha = 1.f, float beta = 0.f);
// `batch` products in one persistent launch, operands stacked along their outer axis (epi 0 or 5;
// M, N multiples of 256, K of 64).
void gemm_bf16_batched(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C,
                       long long ldc, int M, int N, int K, int batch, int epi, const void* aux, int* status,
                       cudaStream_t stream, float alpha = 1.f, float beta = 0.f);

// Grouped expert GEMM over 128-row-aligned expert segments (device offsets [experts + 1]).
// mode 0: C[r] = A[r] @ B_e^T (B stacked per expert, b_rows rows each; epi 0, 1, 3, 4);
// mode 1: C[e * out_rows + m, n] = sum_{r in e} A[r, m] B[r, n] (epi 1 or 2).
void grouped_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, bool b_mn, void* C, long long ldc,
                       int rows, int N, int K, const int* offsets, int experts, int b_rows, int mode, int out_rows,
                       int epi, const void* aux, int swiglu_h, int* status, cudaStream_t stream);

// MXFP8 (mxfp8.cu): E4M3 elements with one E8M0 scale per 32 along the contraction dim, scales
// in the blocked layout of mx_scale_bytes(rows, k) bytes.
long long mx_scale_bytes(long long rows, long long k);
void mx_quantize(const void* x, long long ldx, void* q, void* sf, int R, int K, bool transpose, cudaStream_t stream);
void mx_gemm(const void* A, const void* sfa, const void* B, const void* sfb, void* C, long long ldc, int M, int N, int K,
             int epi, int* status, cudaStream_t stream);

// RMSNorm over the last dim C of R rows. x: bf16 or fp32 (x_f32 selects), y: bf16 or fp32.
// Residual form: with an addend d the normalized value is h = x + d, stored to h when given.
void rmsnorm_fwd(const void* x, bool x_f32, const float* w, void* y, bool y_f32, float* rstd, int R, int C, float eps,
                 cudaStream_t stream, const void* d = nullptr, bool d_f32 = false, void* h = nullptr,
                 bool h_f32 = false);
// dx = dres (optional residual-path gradient) + the normalization's gradient; dx2 (optional)
// receives the same values in a second dtype.
void rmsnorm_bwd(const void* dy, bool dy_f32, const void* x, bool x_f32, const float* w, const float* rstd, void* dx,
                 bool dx_f32, float* dw, int R, int C, cudaStream_t stream, const void* dres = nullptr,
                 bool dres_f32 = false, void* dx2 = nullptr, bool dx2_f32 = false);

// Half-split RoPE on [B, S, H, D] views (last dim contiguous); cos/sin fp32 [S, D/2].
// sign = +1 forward rotation, -1 inverse (backward).
void rope_apply(const void* x, long long sb, long long ss, long long sh, void* y, int B, int S, int H, int D,
                const float* cos, const float* sin, float sign, cudaStream_t stream);

// SwiGLU on [R, 2H] (gate | up) -> [R, H]; backward writes d[gate | up].
void swiglu_fwd(const void* gu, void* h, long long R, int H, cudaStream_t stream);
void swiglu_bwd(const void* gu, const void* dh, void* dgu, long long R, int H, cudaStream_t stream);

// Cross-entropy over bf16 logits [R, V] (row stride ld): loss[R] (fp32), lse[R];
// ignore_index rows get loss 0. Backward writes d(logits) = (softmax - onehot) * g[r] in bf16.
// Row-wise token cross-entropy over bf16 logits with an fp32 log-sum-exp. softcap > 0 applies
// z = softcap * tanh(x / softcap) to every logit first (and its derivative in the backward).
void ce_fwd(const void* logits, long long ld, const int64_t* targets, float* loss, float* lse, long long R, int V,
            long long ignore_index, float softcap, cudaStream_t stream);
void ce_bwd(const void* logits, long long ld, const int64_t* targets, const float* lse, const float* g,
            long long g_stride, void* dlogits, long long R, int V, long long ignore_index, float softcap,
            cudaStream_t stream);

// Multi-tensor AdamW. Tensor descriptors live in device memory (see AdamTensor).
struct AdamTensor {
  float* p;
  const void* g;  // fp32 or bf16 (g_bf16)
  float* m;
  float* v;
  void* shadow;   // optional bf16 copy of the updated parameter (nullptr = none)
  long long n;
  int g_bf16;
  int pad;
};
void adamw_multi(const AdamTensor* tensors, const int* chunk_tensor, const long long* chunk_start, int num_chunks,
                 int chunk_elems, float lr, float beta1, float beta2, float eps, float weight_decay, float bias1,
                 float bias2, const float* grad_scale, cudaStream_t stream);
// Sum of squares of every gradient into out[0] (fp32, zeroed by the caller).
void multi_sumsq(const AdamTensor* tensors, const int* chunk_tensor, const long long* chunk_start, int num_chunks,
                 int chunk_elems, float* out, cudaStream_t stream);
// clip[0] = min(1, max_norm / (sqrt(sumsq[0]) + 1e-6)); norm[0] = sqrt(sumsq[0]).
void clip_coef(const float* sumsq, float max_norm, float* clip, float* norm, cudaStream_t stream);

// Attention operand: [batch, seq, heads, D] bf16 with arbitrary batch / token strides
// (elements) and contiguous heads x D.
struct AttnTensor {
  void* ptr;
  int batch;
  int seq;
  long long s_batch;
  long long s_seq;
};
// D: query / key head dim; Dv: value head dim (0: same as D). Supported pairs: (64, 64),
// (128, 128) and (192, 128) (multi-head latent attention).
void attn_fwd(const AttnTensor& q, const AttnTensor& k, const AttnTensor& v, const AttnTensor& o, float* lse, int H,
              int Hkv, int D, float scale, bool causal, int window, int* status, cudaStream_t stream,
              int* trace = nullptr, int Dv = 0);
// dq_acc: optional fp32 scratch of B*H*S*D floats; with it (and D == Dv == 64) the
// backward runs as one fused kernel that bulk-reduces dQ partials into it, and
// `delta` must then hold 2 * (B*H*S + 128) floats.
void attn_bwd(const AttnTensor& q, const AttnTensor& k, const AttnTensor& v, const AttnTensor& o,
              const AttnTensor& dout, const float* lse, float* delta, const AttnTensor& dq, const AttnTensor& dk,
              const AttnTensor& dv, int H, int Hkv, int D, float scale, bool causal, int window, int* status,
              cudaStream_t stream, float* dq_acc = nullptr, int Dv = 0);

// fp32 -> bf16 cast of n elements.
void cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t stream);

// ---------------------------------------------------------------- peer collectives
// Sharded data parallelism over IPC-mapped peer memory (collective.cu).
constexpr int kMaxRanks = 8;
constexpr int kMaxBuckets = 256;
// Signal array layout (unsigned long long words, one array per rank).
constexpr int kSigReady = 0;                                  // [bucket][src] epoch flags
constexpr int kSigNorm = kSigReady + kMaxBuckets * kMaxRanks;  // [epoch & 1][src] (epoch << 32 | sumsq bits)
constexpr int kSigDone = kSigNorm + 2 * kMaxRanks;            // scatter-completion counter
constexpr int kSigWords = 4096;

// Base addresses of every rank's buffers, as seen from this rank.
struct PeerTable {
  unsigned long long grad[kMaxRanks];    // fp32 gradient buffers
  unsigned long long param[kMaxRanks];   // bf16 weight copies
  unsigned long long signal[kMaxRanks];  // signal arrays
};

// A run of the local shard whose elements map contiguously into the gathered
// weight buffer and share one hyper-parameter group.
struct ShardSegment {
  long long local_off;
  long long gathered_off;
  int group;
  int pad;
};

constexpr int kMaxGroups = 8;
struct AdamHyper {
  float lr[kMaxGroups];
  float beta1[kMaxGroups];
  float beta2[kMaxGroups];
  float eps[kMaxGroups];
  float wd[kMaxGroups];
  float bias1[kMaxGroups];
  float bias2[kMaxGroups];
};

void* sym_alloc(size_t bytes);
void sym_free(void* p);
void ipc_handle(void* p, char out[64]);
void* ipc_open(const char handle[64]);
void ipc_close(void* p);
void rs_bucket(const PeerTable& t, int rank, int world, int bucket, long long bucket_off, long long shard, float* out,
               float* partial, int blocks, unsigned long long epoch, float scale, long long timeout_ns, int* status,
               cudaStream_t stream);
void norm_exchange(const PeerTable& t, int rank, int world, const float* partial, int n_partial,
                   unsigned long long epoch, float max_norm, float* norm_out, float* clip_out, long long timeout_ns,
                   int* status, cudaStream_t stream);
// local_rank >= 0: store the new bf16 weights into that rank's buffer only (sharded weights).
void adamw_scatter(const PeerTable& t, int world, const ShardSegment* segs, int nseg, long long n_local, float* master,
                   float* m1, float* m2, const float* grad, const float* clip, const AdamHyper& hp, int blocks,
                   cudaStream_t stream, int local_rank = -1);
// dst[r * count .. (r + 1) * count) = rank r's param buffer [src_off, src_off + count), r < world (bf16).
void gather_shards(const PeerTable& t, int world, long long src_off, long long count, void* dst, cudaStream_t stream);
void peer_barrier(const unsigned long long* done, unsigned long long target, long long timeout_ns, int* status,
                  cudaStream_t stream);

// ---------------------------------------------------------------- augmentation
// dtype: 0 fp32, 1 bf16, 2 uint8; mode: 0 constant, 1 replicate, 2 reflect. flip may be null.
void pad_crop_flip_cutout(const void* in, void* out, int dtype, int B, int C, int H, int W, int crop, int pad,
                          int mode, float fill, const int32_t* dy, const int32_t* dx, const uint8_t* flip,
                          const int32_t* cy, const int32_t* cx, int cut, cudaStream_t stream);

// ---------------------------------------------------------------- tensor-parallel GEMMs (tp_gemm.cu)
// Signal-array words (same IPC-mapped signal layout as the data-parallel group).
constexpr int kTpSigAgDone = kSigDone + 1;  // peers finished reading this rank's A shard
constexpr int kTpSigRsDone = kSigDone + 2;  // peers finished storing partials into this rank's slots
constexpr int kTpSigRsFree = kSigDone + 3;  // owners finished reducing (slots reusable)
constexpr int kTpSigAgReady = kSigDone + 4;  // [src rank]: epoch whose A shard the source has written

struct TpGemmParams {
  int N, K, m_shard, rank, world;
  long long epoch;       // 1, 2, ... per call of the same kind
  long long timeout_ns;
  int* status;
  void* C;               // all-gather GEMM output [world * m_shard, N]
  long long ldc;
  void* a_full;          // local gather buffer [world * m_shard, K]
  unsigned int* chunk_flags;  // [(world - 1) * m_shard / 128]: pieces copied per chunk (zeroed before each launch)
  int reduce_grid;
  unsigned long long peer_a[kMaxRanks];  // every rank's A shard buffer
  unsigned long long slots[kMaxRanks];   // every rank's receive slots [world, m_shard, N]
  unsigned long long signal[kMaxRanks];
};

// ---------------------------------------------------------------- expert-parallel exchange (ep.cu)
struct EpScatterParams {
  const __nv_bfloat16* src;
  long long ld_src;                 // row stride of src (elements)
  const long long* gather;          // optional: row i reads src[gather[i]]
  const int* dest_rank;             // [rows], -1 = skip
  const long long* dest_row;        // [rows]
  const int* meta;                  // optional metadata word per row
  long long rows;
  int cols;                         // channels (multiple of 8)
  long long dest_cap;               // rows of every rank's receive buffer (rows at or past it are refused)
  unsigned long long buf[kMaxRanks];       // every rank's receive rows
  unsigned long long meta_buf[kMaxRanks];  // every rank's receive metadata
  unsigned long long signal[kMaxRanks];    // every rank's signal words (u64)
  int done_word, free_word;         // signal words: rows of this buffer written / buffer consumed
  int rank, world;
  long long epoch;                  // 1, 2, ... per buffer
  unsigned int* block_counter;      // local, zero between launches
  long long timeout_ns;
  int* status;
};
struct EpSignalParams {
  unsigned long long signal[kMaxRanks];
  int word, world;
};
void ep_scatter(const EpScatterParams& p, cudaStream_t stream);
void ep_collect(const void* buf, const int* meta, void* dst, int* meta_dst, const int* seg_start, const int* totals,
                int segs, int cols, long long cap, cudaStream_t stream);
void ep_signal(const EpSignalParams& p, cudaStream_t stream);

// ---------------------------------------------------------------- expert GEMMs fused with the exchange (ep_gemm.cu)
// Signal words (u64) of an EpGemmGroup's signal array.
constexpr int kEpSigSendReady = 128;                  // [src rank]: epoch whose rows the source's send buffer holds
constexpr int kEpSigSendDone = kEpSigSendReady + kMaxRanks;  // ranks finished pulling from this rank's send buffer
constexpr int kEpSigRecvDone = kEpSigSendDone + 1;    // owners finished pushing into this rank's recv buffer
constexpr int kEpSigRecvFree = kEpSigSendDone + 2;    // sources finished reading their recv buffers

struct EpGemmParams {
  int M, N, K;                  // M = row capacity (multiple of 128)
  void* C;                      // pull epilogue output (local), row stride ldc
  long long ldc;
  const void* aux;              // SwiGLU pre-activation [M, 2H] (epilogue 3 writes it, 4 reads it)
  int swiglu_h;                 // H
  int* status;
  const int* offsets;           // [experts + 1] 128-aligned segment starts of this rank's rows
  int experts, b_rows;          // B stacks experts * b_rows rows
  int epi;                      // pull: 3 (SwiGLU) or 4 (SwiGLU backward); push: 0
  int rank, world;
  long long epoch;              // 1, 2, ... per call of the same kind
  long long timeout_ns;
  // pull: row r of A = row (row_src[r] & 0xFFFFFF) of rank (row_src[r] >> 24)'s send buffer; -1 = zero row
  const int* row_src;
  unsigned long long src[kMaxRanks];
  long long src_rows;           // rows of every send buffer (rows at or past it are refused)
  void* a_local;                // [M, K] gathered A (kept by the caller)
  unsigned int* chunk_flags;    // [M / 128] pieces in place per chunk (zeroed before the launch)
  // push: output row r -> row (row_dst[r] & 0xFFFFFF) of rank (row_dst[r] >> 24)'s recv buffer; -1 = dropped
  const int* row_dst;
  unsigned long long dst[kMaxRanks];
  long long dst_rows;           // rows of every recv buffer (rows at or past it are refused)
  unsigned long long signal[kMaxRanks];
  unsigned int* block_counter;  // local, zero between launches
};
struct EpCombineParams {
  const void* recv;             // local recv rows [tokens * k, cols] bf16
  const float* weights;         // [tokens * k] or null (plain sum)
  void* out;                    // [tokens, cols] bf16
  void* keep;                   // optional copy of the recv rows
  long long tokens;
  int k, cols, rank, world;
  unsigned long long done_target;
  unsigned long long signal[kMaxRanks];
  unsigned int* block_counter;
  long long timeout_ns;
  int* status;
};
void ep_pull_gemm(const EpGemmParams& p, const void* B, long long ldb, bool b_mn, cudaStream_t stream);
void ep_push_gemm(const EpGemmParams& p, const void* A, long long lda, const void* B, long long ldb, bool b_mn,
                  cudaStream_t stream);
void ep_combine(const EpCombineParams& p, cudaStream_t stream);
void ep_expand(const void* dy, const float* w, const void* y, void* out, float* dw, long long slots, int k, int cols,
               cudaStream_t stream);

// Multi-head latent attention decode in latent space (mla_decode.cu): one query per sequence,
// q [B, H, 576] = [q_abs (512) | q_pe (64)] rows, caches c_kv [B, T, 512] and k_pe [B, T, 64]
// (contiguous channels, element strides for rows and sequences); out [B, H, 512] bf16.
struct MlaDecodeParams {
  int B, H, T;
  int splits, tiles_per_split, head_groups;
  const int* lengths;      // [B] keys visible per sequence, or null (all T)
  float scale_log2;        // softmax scale * log2(e)
  __nv_bfloat16* out;
  float* part_o;           // [B, splits, H, 512] (splits > 1)
  float* part_ml;          // [B, splits, H, 2]
  int* status;
};
int mla_decode_head_tile(int H);
void mla_decode_plan(int B, int H, int T, int sm_count, int* splits, int* tiles_per_split);
void mla_decode(const MlaDecodeParams& p, const void* q, const void* ckv, long long c_sb, long long c_st, const void* kpe,
                long long r_sb, long long r_st, cudaStream_t stream);

int tp_gemm_grid(int M, int N);
void tp_ag_gemm(const TpGemmParams& p, const void* a_shard, const void* B, long long ldb, bool b_mn, int grid,
                cudaStream_t stream);
void tp_gemm_rs(const TpGemmParams& p, const void* A, long long lda, const void* B, long long ldb, bool b_mn, void* out,
                long long ldo, int grid, int reduce_grid, unsigned long long done_target, cudaStream_t stream);
void tp_wait(const void* signal_local, int word, unsigned long long target, long long timeout_ns, int* status,
             cudaStream_t stream);

// Decode attention (decode_attention.cu): one query token per sequence over a KV
// cache with per-sequence device lengths. Element strides; cache rows contiguous.
struct DecodeAttnParams {
  const __nv_bfloat16* q;  // [B, H, D]
  const __nv_bfloat16* k;  // [B, Hkv, T, D]
  const __nv_bfloat16* v;
  long long k_sb, k_sh, v_sb, v_sh;
  const int* lengths;      // [B] keys visible to the query, its own included
  __nv_bfloat16* out;      // [B, H, D]
  float* part_acc;         // [B, H, splits, D] (splits > 1)
  float* part_ml;          // [B, H, splits, 2]
  int H, group, T, splits, chunk, window;
  float scale_log2;        // softmax scale * log2(e)
  int* status;             // error word for a wait that runs out
};
int decode_attn_heads_per_cta(int group);
int decode_attn_splits(int B, int H, int group, int T, int sm_count);
void decode_attn(const DecodeAttnParams& p, int B, int D, cudaStream_t stream);

// Gated delta-rule chunk scan (gated_delta.cu): one CTA per (batch, head) walks its
// `n_chunks` chunks of 128 tokens; dk = dv = 128. Every operand is a row-major
// [bh * n_chunks * 128, 128] matrix whose rows are ordered (batch-head, chunk, row).
struct GdnParams {
  int bh, n_chunks;
  const float* ut;     // forward: [rows, dv] fp32 (I + A)^-1 (beta V)
  const float* gc;     // [bh * n_chunks] per-chunk decay gamma_C
  __nv_bfloat16* o;    // forward out: [rows, dv]
  __nv_bfloat16* hs;   // forward out: entry state of every chunk, [bh * n_chunks * dk, dv]
  __nv_bfloat16* us;   // forward out: corrected values U, [rows, dv]
  float* du;           // backward out: dU, [rows, dv]
  float* dhs;          // backward out: gradient of every chunk's exit state, [bh * n_chunks * dk, dv]
  int* status;
};
// Forward: operands W, Qg, Mqk, Kr (bf16); writes o, hs, us.
void gdn_chunk_fwd(const void* w, const void* qg, const void* mqk, const void* kr, const GdnParams& p,
                   cudaStream_t stream);
// Backward: operands Kr, Mqk, dO, Qg, W (bf16); writes du, dhs.
void gdn_chunk_bwd(const void* kr, const void* mqk, const void* dout, const void* qg, const void* w,
                   const GdnParams& p, cudaStream_t stream);

}  // namespace pb

// Python bindings for the sm_100a kernels. The only translation unit that
// includes torch: it validates shapes / dtypes / strides and passes raw
// pointers plus the current CUDA stream to the kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kernels.h"

namespace {

using torch::Tensor;

#define PB_CHECK(cond, msg) TORCH_CHECK(cond, "priml_b200: ", msg)

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  PB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
}

// A side input (weights, tables, targets) as `dtype` on `ref`'s device: a kernel is never handed a
// host pointer or another GPU's memory because a caller built a small tensor elsewhere.
Tensor aux(const Tensor& t, const Tensor& ref, torch::ScalarType dtype) {
  return t.to(ref.device(), dtype).contiguous();
}

// Per-device error status word (int32) that kernels write on a timed-out wait.
Tensor& status_tensor() {
  static std::mutex mu;
  static std::unordered_map<int, Tensor> per_dev;
  int dev = at::cuda::current_device();
  std::lock_guard<std::mutex> g(mu);
  auto it = per_dev.find(dev);
  if (it == per_dev.end()) {
    it = per_dev.emplace(dev, torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, dev))).first;
  }
  return it->second;
}

int* status_ptr() { return status_tensor().data_ptr<int>(); }

// Leading stride of a 2-D view whose last dim is contiguous.
long long row_stride(const Tensor& t) {
  PB_CHECK(t.dim() == 2, "expected a 2-D tensor");
  PB_CHECK(t.stride(1) == 1 || t.size(1) == 1, "last dim must be contiguous");
  return t.size(0) == 1 ? t.size(1) : t.stride(0);
}

// C (op)= A @ B^T in the layouts documented in gemm.cu.
// A: [M, K] (a_mn = false) or [K, M] (a_mn = true); B: [N, K] or [K, N]; C: [M, N].
void gemm(const Tensor& A, const Tensor& B, Tensor& C, bool a_mn, bool b_mn, int64_t epi) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  PB_CHECK(A.scalar_type() == torch::kBFloat16 && B.scalar_type() == torch::kBFloat16, "A and B must be bf16");
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  const int KB = b_mn ? B.size(0) : B.size(1);
  PB_CHECK(K == KB, "contraction sizes differ");
  PB_CHECK(C.size(0) == M && C.size(1) == N, "C has the wrong shape");
  if (epi == 0) PB_CHECK(C.scalar_type() == torch::kBFloat16, "epi 0 writes bf16");
  if (epi == 1 || epi == 2) PB_CHECK(C.scalar_type() == torch::kFloat32, "epi 1/2 write fp32");
  if (M == 0 || N == 0) return;
  if (K == 0) {
    if (epi != 2) C.zero_();
    return;
  }
  const c10::cuda::CUDAGuard guard(A.device());
  pb::gemm_bf16(A.data_ptr(), row_stride(A), a_mn, B.data_ptr(), row_stride(B), b_mn, C.data_ptr(), row_stride(C), M, N,
                K, static_cast<int>(epi), nullptr, 0, status_ptr(), stream());
}

// C = alpha * (A @ B^T) + beta * X in bf16, with X [M, N] bf16 in C's row stride (epilogue 5; 2-CTA
// tiles, so M and N of at least 256). C must not overlap A or B: other tiles still read them.
void gemm_axpby(const Tensor& A, const Tensor& B, const Tensor& X, Tensor& C, bool a_mn, bool b_mn, double alpha,
                double beta) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(X, "X");
  check_cuda(C, "C");
  PB_CHECK(A.scalar_type() == torch::kBFloat16 && B.scalar_type() == torch::kBFloat16 &&
               X.scalar_type() == torch::kBFloat16 && C.scalar_type() == torch::kBFloat16,
           "bf16 tensors");
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  PB_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "contraction sizes differ");
  PB_CHECK(C.size(0) == M && C.size(1) == N && X.sizes() == C.sizes(), "C and X must be [M, N]");
  PB_CHECK(row_stride(X) == row_stride(C), "X and C must share a row stride");
  PB_CHECK(M >= 256 && N >= 256 && N % 8 == 0 && K > 0, "the scaled-add GEMM needs M, N >= 256, N % 8 == 0, K > 0");
  const c10::cuda::CUDAGuard guard(A.device());
  pb::gemm_bf16(A.data_ptr(), row_stride(A), a_mn, B.data_ptr(), row_stride(B), b_mn, C.data_ptr(), row_stride(C), M, N,
                K, 5, X.data_ptr(), 0, status_ptr(), stream(), static_cast<float>(alpha), static_cast<float>(beta));
}

// Batched products over contiguous 3-D stacks: C[b] = alpha * A[b] @ B[b]^T (+ beta * X[b]), in one
// persistent launch (A [b, M, K] or [b, K, M] with a_mn; B [b, N, K] or [b, K, N] with b_mn; C, X [b, M, N]).
void gemm_batched(const Tensor& A, const Tensor& B, Tensor& C, bool a_mn, bool b_mn, const c10::optional<Tensor>& X,
                  double alpha, double beta) {
  for (const Tensor* t : {&A, &B, static_cast<const Tensor*>(&C)}) {
    check_cuda(*t, "operand");
    PB_CHECK(t->dim() == 3 && t->is_contiguous() && t->scalar_type() == torch::kBFloat16,
             "batched GEMM operands must be contiguous bf16 [batch, rows, cols]");
  }
  const int batch = A.size(0);
  const int M = a_mn ? A.size(2) : A.size(1);
  const int K = a_mn ? A.size(1) : A.size(2);
  const int N = b_mn ? B.size(2) : B.size(1);
  PB_CHECK(B.size(0) == batch && C.size(0) == batch, "batch sizes differ");
  PB_CHECK((b_mn ? B.size(1) : B.size(2)) == K, "contraction sizes differ");
  PB_CHECK(C.size(1) == M && C.size(2) == N, "C has the wrong shape");
  PB_CHECK(X.has_value() || alpha == 1.0, "alpha scales the product only together with X");
  const void* aux = nullptr;
  if (X.has_value()) {
    PB_CHECK(X->sizes() == C.sizes() && X->is_contiguous() && X->scalar_type() == torch::kBFloat16, "X like C");
    aux = X->data_ptr();
  }
  if (batch == 0 || M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(A.device());
  pb::gemm_bf16_batched(A.data_ptr(), A.size(2), a_mn, B.data_ptr(), B.size(2), b_mn, C.data_ptr(), N, M, N, K, batch,
                        aux != nullptr ? 5 : 0, aux, status_ptr(), stream(), static_cast<float>(alpha),
                        static_cast<float>(beta));
}

// h = silu(x @ Wg^T) * (x @ Wu^T) with W = [Wg; Wu] ([2H, K]); also writes the bf16 pre-activation gu [M, 2H].
void gemm_swiglu(const Tensor& X, const Tensor& W, Tensor& H, Tensor& GU) {
  check_cuda(X, "X");
  PB_CHECK(X.scalar_type() == torch::kBFloat16 && W.scalar_type() == torch::kBFloat16, "bf16 inputs");
  const int M = X.size(0), K = X.size(1);
  const int two_h = W.size(0);
  PB_CHECK(W.size(1) == K && two_h % 2 == 0, "W must be [2H, K]");
  PB_CHECK(H.size(0) == M && H.size(1) == two_h / 2 && GU.size(0) == M && GU.size(1) == two_h, "bad outputs");
  PB_CHECK(H.is_contiguous() && GU.is_contiguous(), "outputs must be contiguous");
  PB_CHECK((two_h / 2) % 8 == 0, "H must be a multiple of 8");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(X.device());
  pb::gemm_bf16(X.data_ptr(), row_stride(X), false, W.data_ptr(), row_stride(W), false, H.data_ptr(), H.stride(0), M,
                two_h, K, 3, GU.data_ptr(), two_h / 2, status_ptr(), stream());
}

// DGU [M, 2H] = SwiGLU backward of GU [M, 2H] for dh = DY [M, C] @ WD [C, H], computed in the
// GEMM epilogue (dh never reaches memory).
void gemm_swiglu_bwd(const Tensor& DY, const Tensor& WD, const Tensor& GU, Tensor& DGU) {
  check_cuda(DY, "DY");
  PB_CHECK(DY.scalar_type() == torch::kBFloat16 && WD.scalar_type() == torch::kBFloat16 &&
               GU.scalar_type() == torch::kBFloat16 && DGU.scalar_type() == torch::kBFloat16,
           "bf16 tensors");
  const int M = DY.size(0), C = DY.size(1), H = WD.size(1);
  PB_CHECK(WD.size(0) == C, "WD must be [C, H]");
  PB_CHECK(GU.is_contiguous() && DGU.is_contiguous() && GU.size(0) == M && GU.size(1) == 2 * H &&
               DGU.size(0) == M && DGU.size(1) == 2 * H,
           "GU / DGU must be contiguous [M, 2H]");
  PB_CHECK(H % 8 == 0, "H must be a multiple of 8");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(DY.device());
  pb::gemm_bf16(DY.data_ptr(), row_stride(DY), false, WD.data_ptr(), row_stride(WD), true, DGU.data_ptr(), DGU.stride(0),
                M, H, C, 4, GU.data_ptr(), H, status_ptr(), stream());
}

// Grouped expert GEMM (grouped_gemm.cu) over 128-row-aligned expert segments; offsets: int32 [experts + 1].
// mode 0: A [rows, K]; B stacked per expert: [experts * b_rows, K] (K-major) or [experts * b_rows, N] (b_mn);
//         epi 3: B = up weights [experts * 2H, K], C = h [rows, H], aux = gu [rows, 2H] (written);
//         epi 4: B = down weights [experts * C, H] (b_mn), aux = gu (read), C = dgu [rows, 2H].
// mode 1: A [rows, out_rows], B [rows, N] -> C [experts * out_rows, N] fp32 (epi 1 store, 2 accumulate).
void grouped_gemm(const Tensor& A, const Tensor& B, Tensor& C, const Tensor& offsets, bool b_mn, int64_t epi,
                  int64_t mode, int64_t b_rows, const c10::optional<Tensor>& aux, int64_t swiglu_h) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  check_cuda(offsets, "offsets");
  PB_CHECK(A.scalar_type() == torch::kBFloat16 && B.scalar_type() == torch::kBFloat16, "A and B must be bf16");
  PB_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.is_contiguous(), "offsets must be contiguous int32");
  PB_CHECK(C.is_contiguous(), "C must be contiguous");
  const int experts = static_cast<int>(offsets.numel()) - 1;
  const int rows = A.size(0);
  int N = 0, K = 0, out_rows = 0;
  if (mode == 1) {
    out_rows = A.size(1);
    N = B.size(1);
    K = rows;
    PB_CHECK(B.size(0) == rows, "A and B must have the same rows");
    PB_CHECK(C.size(0) == static_cast<int64_t>(experts) * out_rows && C.size(1) == N && C.scalar_type() == torch::kFloat32,
             "C must be fp32 [experts * out_rows, N]");
  } else {
    K = A.size(1);
    if (epi == 3) {
      N = 2 * swiglu_h;
      PB_CHECK(!b_mn && B.size(1) == K && b_rows == 2 * swiglu_h, "epi 3: B = up weights [experts * 2H, K]");
      PB_CHECK(C.size(0) == rows && C.size(1) == swiglu_h && aux.has_value() && aux->is_contiguous() &&
                   aux->size(0) == rows && aux->size(1) == 2 * swiglu_h,
               "epi 3: C = h [rows, H], aux = gu [rows, 2H]");
    } else if (b_mn) {
      N = B.size(1);
      PB_CHECK(b_rows == K, "B N-major: rows per expert must equal K");
    } else {
      N = b_rows;
      PB_CHECK(B.size(1) == K, "B K-major: [experts * N, K]");
    }
    if (epi == 4) {
      PB_CHECK(b_mn && N == swiglu_h && aux.has_value() && aux->size(1) == 2 * swiglu_h && C.size(1) == 2 * swiglu_h,
               "epi 4: B = down weights (N-major), aux = gu, C = dgu [rows, 2H]");
    } else if (epi != 3) {
      PB_CHECK(C.size(0) == rows && C.size(1) == N, "C must be [rows, N]");
    }
    PB_CHECK(B.size(0) == static_cast<int64_t>(experts) * b_rows, "B must stack experts * b_rows rows");
  }
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(A.device());
  pb::grouped_gemm_bf16(A.data_ptr(), row_stride(A), B.data_ptr(), row_stride(B), b_mn, C.data_ptr(), C.stride(0), rows,
                        N, K, offsets.data_ptr<int>(), experts, static_cast<int>(b_rows), static_cast<int>(mode),
                        out_rows, static_cast<int>(epi), aux.has_value() ? aux->data_ptr() : nullptr,
                        static_cast<int>(swiglu_h), status_ptr(), stream());
}

// MXFP8 quantization of bf16 x [R, K]: returns (q uint8, scales uint8 in the blocked layout).
// transpose = false: q [R, K], 32-element blocks along K; true: q [K, R], blocks along R.
std::vector<Tensor> mx_quantize(const Tensor& x, bool transpose) {
  check_cuda(x, "x");
  PB_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x must be bf16 [R, K], rows contiguous");
  const int64_t R = x.size(0), K = x.size(1);
  auto opts = torch::TensorOptions().device(x.device()).dtype(torch::kUInt8);
  Tensor q = transpose ? torch::empty({K, R}, opts) : torch::empty({R, K}, opts);
  Tensor sf = torch::empty({pb::mx_scale_bytes(transpose ? K : R, transpose ? R : K)}, opts);
  if (R == 0 || K == 0) return {q, sf};
  const c10::cuda::CUDAGuard guard(x.device());
  pb::mx_quantize(x.data_ptr(), row_stride(x), q.data_ptr(), sf.data_ptr(), static_cast<int>(R), static_cast<int>(K),
                  transpose, stream());
  return {q, sf};
}

// C [M, N] (op)= MX(A [M, K]) @ MX(B [N, K])^T; epi 0 bf16, 1 fp32, 2 fp32 +=.
void mx_gemm(const Tensor& A, const Tensor& sfa, const Tensor& B, const Tensor& sfb, Tensor& C, int64_t epi) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  PB_CHECK(A.scalar_type() == torch::kUInt8 && B.scalar_type() == torch::kUInt8 && A.is_contiguous() && B.is_contiguous(),
           "A and B must be contiguous uint8 (fp8 E4M3 bytes)");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  PB_CHECK(B.size(1) == K && K % 32 == 0, "A [M, K] and B [N, K] with K a multiple of 32");
  PB_CHECK(sfa.numel() >= pb::mx_scale_bytes(M, K) && sfb.numel() >= pb::mx_scale_bytes(N, K), "scale buffers too small");
  PB_CHECK(C.dim() == 2 && C.size(0) == M && C.size(1) == N && C.is_contiguous(), "C must be contiguous [M, N]");
  if (epi == 0) PB_CHECK(C.scalar_type() == torch::kBFloat16, "epi 0 writes bf16");
  if (epi == 1 || epi == 2) PB_CHECK(C.scalar_type() == torch::kFloat32, "epi 1/2 write fp32");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(A.device());
  pb::mx_gemm(A.data_ptr(), sfa.data_ptr(), B.data_ptr(), sfb.data_ptr(), C.data_ptr(), N, static_cast<int>(M),
              static_cast<int>(N), static_cast<int>(K), static_cast<int>(epi), status_ptr(), stream());
}

std::vector<Tensor> rmsnorm_fwd(const Tensor& x, const c10::optional<Tensor>& w, double eps, bool out_f32) {
  check_cuda(x, "x");
  PB_CHECK(x.is_contiguous(), "x must be contiguous");
  const int C = x.size(-1);
  PB_CHECK(C % 8 == 0, "channels must be a multiple of 8");
  const int R = x.numel() / C;
  auto y = torch::empty(x.sizes(), x.options().dtype(out_f32 ? torch::kFloat32 : torch::kBFloat16));
  auto rstd = torch::empty({R}, x.options().dtype(torch::kFloat32));
  const float* wp = nullptr;
  Tensor wc;
  if (w.has_value() && w->defined()) {
    wc = aux(*w, x, torch::kFloat32);
    wp = wc.data_ptr<float>();
  }
  if (R > 0)
    pb::rmsnorm_fwd(x.data_ptr(), x.scalar_type() == torch::kFloat32, wp, y.data_ptr(), out_f32, rstd.data_ptr<float>(),
                    R, C, static_cast<float>(eps), stream());
  return {y, rstd};
}

std::vector<Tensor> rmsnorm_bwd(const Tensor& dy, const Tensor& x, const c10::optional<Tensor>& w, const Tensor& rstd,
                                bool dx_f32) {
  const int C = x.size(-1);
  const int R = x.numel() / C;
  auto dyc = dy.contiguous();
  auto dx = torch::empty(x.sizes(), x.options().dtype(dx_f32 ? torch::kFloat32 : torch::kBFloat16));
  Tensor dw, wc;
  const float* wp = nullptr;
  float* dwp = nullptr;
  if (w.has_value() && w->defined()) {
    wc = aux(*w, x, torch::kFloat32);
    wp = wc.data_ptr<float>();
    dw = torch::zeros({C}, x.options().dtype(torch::kFloat32));
    dwp = dw.data_ptr<float>();
  }
  if (R > 0)
    pb::rmsnorm_bwd(dyc.data_ptr(), dyc.scalar_type() == torch::kFloat32, x.data_ptr(),
                    x.scalar_type() == torch::kFloat32, wp, rstd.data_ptr<float>(), dx.data_ptr(), dx_f32, dwp, R, C,
                    stream());
  return {dx, dw};
}

// h = x + d (fp32 when either operand is fp32), y = rmsnorm(h); returns {h, y, rstd}.
std::vector<Tensor> add_rmsnorm_fwd(const Tensor& x, const Tensor& d, const c10::optional<Tensor>& w, double eps,
                                    bool out_f32) {
  check_cuda(x, "x");
  check_cuda(d, "d");
  PB_CHECK(x.sizes() == d.sizes(), "x and d must have the same shape");
  PB_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "x must be fp32 or bf16");
  PB_CHECK(d.scalar_type() == torch::kFloat32 || d.scalar_type() == torch::kBFloat16, "d must be fp32 or bf16");
  const int C = x.size(-1);
  PB_CHECK(C % 8 == 0, "channels must be a multiple of 8");
  const int R = x.numel() / C;
  auto xc = x.contiguous();
  auto dc = d.contiguous();
  const bool h_f32 = x.scalar_type() == torch::kFloat32 || d.scalar_type() == torch::kFloat32;
  auto h = torch::empty(x.sizes(), x.options().dtype(h_f32 ? torch::kFloat32 : torch::kBFloat16));
  auto y = torch::empty(x.sizes(), x.options().dtype(out_f32 ? torch::kFloat32 : torch::kBFloat16));
  auto rstd = torch::empty({R}, x.options().dtype(torch::kFloat32));
  const float* wp = nullptr;
  Tensor wc;
  if (w.has_value() && w->defined()) {
    wc = aux(*w, x, torch::kFloat32);
    wp = wc.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  if (R > 0)
    pb::rmsnorm_fwd(xc.data_ptr(), xc.scalar_type() == torch::kFloat32, wp, y.data_ptr(), out_f32,
                    rstd.data_ptr<float>(), R, C, static_cast<float>(eps), stream(), dc.data_ptr(),
                    dc.scalar_type() == torch::kFloat32, h.data_ptr(), h_f32);
  return {h, y, rstd};
}

// Gradient of (h, y) = (x + d, rmsnorm(x + d)) given dy and the residual-path gradient dres
// (optional): returns {dx (dx_f32 selects fp32), dd (dtype code: -1 none, 0 bf16, 1 fp32), dw}.
std::vector<Tensor> add_rmsnorm_bwd(const Tensor& dy, const Tensor& h, const c10::optional<Tensor>& w,
                                    const Tensor& rstd, const c10::optional<Tensor>& dres, bool dx_f32,
                                    int64_t dd_dtype) {
  check_cuda(h, "h");
  const int C = h.size(-1);
  const int R = h.numel() / C;
  auto dyc = dy.contiguous();
  PB_CHECK(dyc.sizes() == h.sizes(), "dy must match h");
  Tensor drc;
  if (dres.has_value() && dres->defined()) {
    drc = dres->contiguous();
    PB_CHECK(drc.sizes() == h.sizes(), "dres must match h");
    PB_CHECK(drc.scalar_type() == torch::kFloat32 || drc.scalar_type() == torch::kBFloat16, "dres must be fp32/bf16");
  }
  auto dx = torch::empty(h.sizes(), h.options().dtype(dx_f32 ? torch::kFloat32 : torch::kBFloat16));
  Tensor dd;
  if (dd_dtype >= 0) dd = torch::empty(h.sizes(), h.options().dtype(dd_dtype == 1 ? torch::kFloat32 : torch::kBFloat16));
  Tensor dw, wc;
  const float* wp = nullptr;
  float* dwp = nullptr;
  if (w.has_value() && w->defined()) {
    wc = aux(*w, h, torch::kFloat32);
    wp = wc.data_ptr<float>();
    dw = torch::zeros({C}, h.options().dtype(torch::kFloat32));
    dwp = dw.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(h.device());
  if (R > 0)
    pb::rmsnorm_bwd(dyc.data_ptr(), dyc.scalar_type() == torch::kFloat32, h.data_ptr(),
                    h.scalar_type() == torch::kFloat32, wp, rstd.data_ptr<float>(), dx.data_ptr(), dx_f32, dwp, R, C,
                    stream(), drc.defined() ? drc.data_ptr() : nullptr,
                    drc.defined() && drc.scalar_type() == torch::kFloat32, dd.defined() ? dd.data_ptr() : nullptr,
                    dd_dtype == 1);
  return {dx, dd, dw};
}

// x: [B, S, H, D] bf16 (last dim contiguous, any other strides). cos/sin: fp32 [S, D/2] contiguous.
Tensor rope(const Tensor& x, const Tensor& cos, const Tensor& sin, double sign) {
  check_cuda(x, "x");
  PB_CHECK(x.dim() == 4 && x.stride(3) == 1 && x.scalar_type() == torch::kBFloat16, "x must be [B,S,H,D] bf16");
  const int B = x.size(0), S = x.size(1), H = x.size(2), D = x.size(3);
  PB_CHECK(D % 4 == 0, "head dim must be a multiple of 4");
  PB_CHECK(cos.numel() == static_cast<long long>(S) * D / 2, "cos must hold S * D/2 values");
  auto y = torch::empty({B, S, H, D}, x.options());
  auto c = aux(cos, x, torch::kFloat32);
  auto s = aux(sin, x, torch::kFloat32);
  if (x.numel() > 0)
    pb::rope_apply(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), y.data_ptr(), B, S, H, D, c.data_ptr<float>(),
                   s.data_ptr<float>(), static_cast<float>(sign), stream());
  return y;
}

Tensor swiglu_fwd(const Tensor& gu) {
  PB_CHECK(gu.is_contiguous() && gu.scalar_type() == torch::kBFloat16, "gu must be contiguous bf16");
  const int H = gu.size(-1) / 2;
  PB_CHECK(H % 8 == 0, "hidden must be a multiple of 8");
  auto sizes = gu.sizes().vec();
  sizes.back() = H;
  auto h = torch::empty(sizes, gu.options());
  const long long R = gu.numel() / (2 * H);
  if (R > 0) pb::swiglu_fwd(gu.data_ptr(), h.data_ptr(), R, H, stream());
  return h;
}

Tensor swiglu_bwd(const Tensor& gu, const Tensor& dh) {
  const int H = gu.size(-1) / 2;
  auto dhc = dh.contiguous();
  auto dgu = torch::empty(gu.sizes(), gu.options());
  const long long R = gu.numel() / (2 * H);
  if (R > 0) pb::swiglu_bwd(gu.data_ptr(), dhc.data_ptr(), dgu.data_ptr(), R, H, stream());
  return dgu;
}

std::vector<Tensor> ce_fwd(const Tensor& logits, const Tensor& targets, int64_t ignore_index, double softcap) {
  PB_CHECK(logits.dim() == 2 && logits.scalar_type() == torch::kBFloat16 && logits.stride(1) == 1, "logits [R, V] bf16");
  const long long R = logits.size(0);
  const int V = logits.size(1);
  auto t = aux(targets, logits, torch::kInt64);
  auto loss = torch::empty({R}, logits.options().dtype(torch::kFloat32));
  auto lse = torch::empty({R}, logits.options().dtype(torch::kFloat32));
  PB_CHECK(logits.stride(0) % 8 == 0, "logits row stride must be a multiple of 8");
  if (R > 0)
    pb::ce_fwd(logits.data_ptr(), logits.stride(0), t.data_ptr<int64_t>(), loss.data_ptr<float>(), lse.data_ptr<float>(),
               R, V, ignore_index, static_cast<float>(softcap), stream());
  return {loss, lse};
}

// Writes d(logits) into `out` (may alias logits).
void ce_bwd(const Tensor& logits, const Tensor& targets, const Tensor& lse, const Tensor& g, Tensor& out,
            int64_t ignore_index, double softcap) {
  const long long R = logits.size(0);
  const int V = logits.size(1);
  auto t = aux(targets, logits, torch::kInt64);
  auto gf = aux(g, logits, torch::kFloat32);
  const long long g_stride = gf.numel() == 1 ? 0 : 1;
  PB_CHECK(out.stride(0) == logits.stride(0), "out must share the logits layout");
  if (R > 0)
    pb::ce_bwd(logits.data_ptr(), logits.stride(0), t.data_ptr<int64_t>(), lse.data_ptr<float>(), gf.data_ptr<float>(),
               g_stride, out.data_ptr(), R, V, ignore_index, static_cast<float>(softcap), stream());
}

// Multi-tensor optimizer plan: device-resident tensor table + chunk map, built once per parameter set.
class MultiTensorPlan {
 public:
  MultiTensorPlan(std::vector<Tensor> params, std::vector<Tensor> grads, std::vector<Tensor> m, std::vector<Tensor> v,
                  std::vector<c10::optional<Tensor>> shadows, int64_t chunk)
      : params_(params), grads_(grads), m_(m), v_(v), chunk_(static_cast<int>(chunk)) {
    PB_CHECK(params.size() == grads.size() && params.size() == m.size() && params.size() == v.size(), "list sizes");
    std::vector<pb::AdamTensor> table;
    std::vector<int> ct;
    std::vector<long long> cs;
    for (size_t i = 0; i < params.size(); ++i) {
      PB_CHECK(params[i].scalar_type() == torch::kFloat32 && params[i].is_contiguous(), "params must be fp32 contiguous");
      PB_CHECK(grads[i].is_contiguous() && grads[i].numel() == params[i].numel(), "grad layout");
      pb::AdamTensor a{};
      a.p = params[i].data_ptr<float>();
      a.g = grads[i].data_ptr();
      a.g_bf16 = grads[i].scalar_type() == torch::kBFloat16;
      a.m = m[i].data_ptr<float>();
      a.v = v[i].data_ptr<float>();
      a.shadow = nullptr;
      if (i < shadows.size() && shadows[i].has_value() && shadows[i]->defined()) {
        PB_CHECK(shadows[i]->scalar_type() == torch::kBFloat16 && shadows[i]->is_contiguous(), "shadow bf16");
        a.shadow = shadows[i]->data_ptr();
        shadows_.push_back(*shadows[i]);
      }
      a.n = params[i].numel();
      table.push_back(a);
      for (long long s = 0; s < a.n; s += chunk_) {
        ct.push_back(static_cast<int>(i));
        cs.push_back(s);
      }
    }
    num_chunks_ = static_cast<int>(ct.size());
    auto dev = params.empty() ? torch::Device(torch::kCUDA) : params[0].device();
    table_ = torch::empty({static_cast<long long>(table.size() * sizeof(pb::AdamTensor))},
                          torch::dtype(torch::kUInt8).device(dev));
    if (!table.empty()) {
      auto host = torch::from_blob(table.data(), {table_.numel()}, torch::kUInt8).clone();
      table_.copy_(host);
      chunk_tensor_ = torch::from_blob(ct.data(), {num_chunks_}, torch::kInt32).to(dev);
      chunk_start_ = torch::from_blob(cs.data(), {num_chunks_}, torch::kInt64).to(dev);
    }
  }

  void adamw(double lr, double beta1, double beta2, double eps, double wd, double bias1, double bias2,
             const c10::optional<Tensor>& grad_scale) {
    if (num_chunks_ == 0) return;
    const float* gs = grad_scale.has_value() && grad_scale->defined() ? grad_scale->data_ptr<float>() : nullptr;
    pb::adamw_multi(reinterpret_cast<const pb::AdamTensor*>(table_.data_ptr()), chunk_tensor_.data_ptr<int>(),
                    reinterpret_cast<const long long*>(chunk_start_.data_ptr<int64_t>()), num_chunks_, chunk_, lr, beta1, beta2, eps, wd, bias1, bias2, gs,
                    stream());
  }

  // Returns [norm, clip] (fp32 device tensors) without a host sync.
  std::vector<Tensor> grad_norm_clip(double max_norm) {
    auto opts = torch::dtype(torch::kFloat32).device(params_.empty() ? torch::Device(torch::kCUDA) : params_[0].device());
    auto sumsq = torch::zeros({1}, opts);
    auto norm = torch::empty({1}, opts);
    auto clip = torch::empty({1}, opts);
    if (num_chunks_ > 0)
      pb::multi_sumsq(reinterpret_cast<const pb::AdamTensor*>(table_.data_ptr()), chunk_tensor_.data_ptr<int>(),
                      reinterpret_cast<const long long*>(chunk_start_.data_ptr<int64_t>()), num_chunks_, chunk_, sumsq.data_ptr<float>(), stream());
    pb::clip_coef(sumsq.data_ptr<float>(), static_cast<float>(max_norm), clip.data_ptr<float>(), norm.data_ptr<float>(),
                  stream());
    return {norm, clip};
  }

  int64_t num_chunks() const { return num_chunks_; }

 private:
  std::vector<Tensor> params_, grads_, m_, v_, shadows_;
  Tensor table_, chunk_tensor_, chunk_start_;
  int num_chunks_ = 0;
  int chunk_;
};

Tensor cast_bf16(const Tensor& x, c10::optional<Tensor> out) {
  PB_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "x must be contiguous fp32");
  Tensor y = out.has_value() ? *out : torch::empty(x.sizes(), x.options().dtype(torch::kBFloat16));
  if (x.numel() > 0) pb::cast_f32_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), stream());
  return y;
}

pb::AttnTensor attn_view(const Tensor& t, const char* name) {
  PB_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16, std::string(name) + " must be CUDA bf16");
  PB_CHECK(t.dim() == 4, std::string(name) + " must be [B, S, H, D]");
  PB_CHECK(t.stride(3) == 1 && t.stride(2) == t.size(3), std::string(name) + " needs contiguous heads x head_dim");
  PB_CHECK((t.stride(1) * 2) % 16 == 0 && (t.stride(0) * 2) % 16 == 0, std::string(name) + " strides must be 16-byte aligned");
  PB_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, std::string(name) + " must be 16-byte aligned");
  return pb::AttnTensor{t.data_ptr(), static_cast<int>(t.size(0)), static_cast<int>(t.size(1)), t.stride(0), t.stride(1)};
}

// (o [B,S,H,D] bf16, lse [B,H,S] fp32)
std::vector<Tensor> attn_fwd(const Tensor& q, const Tensor& k, const Tensor& v, double scale, bool causal,
                             int64_t window, const c10::optional<Tensor>& trace) {
  const int D = q.size(3), Dv = v.size(3), H = q.size(2), Hkv = k.size(2);
  PB_CHECK((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 192 && Dv == 128),
           "head dims (query/key, value) must be (64, 64), (128, 128) or (192, 128)");
  PB_CHECK(k.size(3) == D && H % Hkv == 0 && v.size(2) == Hkv, "q/k/v shapes");
  PB_CHECK(D != 192 || !trace.has_value(), "the progress trace covers head dims 64 and 128 only");
  PB_CHECK(k.size(0) == q.size(0) && v.size(1) == k.size(1), "batch / key lengths");
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({q.size(0), q.size(1), H, Dv}, q.options());
  // 128 floats of tail padding: the backward reads lse rows in 512-byte bulk copies.
  const long long n_lse = q.size(0) * H * q.size(1);
  auto lse = torch::empty({n_lse + 128}, q.options().dtype(torch::kFloat32)).narrow(0, 0, n_lse).view({q.size(0), H, q.size(1)});
  if (q.numel() == 0) return {o, lse};
  pb::attn_fwd(attn_view(q, "q"), attn_view(k, "k"), attn_view(v, "v"), attn_view(o, "o"), lse.data_ptr<float>(), H, Hkv,
               D, static_cast<float>(scale), causal, static_cast<int>(window), status_ptr(), stream(),
               trace.has_value() ? trace->data_ptr<int>() : nullptr, Dv);
  return {o, lse};
}

// Gated delta-rule chunk scan. Operands are contiguous [bh, n, 128, 128] (bf16, Ut fp32),
// gc is fp32 [bh, n]. Returns (O bf16, entry states bf16, U bf16), each [bh, n, 128, 128].
void check_gdn(const Tensor& t, const Tensor& ref, torch::ScalarType dtype, const char* name) {
  PB_CHECK(t.is_cuda() && t.scalar_type() == dtype && t.is_contiguous(), std::string(name) + " has the wrong dtype or layout");
  PB_CHECK(t.device() == ref.device(), std::string(name) + " is on another device");
  PB_CHECK(t.dim() == 4 && t.size(0) == ref.size(0) && t.size(1) == ref.size(1) && t.size(2) == 128 && t.size(3) == 128,
           std::string(name) + " must be [bh, n, 128, 128]");
}

std::vector<Tensor> gdn_fwd(const Tensor& w, const Tensor& ut, const Tensor& qg, const Tensor& mqk, const Tensor& kr,
                            const Tensor& gc) {
  check_gdn(w, w, torch::kBFloat16, "W");
  check_gdn(ut, w, torch::kFloat32, "Ut");
  check_gdn(qg, w, torch::kBFloat16, "Qg");
  check_gdn(mqk, w, torch::kBFloat16, "Mqk");
  check_gdn(kr, w, torch::kBFloat16, "Kr");
  PB_CHECK(gc.is_cuda() && gc.scalar_type() == torch::kFloat32 && gc.is_contiguous() && gc.numel() == w.size(0) * w.size(1),
           "gc must be contiguous fp32 [bh, n]");
  const c10::cuda::CUDAGuard guard(w.device());
  auto o = torch::empty_like(w);
  auto hs = torch::empty_like(w);
  auto us = torch::empty_like(w);
  if (w.numel() == 0) return {o, hs, us};
  pb::GdnParams p{};
  p.bh = w.size(0);
  p.n_chunks = w.size(1);
  p.ut = ut.data_ptr<float>();
  p.gc = gc.data_ptr<float>();
  p.o = static_cast<__nv_bfloat16*>(o.data_ptr());
  p.hs = static_cast<__nv_bfloat16*>(hs.data_ptr());
  p.us = static_cast<__nv_bfloat16*>(us.data_ptr());
  p.status = status_ptr();
  pb::gdn_chunk_fwd(w.data_ptr(), qg.data_ptr(), mqk.data_ptr(), kr.data_ptr(), p, stream());
  return {o, hs, us};
}

// Backward of gdn_fwd's scan: returns (dU fp32, gradient of every chunk's exit state fp32).
std::vector<Tensor> gdn_bwd(const Tensor& kr, const Tensor& mqk, const Tensor& dout, const Tensor& qg, const Tensor& w,
                            const Tensor& gc) {
  check_gdn(kr, kr, torch::kBFloat16, "Kr");
  check_gdn(mqk, kr, torch::kBFloat16, "Mqk");
  check_gdn(dout, kr, torch::kBFloat16, "dO");
  check_gdn(qg, kr, torch::kBFloat16, "Qg");
  check_gdn(w, kr, torch::kBFloat16, "W");
  PB_CHECK(gc.is_cuda() && gc.scalar_type() == torch::kFloat32 && gc.is_contiguous() && gc.numel() == kr.size(0) * kr.size(1),
           "gc must be contiguous fp32 [bh, n]");
  const c10::cuda::CUDAGuard guard(kr.device());
  auto du = torch::empty(kr.sizes(), kr.options().dtype(torch::kFloat32));
  auto dhs = torch::empty(kr.sizes(), kr.options().dtype(torch::kFloat32));
  if (kr.numel() == 0) return {du, dhs};
  pb::GdnParams p{};
  p.bh = kr.size(0);
  p.n_chunks = kr.size(1);
  p.gc = gc.data_ptr<float>();
  p.du = du.data_ptr<float>();
  p.dhs = dhs.data_ptr<float>();
  p.status = status_ptr();
  pb::gdn_chunk_bwd(kr.data_ptr(), mqk.data_ptr(), dout.data_ptr(), qg.data_ptr(), w.data_ptr(), p, stream());
  return {du, dhs};
}

// Decode attention: q [B, H, D] over caches [B, Hkv, T, D] (rows contiguous) with
// int32 lengths [B] on the device; returns [B, H, D].
// Multi-head latent attention decode in latent space (mla_decode.cu). q [B, H, 576] = [q_abs | q_pe]
// (contiguous bf16); c_kv [B, T, 512] and k_pe [B, T, 64] bf16 with contiguous channels and 16-byte
// aligned row / sequence strides; lengths int32 [B] (keys visible per sequence) or none (all T).
// Returns the attention-weighted latent rows [B, H, 512] (bf16).
Tensor mla_decode(const Tensor& q, const Tensor& ckv, const Tensor& kpe, const c10::optional<Tensor>& lengths,
                  double scale) {
  check_cuda(q, "q");
  check_cuda(ckv, "c_kv");
  check_cuda(kpe, "k_pe");
  PB_CHECK(q.scalar_type() == torch::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == 576,
           "q must be contiguous bf16 [B, H, 576]");
  const int64_t B = q.size(0), H = q.size(1);
  PB_CHECK(ckv.scalar_type() == torch::kBFloat16 && ckv.dim() == 3 && ckv.size(0) == B && ckv.size(2) == 512 &&
               ckv.stride(2) == 1 && ckv.stride(1) % 8 == 0 && ckv.stride(0) % 8 == 0,
           "c_kv must be bf16 [B, T, 512] with contiguous channels and 16-byte aligned strides");
  const int64_t T = ckv.size(1);
  PB_CHECK(kpe.scalar_type() == torch::kBFloat16 && kpe.dim() == 3 && kpe.size(0) == B && kpe.size(1) == T &&
               kpe.size(2) == 64 && kpe.stride(2) == 1 && kpe.stride(1) % 8 == 0 && kpe.stride(0) % 8 == 0,
           "k_pe must be bf16 [B, T, 64] with contiguous channels and 16-byte aligned strides");
  PB_CHECK(T >= 1 && T < (1LL << 31) && B * H < (1LL << 31), "sizes out of range");
  auto out = torch::empty({B, H, 512}, q.options());
  pb::MlaDecodeParams p{};
  p.B = static_cast<int>(B);
  p.H = static_cast<int>(H);
  p.T = static_cast<int>(T);
  const int nh = pb::mla_decode_head_tile(p.H);
  p.head_groups = (p.H + nh - 1) / nh;
  pb::mla_decode_plan(p.B, p.H, p.T, pb::device_sm_count(), &p.splits, &p.tiles_per_split);
  Tensor part_o, part_ml, lens;
  if (lengths.has_value()) {
    PB_CHECK(lengths->numel() == B, "lengths must have one entry per sequence");
    lens = lengths->to(q.device(), torch::kInt32).contiguous();
    p.lengths = lens.data_ptr<int>();
  }
  if (p.splits > 1) {
    part_o = torch::empty({B, p.splits, H, 512}, q.options().dtype(torch::kFloat32));
    part_ml = torch::empty({B, p.splits, H, 2}, q.options().dtype(torch::kFloat32));
    p.part_o = part_o.data_ptr<float>();
    p.part_ml = part_ml.data_ptr<float>();
  }
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.status = status_ptr();
  const c10::cuda::CUDAGuard guard(q.device());
  pb::mla_decode(p, q.data_ptr(), ckv.data_ptr(), ckv.stride(0), ckv.stride(1), kpe.data_ptr(), kpe.stride(0),
                 kpe.stride(1), stream());
  return out;
}

Tensor decode_attn(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& lengths, double scale,
                   int64_t window) {
  PB_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.is_contiguous(),
           "q must be contiguous CUDA bf16 [B, H, D]");
  const int B = q.size(0), H = q.size(1), D = q.size(2);
  PB_CHECK(D == 64 || D == 128, "decode attention covers head dims 64 and 128");
  for (const Tensor* t : {&k, &v}) {
    PB_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->dim() == 4, "caches must be CUDA bf16 [B, Hkv, T, D]");
    PB_CHECK(t->size(0) == B && t->size(3) == D && t->stride(3) == 1 && t->stride(2) == D,
             "cache rows must be contiguous with the query's head dim");
    PB_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0 && t->stride(0) % 8 == 0 && t->stride(1) % 8 == 0,
             "cache base and strides must be 16-byte aligned");
  }
  PB_CHECK(k.sizes() == v.sizes(), "k and v caches differ in shape");
  const int Hkv = k.size(1), T = k.size(2);
  PB_CHECK(Hkv > 0 && H % Hkv == 0, "query heads must be a multiple of the KV heads");
  PB_CHECK(lengths.is_cuda() && lengths.scalar_type() == torch::kInt32 && lengths.numel() == B && lengths.is_contiguous(),
           "lengths must be contiguous int32 [B] on the device");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty_like(q);
  if (q.numel() == 0) return out;
  const int group = H / Hkv;
  const int splits = pb::decode_attn_splits(B, H, group, T, pb::device_sm_count());
  Tensor part_acc, part_ml;
  if (splits > 1) {
    part_acc = torch::empty({static_cast<long long>(B) * H * splits * D}, q.options().dtype(torch::kFloat32));
    part_ml = torch::empty({static_cast<long long>(B) * H * splits * 2}, q.options().dtype(torch::kFloat32));
  }
  pb::DecodeAttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = static_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = static_cast<const __nv_bfloat16*>(v.data_ptr());
  p.k_sb = k.stride(0);
  p.k_sh = k.stride(1);
  p.v_sb = v.stride(0);
  p.v_sh = v.stride(1);
  p.lengths = lengths.data_ptr<int>();
  p.out = static_cast<__nv_bfloat16*>(out.data_ptr());
  p.part_acc = splits > 1 ? part_acc.data_ptr<float>() : nullptr;
  p.part_ml = splits > 1 ? part_ml.data_ptr<float>() : nullptr;
  p.H = H;
  p.group = group;
  p.T = T;
  p.splits = splits;
  p.chunk = (T + splits - 1) / splits;
  p.window = static_cast<int>(window);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.status = status_ptr();
  pb::decode_attn(p, B, D, stream());
  return out;
}

// (dq, dk, dv) in the layouts of q / k / v (contiguous).
std::vector<Tensor> attn_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& dout,
                             const Tensor& lse, double scale, bool causal, int64_t window) {
  const int D = q.size(3), Dv = v.size(3), H = q.size(2), Hkv = k.size(2);
  PB_CHECK((D == 64 && Dv == 64) || (D == 128 && Dv == 128) || (D == 192 && Dv == 128),
           "head dims (query/key, value) must be (64, 64), (128, 128) or (192, 128)");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = torch::empty({q.size(0), q.size(1), H, D}, q.options());
  auto dk = torch::empty({k.size(0), k.size(1), Hkv, D}, k.options());
  auto dv = torch::empty({v.size(0), v.size(1), Hkv, Dv}, v.options());
  const long long n_rows = q.size(0) * H * q.size(1);
  // delta rows + 128 floats of padding; the fused D = 64 path pads each (b, h) row of delta to a
  // multiple of 4 floats and keeps -lse*log2(e) after it in the same layout.
  const long long n_vec = q.size(0) * H * ((q.size(1) + 3) / 4 * 4);
  const bool fused = D == 64 && Dv == 64;
  auto delta = torch::empty({fused ? 2 * (n_vec + 128) : n_rows + 128}, q.options().dtype(torch::kFloat32));
  PB_CHECK(lse.is_contiguous() && lse.numel() == n_rows, "lse must be the forward's [B, H, S] output");
  auto doc = dout.stride(3) == 1 && dout.stride(2) == Dv ? dout : dout.contiguous();
  if (q.numel() == 0) return {dq, dk, dv};
  // D = 64 runs the fused dK/dV/dQ kernel, which bulk-reduces dQ into fp32 scratch.
  Tensor dq_acc;
  if (fused) dq_acc = torch::empty({n_rows * D}, q.options().dtype(torch::kFloat32));
  pb::attn_bwd(attn_view(q, "q"), attn_view(k, "k"), attn_view(v, "v"), attn_view(o, "o"), attn_view(doc, "dout"),
               lse.data_ptr<float>(), delta.data_ptr<float>(), attn_view(dq, "dq"), attn_view(dk, "dk"),
               attn_view(dv, "dv"), H, Hkv, D, static_cast<float>(scale), causal, static_cast<int>(window),
               status_ptr(), stream(), dq_acc.defined() ? dq_acc.data_ptr<float>() : nullptr, Dv);
  return {dq, dk, dv};
}

int64_t read_status(bool reset) {
  auto& s = status_tensor();
  const int64_t v = s.item<int>();
  if (reset && v != 0) s.zero_();
  return v;
}


// Peer-shared weight / gradient / signal buffers of one data-parallel rank plus
// the fused collective launches over them (collective.cu). The buffers are
// cudaMalloc'd (IPC needs an allocation base) and exposed as tensors that keep
// the allocation alive; peer buffers are mapped with cudaIpcOpenMemHandle.
class PeerGroup {
 public:
  PeerGroup(int64_t rank, int64_t world, int64_t param_elems, int64_t grad_elems)
      : rank_(rank), world_(world), device_(at::cuda::current_device()) {
    PB_CHECK(world >= 1 && world <= pb::kMaxRanks, "world size must be 1..8");
    PB_CHECK(rank >= 0 && rank < world, "rank out of range");
    local_ = std::make_shared<Local>();
    local_->param = pb::sym_alloc(std::max<int64_t>(param_elems, 8) * 2);
    local_->grad = pb::sym_alloc(std::max<int64_t>(grad_elems, 4) * 4);
    local_->signal = pb::sym_alloc(pb::kSigWords * 8);
    auto opts = torch::TensorOptions().device(torch::kCUDA, device_);
    auto keep = local_;
    param_ = torch::from_blob(local_->param, {param_elems}, [keep](void*) {}, opts.dtype(torch::kBFloat16));
    grad_ = torch::from_blob(local_->grad, {grad_elems}, [keep](void*) {}, opts.dtype(torch::kFloat32));
    signal_ = torch::from_blob(local_->signal, {pb::kSigWords}, [keep](void*) {}, opts.dtype(torch::kInt64));
    std::memset(&table_, 0, sizeof(table_));
  }

  ~PeerGroup() {
    for (void* p : opened_) pb::ipc_close(p);
  }

  py::bytes handles() const {
    char buf[192];
    pb::ipc_handle(local_->param, buf);
    pb::ipc_handle(local_->grad, buf + 64);
    pb::ipc_handle(local_->signal, buf + 128);
    return py::bytes(buf, 192);
  }

  // `all` holds every rank's handles() in rank order.
  void open(const std::vector<std::string>& all) {
    PB_CHECK(static_cast<int64_t>(all.size()) == world_, "need one handle record per rank");
    const c10::cuda::CUDAGuard guard(device_);
    for (int64_t r = 0; r < world_; ++r) {
      PB_CHECK(all[r].size() == 192, "bad handle record");
      if (r == rank_) {
        table_.param[r] = reinterpret_cast<unsigned long long>(local_->param);
        table_.grad[r] = reinterpret_cast<unsigned long long>(local_->grad);
        table_.signal[r] = reinterpret_cast<unsigned long long>(local_->signal);
        continue;
      }
      void* p = pb::ipc_open(all[r].data());
      void* g = pb::ipc_open(all[r].data() + 64);
      void* s = pb::ipc_open(all[r].data() + 128);
      opened_.insert(opened_.end(), {p, g, s});
      table_.param[r] = reinterpret_cast<unsigned long long>(p);
      table_.grad[r] = reinterpret_cast<unsigned long long>(g);
      table_.signal[r] = reinterpret_cast<unsigned long long>(s);
    }
    opened_ok_ = true;
  }

  Tensor param() const { return param_; }
  Tensor grad() const { return grad_; }
  Tensor signal() const { return signal_; }

  void reduce_scatter(int64_t bucket, int64_t bucket_off, int64_t shard, Tensor& out, Tensor& partial, int64_t epoch,
                      double scale, double timeout_s) {
    PB_CHECK(opened_ok_, "open() the peer group first");
    PB_CHECK(out.is_contiguous() && out.scalar_type() == torch::kFloat32 && out.numel() == shard, "out shard");
    PB_CHECK(partial.is_contiguous() && partial.scalar_type() == torch::kFloat32, "partial sums");
    PB_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 && bucket_off % 4 == 0, "16-byte alignment");
    pb::rs_bucket(table_, rank_, world_, bucket, bucket_off, shard, out.data_ptr<float>(), partial.data_ptr<float>(),
                  partial.numel(), static_cast<unsigned long long>(epoch), static_cast<float>(scale),
                  static_cast<long long>(timeout_s * 1e9), status_ptr(), stream());
  }

  void norm_exchange(const Tensor& partial, int64_t epoch, double max_norm, Tensor& norm, Tensor& clip,
                     double timeout_s) {
    PB_CHECK(opened_ok_, "open() the peer group first");
    pb::norm_exchange(table_, rank_, world_, partial.data_ptr<float>(), partial.numel(),
                      static_cast<unsigned long long>(epoch), static_cast<float>(max_norm), norm.data_ptr<float>(),
                      clip.data_ptr<float>(), static_cast<long long>(timeout_s * 1e9), status_ptr(), stream());
  }

  // segs: int64 [n, 3] = (local_off, gathered_off, group); hyper: 7 lists of per-group floats.
  void adamw_scatter(const Tensor& segs, Tensor& master, Tensor& m1, Tensor& m2, const Tensor& grad,
                     c10::optional<Tensor> clip, const std::vector<std::vector<double>>& hyper, int64_t blocks,
                     bool local_only) {
    PB_CHECK(opened_ok_, "open() the peer group first");
    PB_CHECK(segs.is_cuda() && segs.scalar_type() == torch::kInt64 && segs.dim() == 2 && segs.size(1) == 3, "segments");
    PB_CHECK(hyper.size() == 7, "hyper = [lr, beta1, beta2, eps, wd, bias1, bias2]");
    const int64_t n = master.numel();
    for (const Tensor* t : {static_cast<const Tensor*>(&master), static_cast<const Tensor*>(&m1), static_cast<const Tensor*>(&m2), &grad})
      PB_CHECK(t->is_contiguous() && t->scalar_type() == torch::kFloat32 && t->numel() == n, "fp32 shard tensors");
    pb::AdamHyper hp{};
    float* dst[7] = {hp.lr, hp.beta1, hp.beta2, hp.eps, hp.wd, hp.bias1, hp.bias2};
    for (int k = 0; k < 7; ++k) {
      PB_CHECK(hyper[k].size() <= static_cast<size_t>(pb::kMaxGroups), "at most 8 parameter groups");
      for (size_t g = 0; g < hyper[k].size(); ++g) dst[k][g] = static_cast<float>(hyper[k][g]);
    }
    pb::adamw_scatter(table_, world_, reinterpret_cast<const pb::ShardSegment*>(segs.data_ptr()), segs.size(0), n,
                      master.data_ptr<float>(), m1.data_ptr<float>(), m2.data_ptr<float>(), grad.data_ptr<float>(),
                      clip.has_value() ? clip->data_ptr<float>() : nullptr, hp, blocks, stream(),
                      local_only ? static_cast<int>(rank_) : -1);
  }

  // Sharded weights: dst (bf16, world * count elements) = every rank's param[src_off, src_off + count)
  // in rank order, copied on the current stream by the copy engines.
  void gather_shards(int64_t src_off, int64_t count, Tensor& dst) {
    PB_CHECK(opened_ok_, "open() the peer group first");
    PB_CHECK(dst.is_cuda() && dst.scalar_type() == torch::kBFloat16 && dst.is_contiguous() &&
                 dst.numel() == world_ * count,
             "dst must be contiguous bf16 of world * count elements");
    PB_CHECK(src_off >= 0 && src_off + count <= param_.numel(), "shard range outside the param buffer");
    pb::gather_shards(table_, static_cast<int>(world_), src_off, count, dst.data_ptr(), stream());
  }

  void barrier(int64_t target, double timeout_s) {
    PB_CHECK(opened_ok_, "open() the peer group first");
    pb::peer_barrier(reinterpret_cast<const unsigned long long*>(local_->signal) + pb::kSigDone,
                     static_cast<unsigned long long>(target), static_cast<long long>(timeout_s * 1e9), status_ptr(),
                     stream());
  }

 private:
  struct Local {
    void* param = nullptr;
    void* grad = nullptr;
    void* signal = nullptr;
    ~Local() {
      pb::sym_free(param);
      pb::sym_free(grad);
      pb::sym_free(signal);
    }
  };
  int64_t rank_, world_;
  int device_;
  std::shared_ptr<Local> local_;
  Tensor param_, grad_, signal_;
  pb::PeerTable table_;
  std::vector<void*> opened_;
  bool opened_ok_ = false;
};

Tensor status_tensor_py() { return status_tensor(); }
// Tensor-parallel group of the fused all-gather GEMM / GEMM reduce-scatter (tp_gemm.cu):
// IPC-mapped A-shard buffer, receive slots and signal words of every rank, plus the
// host-side epochs and counter targets of the two operations.
class TpGroup {
 public:
  TpGroup(int64_t rank, int64_t world, int64_t shard_elems, int64_t slot_elems, int64_t max_chunks, double timeout_s)
      : rank_(rank), world_(world), timeout_ns_(static_cast<long long>(timeout_s * 1e9)),
        device_(at::cuda::current_device()) {
    PB_CHECK(world >= 1 && world <= pb::kMaxRanks, "world size must be 1..8");
    local_ = std::make_shared<Local>();
    local_->shard = pb::sym_alloc(std::max<int64_t>(shard_elems, 8) * 2);
    local_->slots = pb::sym_alloc(std::max<int64_t>(slot_elems, 8) * 2);
    local_->signal = pb::sym_alloc(pb::kSigWords * 8);
    auto opts = torch::TensorOptions().device(torch::kCUDA, device_);
    auto keep = local_;
    shard_ = torch::from_blob(local_->shard, {shard_elems}, [keep](void*) {}, opts.dtype(torch::kBFloat16));
    flags_ = torch::zeros({std::max<int64_t>(max_chunks, 1)}, opts.dtype(torch::kInt32));
    std::memset(&base_, 0, sizeof(base_));
    slot_bytes_ = std::max<int64_t>(slot_elems, 8) * 2;
  }
  ~TpGroup() {
    for (void* p : opened_) pb::ipc_close(p);
  }
  py::bytes handles() const {
    char buf[192];
    pb::ipc_handle(local_->shard, buf);
    pb::ipc_handle(local_->slots, buf + 64);
    pb::ipc_handle(local_->signal, buf + 128);
    return py::bytes(buf, 192);
  }
  void open(const std::vector<std::string>& all) {
    PB_CHECK(static_cast<int64_t>(all.size()) == world_, "need one handle record per rank");
    const c10::cuda::CUDAGuard guard(device_);
    for (int64_t r = 0; r < world_; ++r) {
      if (r == rank_) {
        base_.peer_a[r] = reinterpret_cast<unsigned long long>(local_->shard);
        base_.slots[r] = reinterpret_cast<unsigned long long>(local_->slots);
        base_.signal[r] = reinterpret_cast<unsigned long long>(local_->signal);
        continue;
      }
      void* a = pb::ipc_open(all[r].data());
      void* sl = pb::ipc_open(all[r].data() + 64);
      void* sg = pb::ipc_open(all[r].data() + 128);
      opened_.insert(opened_.end(), {a, sl, sg});
      base_.peer_a[r] = reinterpret_cast<unsigned long long>(a);
      base_.slots[r] = reinterpret_cast<unsigned long long>(sl);
      base_.signal[r] = reinterpret_cast<unsigned long long>(sg);
    }
    opened_ok_ = true;
  }
  Tensor shard() const { return shard_; }

  // Wait (on the stream) until every peer has finished reading this rank's previous shard.
  void wait_shard_free() {
    PB_CHECK(opened_ok_, "open() first");
    if (ag_target_ == 0) return;
    pb::tp_wait(local_->signal, pb::kTpSigAgDone, ag_target_, timeout_ns_, status_ptr(), stream());
  }

  // C [world*m_shard, N] = AllGather(shard[:m_shard*K]) @ B^T ; B [N, K] (b_mn: [K, N]); a_full [world*m_shard, K].
  void ag_gemm(const Tensor& B, bool b_mn, int64_t m_shard, int64_t K, Tensor& C, Tensor& a_full) {
    PB_CHECK(opened_ok_, "open() first");
    const int64_t N = b_mn ? B.size(1) : B.size(0);
    PB_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "B has the wrong K");
    PB_CHECK(m_shard % 128 == 0 && m_shard * K <= shard_.numel(), "m_shard must be a multiple of 128 and fit the shard buffer");
    PB_CHECK(C.is_contiguous() && C.size(0) == m_shard * world_ && C.size(1) == N && C.scalar_type() == torch::kBFloat16, "C");
    PB_CHECK(a_full.is_contiguous() && a_full.numel() >= m_shard * world_ * K && a_full.scalar_type() == torch::kBFloat16, "a_full");
    const int64_t chunks = (world_ - 1) * (m_shard / 128);
    PB_CHECK(chunks <= flags_.numel(), "too many chunks for the flag buffer");
    pb::TpGemmParams p = base_;
    p.N = N;
    p.K = K;
    p.m_shard = m_shard;
    p.rank = rank_;
    p.world = world_;
    p.epoch = ++ag_epoch_;
    p.timeout_ns = timeout_ns_;
    p.status = status_ptr();
    p.C = C.data_ptr();
    p.ldc = N;
    p.a_full = a_full.data_ptr();
    p.chunk_flags = reinterpret_cast<unsigned int*>(flags_.data_ptr<int32_t>());
    const int grid = pb::tp_gemm_grid(m_shard * world_, N);
    pb::tp_ag_gemm(p, local_->shard, B.data_ptr(), row_stride(B), b_mn, grid, stream());
    ag_target_ += static_cast<unsigned long long>((world_ - 1) * grid * 2);
  }

  // out [m_shard, N] = rows of this rank of sum_ranks(A @ B^T); A [world*m_shard, K]; B [N, K] (b_mn: [K, N]).
  void gemm_rs(const Tensor& A, const Tensor& B, bool b_mn, Tensor& out) {
    PB_CHECK(opened_ok_, "open() first");
    const int64_t M = A.size(0), K = A.size(1);
    const int64_t N = b_mn ? B.size(1) : B.size(0);
    PB_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "B has the wrong K");
    PB_CHECK(M % (128 * world_) == 0, "rows must be a multiple of 128 * world");
    const int64_t m_shard = M / world_;
    PB_CHECK(world_ * m_shard * N * 2 <= static_cast<int64_t>(slot_bytes()), "receive slots too small");
    PB_CHECK(out.is_contiguous() && out.size(0) == m_shard && out.size(1) == N && out.scalar_type() == torch::kBFloat16, "out");
    pb::TpGemmParams p = base_;
    p.N = N;
    p.K = K;
    p.m_shard = m_shard;
    p.rank = rank_;
    p.world = world_;
    p.epoch = ++rs_epoch_;
    p.timeout_ns = timeout_ns_;
    p.status = status_ptr();
    p.reduce_grid = kReduceGrid;
    const int grid = pb::tp_gemm_grid(M, N);
    rs_target_ += static_cast<unsigned long long>(world_ * grid);
    pb::tp_gemm_rs(p, A.data_ptr(), row_stride(A), B.data_ptr(), row_stride(B), b_mn, out.data_ptr(), N, grid,
                   kReduceGrid, rs_target_, stream());
  }

  int64_t slot_bytes() const { return slot_bytes_; }
  void set_slot_bytes(int64_t b) { slot_bytes_ = b; }

 private:
  static constexpr int kReduceGrid = 296;
  struct Local {
    void* shard = nullptr;
    void* slots = nullptr;
    void* signal = nullptr;
    ~Local() {
      pb::sym_free(shard);
      pb::sym_free(slots);
      pb::sym_free(signal);
    }
  };
  int64_t rank_, world_;
  long long timeout_ns_;
  int device_;
  std::shared_ptr<Local> local_;
  Tensor shard_, flags_;
  pb::TpGemmParams base_;
  std::vector<void*> opened_;
  bool opened_ok_ = false;
  long long ag_epoch_ = 0, rs_epoch_ = 0;
  unsigned long long ag_target_ = 0, rs_target_ = 0;
  int64_t slot_bytes_ = 0;
};

// Expert GEMMs fused with the expert-parallel exchange (ep_gemm.cu). Per rank: an IPC-mapped
// send buffer (rows offered to the expert owners, pulled by their GEMMs), a recv buffer (rows
// the owners' GEMM epilogues push back) and a signal array; the host keeps the epochs.
// Every rank must make the same calls in the same order.
class EpGemmGroup {
 public:
  EpGemmGroup(int64_t rank, int64_t world, int64_t send_rows, int64_t recv_rows, int64_t cols, int64_t max_chunks,
              double timeout_s)
      : rank_(rank), world_(world), cols_(cols), send_rows_(std::max<int64_t>(send_rows, 1)),
        recv_rows_(std::max<int64_t>(recv_rows, 1)), timeout_ns_(static_cast<long long>(timeout_s * 1e9)),
        device_(at::cuda::current_device()) {
    PB_CHECK(world >= 1 && world <= pb::kMaxRanks, "world size must be 1..8");
    PB_CHECK(cols % 64 == 0, "channels must be a multiple of 64");
    local_ = std::make_shared<Local>();
    local_->send = pb::sym_alloc(send_rows_ * cols * 2);
    local_->recv = pb::sym_alloc(recv_rows_ * cols * 2);
    local_->signal = pb::sym_alloc(pb::kSigWords * 8);
    auto opts = torch::TensorOptions().device(torch::kCUDA, device_);
    counters_ = torch::zeros({4}, opts.dtype(torch::kInt32));
    flags_ = torch::zeros({std::max<int64_t>(max_chunks, 1)}, opts.dtype(torch::kInt32));
  }
  ~EpGemmGroup() {
    for (void* p : opened_) pb::ipc_close(p);
  }
  py::bytes handles() const {
    char buf[192];
    pb::ipc_handle(local_->send, buf);
    pb::ipc_handle(local_->recv, buf + 64);
    pb::ipc_handle(local_->signal, buf + 128);
    return py::bytes(buf, 192);
  }
  void open(const std::vector<std::string>& all) {
    PB_CHECK(static_cast<int64_t>(all.size()) == world_, "need one handle record per rank");
    const c10::cuda::CUDAGuard guard(device_);
    for (int64_t r = 0; r < world_; ++r) {
      void* ptr[3] = {local_->send, local_->recv, local_->signal};
      if (r != rank_) {
        for (int i = 0; i < 3; ++i) {
          ptr[i] = pb::ipc_open(all[r].data() + 64 * i);
          opened_.push_back(ptr[i]);
        }
      }
      send_[r] = reinterpret_cast<unsigned long long>(ptr[0]);
      recv_[r] = reinterpret_cast<unsigned long long>(ptr[1]);
      sig_[r] = reinterpret_cast<unsigned long long>(ptr[2]);
    }
    opened_ok_ = true;
  }
  // The first `rows` rows of this rank's send buffer, to be filled once wait_send_free() is queued.
  Tensor send_rows(int64_t rows) const {
    PB_CHECK(rows <= send_rows_, "more rows than the send buffer holds");
    auto keep = local_;
    return torch::from_blob(local_->send, {rows, cols_}, [keep](void*) {},
                            torch::TensorOptions().device(torch::kCUDA, device_).dtype(torch::kBFloat16));
  }
  // Wait (on the stream) until every rank has finished pulling this rank's previous send rows.
  void wait_send_free() {
    PB_CHECK(opened_ok_, "open() first");
    if (send_epoch_ == 0) return;
    pb::tp_wait(local_->signal, pb::kEpSigSendDone, static_cast<unsigned long long>(send_epoch_) * world_, timeout_ns_,
                status_ptr(), stream());
  }

  // C = A @ B_e^T with A's rows pulled from the ranks' send buffers (row_src: int32 [M]) into a_local [M, K].
  // epi 3: B = up weights [experts * 2H, K], C = h [M, H], aux = gate/up [M, 2H] (written).
  // epi 4: B = down weights [experts * K, H] (N-major), aux = gate/up (read), C = d(gate/up) [M, 2H].
  void pull_gemm(const Tensor& row_src, const Tensor& offsets, const Tensor& B, int64_t epi, int64_t b_rows,
                 int64_t swiglu_h, Tensor& C, Tensor& aux, Tensor& a_local) {
    PB_CHECK(opened_ok_, "open() first");
    const int64_t M = a_local.size(0), K = a_local.size(1);
    PB_CHECK(K == cols_, "a_local must have the group's channel count");
    PB_CHECK(a_local.is_contiguous() && a_local.scalar_type() == torch::kBFloat16 && M % 128 == 0, "a_local bf16 [M % 128 == 0, K]");
    PB_CHECK(M / 128 <= flags_.numel(), "more row chunks than the flag buffer holds");
    PB_CHECK(row_src.scalar_type() == torch::kInt32 && row_src.is_contiguous() && row_src.numel() >= M, "row_src int32 [M]");
    PB_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.is_contiguous(), "offsets int32");
    PB_CHECK(B.scalar_type() == torch::kBFloat16 && B.dim() == 2 && B.stride(1) == 1, "B bf16, rows contiguous");
    PB_CHECK(aux.is_contiguous() && aux.size(0) == M && aux.size(1) == 2 * swiglu_h, "aux = gate/up [M, 2H]");
    PB_CHECK(C.is_contiguous() && C.size(0) == M, "C rows");
    pb::EpGemmParams p = base();
    const int experts = static_cast<int>(offsets.numel()) - 1;
    if (epi == 3) {
      PB_CHECK(B.size(1) == K && b_rows == 2 * swiglu_h && C.size(1) == swiglu_h, "epi 3: B [experts * 2H, K], C = h [M, H]");
      p.N = static_cast<int>(2 * swiglu_h);
    } else if (epi == 4) {
      PB_CHECK(B.size(1) == swiglu_h && b_rows == K && C.size(1) == 2 * swiglu_h, "epi 4: B [experts * K, H], C [M, 2H]");
      p.N = static_cast<int>(swiglu_h);
    } else {
      PB_CHECK(false, "epi must be 3 or 4");
    }
    PB_CHECK(B.size(0) == static_cast<int64_t>(experts) * b_rows, "B must stack experts * b_rows rows");
    p.M = static_cast<int>(M);
    p.K = static_cast<int>(K);
    p.C = C.data_ptr();
    p.ldc = C.stride(0);
    p.aux = aux.data_ptr();
    p.swiglu_h = static_cast<int>(swiglu_h);
    p.offsets = offsets.data_ptr<int>();
    p.experts = experts;
    p.b_rows = static_cast<int>(b_rows);
    p.epi = static_cast<int>(epi);
    p.epoch = ++send_epoch_;
    p.row_src = row_src.data_ptr<int>();
    p.a_local = a_local.data_ptr();
    p.chunk_flags = reinterpret_cast<unsigned int*>(flags_.data_ptr<int32_t>());
    p.block_counter = reinterpret_cast<unsigned int*>(counters_.data_ptr<int32_t>());
    const c10::cuda::CUDAGuard guard(device_);
    pb::ep_pull_gemm(p, B.data_ptr(), row_stride(B), epi == 4, stream());
  }

  // Rows of A @ B_e^T -> the recv buffers of their sources (row_dst: int32 [M]).
  // b_mn = false: B [experts * N, K]; true: B [experts * K, N].
  void push_gemm(const Tensor& A, const Tensor& row_dst, const Tensor& offsets, const Tensor& B, bool b_mn,
                 int64_t b_rows) {
    PB_CHECK(opened_ok_, "open() first");
    check_cuda(A, "A");
    PB_CHECK(A.scalar_type() == torch::kBFloat16 && A.stride(1) == 1 && A.size(0) % 128 == 0, "A bf16 [M % 128 == 0, K]");
    PB_CHECK(B.scalar_type() == torch::kBFloat16 && B.dim() == 2 && B.stride(1) == 1, "B bf16, rows contiguous");
    PB_CHECK(row_dst.scalar_type() == torch::kInt32 && row_dst.is_contiguous() && row_dst.numel() >= A.size(0), "row_dst int32 [M]");
    PB_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.is_contiguous(), "offsets int32");
    const int experts = static_cast<int>(offsets.numel()) - 1;
    const int64_t K = A.size(1);
    const int64_t N = b_mn ? B.size(1) : b_rows;
    PB_CHECK(N == cols_, "the output width must be the group's channel count");
    PB_CHECK(b_mn ? b_rows == K : B.size(1) == K, "B has the wrong K");
    PB_CHECK(B.size(0) == static_cast<int64_t>(experts) * b_rows, "B must stack experts * b_rows rows");
    pb::EpGemmParams p = base();
    p.M = static_cast<int>(A.size(0));
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.offsets = offsets.data_ptr<int>();
    p.experts = experts;
    p.b_rows = static_cast<int>(b_rows);
    p.epoch = ++push_epoch_;
    p.row_dst = row_dst.data_ptr<int>();
    p.block_counter = reinterpret_cast<unsigned int*>(counters_.data_ptr<int32_t>()) + 1;
    const c10::cuda::CUDAGuard guard(device_);
    pb::ep_push_gemm(p, A.data_ptr(), row_stride(A), B.data_ptr(), row_stride(B), b_mn, stream());
  }

  // out [tokens, cols] = sum_j weights[t, j] * recv[t * k + j] (plain sum without weights) after every
  // owner's push of this epoch; keep (optional) receives a copy of the rows. Frees the recv buffer.
  void combine(int64_t tokens, int64_t k, const c10::optional<Tensor>& weights, Tensor& out,
               const c10::optional<Tensor>& keep) {
    PB_CHECK(opened_ok_, "open() first");
    PB_CHECK(tokens * k <= recv_rows_, "more rows than the recv buffer holds");
    PB_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16 && out.numel() == tokens * cols_, "out bf16 [tokens, cols]");
    if (weights.has_value())
      PB_CHECK(weights->is_contiguous() && weights->scalar_type() == torch::kFloat32 && weights->numel() == tokens * k, "weights fp32 [tokens, k]");
    if (keep.has_value())
      PB_CHECK(keep->is_contiguous() && keep->scalar_type() == torch::kBFloat16 && keep->numel() == tokens * k * cols_, "keep bf16 [tokens * k, cols]");
    pb::EpCombineParams p{};
    p.recv = local_->recv;
    p.weights = weights.has_value() ? weights->data_ptr<float>() : nullptr;
    p.out = out.data_ptr();
    p.keep = keep.has_value() ? keep->data_ptr() : nullptr;
    p.tokens = tokens;
    p.k = static_cast<int>(k);
    p.cols = static_cast<int>(cols_);
    p.rank = static_cast<int>(rank_);
    p.world = static_cast<int>(world_);
    p.done_target = static_cast<unsigned long long>(push_epoch_) * world_;
    for (int r = 0; r < world_; ++r) p.signal[r] = sig_[r];
    p.block_counter = reinterpret_cast<unsigned int*>(counters_.data_ptr<int32_t>()) + 2;
    p.timeout_ns = timeout_ns_;
    p.status = status_ptr();
    const c10::cuda::CUDAGuard guard(device_);
    pb::ep_combine(p, stream());
  }

 private:
  pb::EpGemmParams base() const {
    pb::EpGemmParams p{};
    p.rank = static_cast<int>(rank_);
    p.world = static_cast<int>(world_);
    p.timeout_ns = timeout_ns_;
    p.status = status_ptr();
    p.dst_rows = recv_rows_;
    p.src_rows = send_rows_;
    for (int r = 0; r < world_; ++r) {
      p.src[r] = send_[r];
      p.dst[r] = recv_[r];
      p.signal[r] = sig_[r];
    }
    return p;
  }
  struct Local {
    void* send = nullptr;
    void* recv = nullptr;
    void* signal = nullptr;
    ~Local() {
      pb::sym_free(send);
      pb::sym_free(recv);
      pb::sym_free(signal);
    }
  };
  int64_t rank_, world_, cols_, send_rows_, recv_rows_;
  long long timeout_ns_;
  int device_;
  std::shared_ptr<Local> local_;
  Tensor counters_, flags_;
  unsigned long long send_[pb::kMaxRanks] = {}, recv_[pb::kMaxRanks] = {}, sig_[pb::kMaxRanks] = {};
  std::vector<void*> opened_;
  bool opened_ok_ = false;
  long long send_epoch_ = 0, push_epoch_ = 0;
};

// out[t * k + j] = w[t, j] * dy[t] (bf16) and dw[t, j] = <dy[t], y[t * k + j]> (fp32).
void ep_expand(const Tensor& dy, const Tensor& w, const Tensor& y, Tensor& out, Tensor& dw) {
  check_cuda(dy, "dy");
  const int64_t T = dy.size(0), C = dy.size(1), k = w.size(1);
  PB_CHECK(dy.is_contiguous() && dy.scalar_type() == torch::kBFloat16, "dy bf16 [T, C]");
  PB_CHECK(w.is_contiguous() && w.scalar_type() == torch::kFloat32 && w.size(0) == T, "w fp32 [T, k]");
  PB_CHECK(y.is_contiguous() && y.scalar_type() == torch::kBFloat16 && y.numel() == T * k * C, "y bf16 [T * k, C]");
  PB_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16 && out.numel() == T * k * C, "out bf16 [T * k, C]");
  PB_CHECK(dw.is_contiguous() && dw.scalar_type() == torch::kFloat32 && dw.numel() == T * k, "dw fp32 [T, k]");
  const c10::cuda::CUDAGuard guard(dy.device());
  pb::ep_expand(dy.data_ptr(), w.data_ptr<float>(), y.data_ptr(), out.data_ptr(), dw.data_ptr<float>(), T * k,
                static_cast<int>(k), static_cast<int>(C), stream());
}

// Expert-parallel row exchange (ep.cu): two symmetric row buffers per rank,
// 0 = rows travelling to the expert owners, 1 = rows travelling back to their sources.
class EpGroup {
 public:
  static constexpr int kDoneWord = 64, kFreeWord = 66;  // + buffer id

  EpGroup(int64_t rank, int64_t world, int64_t recv_rows, int64_t back_rows, int64_t cols, double timeout_s)
      : rank_(rank), world_(world), cols_(cols), timeout_ns_(static_cast<long long>(timeout_s * 1e9)),
        device_(at::cuda::current_device()) {
    PB_CHECK(world >= 1 && world <= pb::kMaxRanks, "world size must be 1..8");
    PB_CHECK(cols % 8 == 0, "channels must be a multiple of 8");
    rows_[0] = std::max<int64_t>(recv_rows, 1);
    rows_[1] = std::max<int64_t>(back_rows, 1);
    local_ = std::make_shared<Local>();
    for (int b = 0; b < 2; ++b) {
      local_->rows[b] = pb::sym_alloc(rows_[b] * cols * 2);
      local_->meta[b] = pb::sym_alloc(rows_[b] * 4);
    }
    local_->signal = pb::sym_alloc(pb::kSigWords * 8);
    counters_ = torch::zeros({2}, torch::TensorOptions().device(torch::kCUDA, device_).dtype(torch::kInt32));
  }
  ~EpGroup() {
    for (void* p : opened_) pb::ipc_close(p);
  }
  py::bytes handles() const {
    char buf[320];
    pb::ipc_handle(local_->rows[0], buf);
    pb::ipc_handle(local_->meta[0], buf + 64);
    pb::ipc_handle(local_->rows[1], buf + 128);
    pb::ipc_handle(local_->meta[1], buf + 192);
    pb::ipc_handle(local_->signal, buf + 256);
    return py::bytes(buf, 320);
  }
  void open(const std::vector<std::string>& all) {
    PB_CHECK(static_cast<int64_t>(all.size()) == world_, "need one handle record per rank");
    const c10::cuda::CUDAGuard guard(device_);
    for (int64_t r = 0; r < world_; ++r) {
      void* ptr[5];
      if (r == rank_) {
        ptr[0] = local_->rows[0], ptr[1] = local_->meta[0], ptr[2] = local_->rows[1], ptr[3] = local_->meta[1];
        ptr[4] = local_->signal;
      } else {
        for (int i = 0; i < 5; ++i) {
          ptr[i] = pb::ipc_open(all[r].data() + 64 * i);
          opened_.push_back(ptr[i]);
        }
      }
      for (int b = 0; b < 2; ++b) {
        peer_rows_[b][r] = reinterpret_cast<unsigned long long>(ptr[2 * b]);
        peer_meta_[b][r] = reinterpret_cast<unsigned long long>(ptr[2 * b + 1]);
      }
      peer_sig_[r] = reinterpret_cast<unsigned long long>(ptr[4]);
    }
    opened_ok_ = true;
  }

  // rows i of src (or src[gather[i]]) -> buffer b of rank dest_rank[i], row dest_row[i] (-1 rank: skipped).
  void scatter(int64_t b, const Tensor& src, const c10::optional<Tensor>& gather, const Tensor& dest_rank,
               const Tensor& dest_row, const c10::optional<Tensor>& meta) {
    PB_CHECK(opened_ok_ && (b == 0 || b == 1), "open() first; buffer 0 or 1");
    check_cuda(src, "src");
    PB_CHECK(src.scalar_type() == torch::kBFloat16 && src.dim() == 2 && src.size(1) == cols_ && src.stride(1) == 1 &&
                 src.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0,
             "src must be bf16 [rows, channels] with 16-byte aligned rows");
    PB_CHECK(dest_rank.scalar_type() == torch::kInt32 && dest_row.scalar_type() == torch::kInt64 &&
                 dest_rank.is_contiguous() && dest_row.is_contiguous() && dest_rank.numel() == dest_row.numel(),
             "dest_rank int32 / dest_row int64, contiguous, same length");
    const int64_t rows = dest_rank.numel();
    if (gather.has_value()) {
      PB_CHECK(gather->scalar_type() == torch::kInt64 && gather->is_contiguous() && gather->numel() == rows, "gather");
    } else {
      PB_CHECK(src.size(0) >= rows, "src has too few rows");
    }
    if (meta.has_value()) PB_CHECK(meta->scalar_type() == torch::kInt32 && meta->numel() == rows, "meta");
    pb::EpScatterParams p{};
    p.src = reinterpret_cast<const __nv_bfloat16*>(src.data_ptr());
    p.ld_src = src.stride(0);
    p.gather = gather.has_value() ? reinterpret_cast<const long long*>(gather->data_ptr<int64_t>()) : nullptr;
    p.dest_rank = dest_rank.data_ptr<int>();
    p.dest_row = reinterpret_cast<const long long*>(dest_row.data_ptr<int64_t>());
    p.meta = meta.has_value() ? meta->data_ptr<int>() : nullptr;
    p.rows = rows;
    p.cols = static_cast<int>(cols_);
    p.dest_cap = rows_[b];
    for (int r = 0; r < world_; ++r) {
      p.buf[r] = peer_rows_[b][r];
      p.meta_buf[r] = peer_meta_[b][r];
      p.signal[r] = peer_sig_[r];
    }
    p.done_word = kDoneWord + static_cast<int>(b);
    p.free_word = kFreeWord + static_cast<int>(b);
    p.rank = static_cast<int>(rank_);
    p.world = static_cast<int>(world_);
    p.epoch = ++epoch_[b];
    p.block_counter = reinterpret_cast<unsigned int*>(counters_.data_ptr<int>()) + b;
    p.timeout_ns = timeout_ns_;
    p.status = status_ptr();
    const c10::cuda::CUDAGuard guard(device_);
    pb::ep_scatter(p, stream());
  }
  // Wait (on the stream) until every rank has finished this epoch's scatter into our buffer b.
  void wait(int64_t b) {
    pb::tp_wait(local_->signal, kDoneWord + static_cast<int>(b), static_cast<unsigned long long>(epoch_[b]) * world_,
                timeout_ns_, status_ptr(), stream());
  }
  // First seg_start[segs] rows of our buffer b -> dst (segment padding zeroed, meta -1).
  void collect(int64_t b, Tensor& dst, const c10::optional<Tensor>& meta_dst, const Tensor& seg_start,
               const Tensor& totals) {
    PB_CHECK(dst.scalar_type() == torch::kBFloat16 && dst.is_contiguous() && dst.size(1) == cols_ &&
                 dst.size(0) <= rows_[b],
             "dst must be contiguous bf16 [rows <= capacity, channels]");
    PB_CHECK(seg_start.scalar_type() == torch::kInt32 && totals.scalar_type() == torch::kInt32 &&
                 seg_start.numel() == totals.numel() + 1,
             "seg_start int32 [segs + 1], totals int32 [segs]");
    if (meta_dst.has_value()) PB_CHECK(meta_dst->scalar_type() == torch::kInt32 && meta_dst->numel() >= dst.size(0), "meta_dst");
    pb::ep_collect(local_->rows[b], static_cast<const int*>(local_->meta[b]), dst.data_ptr(),
                   meta_dst.has_value() ? meta_dst->data_ptr<int>() : nullptr, seg_start.data_ptr<int>(),
                   totals.data_ptr<int>(), static_cast<int>(totals.numel()), static_cast<int>(cols_), dst.size(0),
                   stream());
  }
  // This rank has consumed its buffer b: peers may write the next epoch.
  void release(int64_t b) {
    pb::EpSignalParams p{};
    for (int r = 0; r < world_; ++r) p.signal[r] = peer_sig_[r];
    p.word = kFreeWord + static_cast<int>(b);
    p.world = static_cast<int>(world_);
    pb::ep_signal(p, stream());
  }
  // Our buffer b as a tensor (rows x channels), for consumers that read it in place.
  Tensor rows(int64_t b) const {
    auto keep = local_;
    return torch::from_blob(local_->rows[b], {rows_[b], cols_}, [keep](void*) {},
                            torch::TensorOptions().device(torch::kCUDA, device_).dtype(torch::kBFloat16));
  }

 private:
  struct Local {
    void* rows[2] = {nullptr, nullptr};
    void* meta[2] = {nullptr, nullptr};
    void* signal = nullptr;
    ~Local() {
      for (int b = 0; b < 2; ++b) {
        pb::sym_free(rows[b]);
        pb::sym_free(meta[b]);
      }
      pb::sym_free(signal);
    }
  };
  int64_t rank_, world_, cols_;
  long long timeout_ns_;
  int device_;
  int64_t rows_[2];
  std::shared_ptr<Local> local_;
  Tensor counters_;
  unsigned long long peer_rows_[2][pb::kMaxRanks] = {};
  unsigned long long peer_meta_[2][pb::kMaxRanks] = {};
  unsigned long long peer_sig_[pb::kMaxRanks] = {};
  std::vector<void*> opened_;
  bool opened_ok_ = false;
  long long epoch_[2] = {0, 0};
};

// images [B, C, H, W] (fp32 / bf16 / uint8, contiguous) -> [B, C, crop, crop].
Tensor augment_pad_crop_flip_cutout(const Tensor& images, int64_t crop, int64_t pad, int64_t mode, double fill,
                                    const Tensor& dy, const Tensor& dx, c10::optional<Tensor> flip, const Tensor& cy,
                                    const Tensor& cx, int64_t cut) {
  check_cuda(images, "images");
  PB_CHECK(images.dim() == 4 && images.is_contiguous(), "images must be contiguous [B, C, H, W]");
  const int B = images.size(0), C = images.size(1), H = images.size(2), W = images.size(3);
  int dtype = -1;
  if (images.scalar_type() == torch::kFloat32) dtype = 0;
  if (images.scalar_type() == torch::kBFloat16) dtype = 1;
  if (images.scalar_type() == torch::kUInt8) dtype = 2;
  PB_CHECK(dtype >= 0, "images must be fp32, bf16 or uint8");
  for (const Tensor* t : {&dy, &dx, &cy, &cx})
    PB_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->numel() == B, "offsets must be int32 [B]");
  if (flip.has_value()) PB_CHECK(flip->scalar_type() == torch::kUInt8 && flip->numel() == B, "flip must be uint8 [B]");
  PB_CHECK(crop <= H + 2 * pad && crop <= W + 2 * pad, "crop larger than the padded image");
  const c10::cuda::CUDAGuard guard(images.device());
  auto out = torch::empty({B, C, crop, crop}, images.options());
  pb::pad_crop_flip_cutout(images.data_ptr(), out.data_ptr(), dtype, B, C, H, W, static_cast<int>(crop),
                           static_cast<int>(pad), static_cast<int>(mode), static_cast<float>(fill),
                           dy.data_ptr<int32_t>(), dx.data_ptr<int32_t>(),
                           flip.has_value() ? flip->data_ptr<uint8_t>() : nullptr, cy.data_ptr<int32_t>(),
                           cx.data_ptr<int32_t>(), static_cast<int>(cut), stream());
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "priml_b200 sm_100a kernels";
  m.def("mx_quantize", &mx_quantize, "MXFP8 quantization (E4M3 + E8M0 per 32)", py::arg("x"), py::arg("transpose"));
  m.def("mx_gemm", &mx_gemm, "block-scaled MXFP8 tcgen05 GEMM", py::arg("A"), py::arg("sfa"), py::arg("B"), py::arg("sfb"),
        py::arg("C"), py::arg("epi"));
  m.def("grouped_gemm", &grouped_gemm, "grouped expert tcgen05 GEMM over device offsets", py::arg("A"), py::arg("B"),
        py::arg("C"), py::arg("offsets"), py::arg("b_mn"), py::arg("epi"), py::arg("mode"), py::arg("b_rows"),
        py::arg("aux") = py::none(), py::arg("swiglu_h") = 0);
  m.def("gemm", &gemm, "tcgen05 GEMM: C (op)= A B^T", py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn"),
        py::arg("b_mn"), py::arg("epi"));
  m.def("gemm_swiglu", &gemm_swiglu, "tcgen05 GEMM with fused SwiGLU epilogue");
  m.def("gemm_batched", &gemm_batched, "batched tcgen05 GEMM C[b] = alpha * A[b] B[b]^T (+ beta * X[b])",
        py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn"), py::arg("b_mn"), py::arg("X") = py::none(),
        py::arg("alpha") = 1.0, py::arg("beta") = 0.0);
  m.def("gemm_axpby", &gemm_axpby, "tcgen05 GEMM C = alpha * A B^T + beta * X (bf16)", py::arg("A"), py::arg("B"),
        py::arg("X"), py::arg("C"), py::arg("a_mn"), py::arg("b_mn"), py::arg("alpha"), py::arg("beta"));
  m.def("gemm_swiglu_bwd", &gemm_swiglu_bwd, "tcgen05 GEMM dy @ W_down with the SwiGLU backward in the epilogue");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("add_rmsnorm_bwd", &add_rmsnorm_bwd);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("ce_fwd", &ce_fwd, "token CE over bf16 logits -> (loss, lse); softcap > 0 caps the logits first",
        py::arg("logits"), py::arg("targets"), py::arg("ignore_index"), py::arg("softcap") = 0.0);
  m.def("ce_bwd", &ce_bwd, "d(logits) of ce_fwd, written into out (may alias logits)", py::arg("logits"),
        py::arg("targets"), py::arg("lse"), py::arg("g"), py::arg("out"), py::arg("ignore_index"),
        py::arg("softcap") = 0.0);
  m.def("gdn_fwd", &gdn_fwd, "gated delta-rule chunk scan, forward (tcgen05)");
  m.def("gdn_bwd", &gdn_bwd, "gated delta-rule chunk scan, backward (tcgen05)");
  m.def("mla_decode", &mla_decode, "multi-head latent attention decode in latent space (one query per sequence)",
        py::arg("q"), py::arg("c_kv"), py::arg("k_pe"), py::arg("lengths"), py::arg("scale"));
  m.def("decode_attn", &decode_attn, "one-token decode attention over a KV cache with device lengths",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("lengths"), py::arg("scale"), py::arg("window") = -1);
  m.def("attn_fwd", &attn_fwd, "flash attention forward (tcgen05); trace: optional int32 [8 * CTAs] progress record",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("scale"), py::arg("causal"), py::arg("window"),
        py::arg("trace") = py::none());
  m.def("attn_bwd", &attn_bwd, "flash attention backward (tcgen05)");
  m.def("cast_bf16", &cast_bf16, py::arg("x"), py::arg("out") = py::none());
  m.def("read_status", &read_status, py::arg("reset") = true);
  py::class_<PeerGroup>(m, "PeerGroup")
      .def(py::init<int64_t, int64_t, int64_t, int64_t>(), py::arg("rank"), py::arg("world"), py::arg("param_elems"),
           py::arg("grad_elems"))
      .def("handles", &PeerGroup::handles)
      .def("open", &PeerGroup::open)
      .def("param", &PeerGroup::param)
      .def("grad", &PeerGroup::grad)
      .def("signal", &PeerGroup::signal)
      .def("reduce_scatter", &PeerGroup::reduce_scatter)
      .def("norm_exchange", &PeerGroup::norm_exchange)
      .def("adamw_scatter", &PeerGroup::adamw_scatter, py::arg("segs"), py::arg("master"), py::arg("m1"), py::arg("m2"),
           py::arg("grad"), py::arg("clip"), py::arg("hyper"), py::arg("blocks"), py::arg("local_only") = false)
      .def("gather_shards", &PeerGroup::gather_shards, py::arg("src_off"), py::arg("count"), py::arg("dst"))
      .def("barrier", &PeerGroup::barrier);
  m.def("status_tensor", &status_tensor_py);
  py::class_<EpGroup>(m, "EpGroup")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, double>(), py::arg("rank"), py::arg("world"),
           py::arg("recv_rows"), py::arg("back_rows"), py::arg("cols"), py::arg("timeout_s") = 60.0)
      .def("handles", &EpGroup::handles)
      .def("open", &EpGroup::open)
      .def("scatter", &EpGroup::scatter, py::arg("b"), py::arg("src"), py::arg("gather"), py::arg("dest_rank"),
           py::arg("dest_row"), py::arg("meta"))
      .def("wait", &EpGroup::wait)
      .def("collect", &EpGroup::collect, py::arg("b"), py::arg("dst"), py::arg("meta_dst"), py::arg("seg_start"),
           py::arg("totals"))
      .def("release", &EpGroup::release)
      .def("rows", &EpGroup::rows);
  py::class_<EpGemmGroup>(m, "EpGemmGroup")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, double>(), py::arg("rank"), py::arg("world"),
           py::arg("send_rows"), py::arg("recv_rows"), py::arg("cols"), py::arg("max_chunks"), py::arg("timeout_s"))
      .def("handles", &EpGemmGroup::handles)
      .def("open", &EpGemmGroup::open)
      .def("send_rows", &EpGemmGroup::send_rows)
      .def("wait_send_free", &EpGemmGroup::wait_send_free)
      .def("pull_gemm", &EpGemmGroup::pull_gemm, py::arg("row_src"), py::arg("offsets"), py::arg("B"), py::arg("epi"),
           py::arg("b_rows"), py::arg("swiglu_h"), py::arg("C"), py::arg("aux"), py::arg("a_local"))
      .def("push_gemm", &EpGemmGroup::push_gemm, py::arg("A"), py::arg("row_dst"), py::arg("offsets"), py::arg("B"),
           py::arg("b_mn"), py::arg("b_rows"))
      .def("combine", &EpGemmGroup::combine, py::arg("tokens"), py::arg("k"), py::arg("weights"), py::arg("out"),
           py::arg("keep"));
  m.def("ep_expand", &ep_expand, "w * dy into the send rows and the routing-weight gradient", py::arg("dy"),
        py::arg("w"), py::arg("y"), py::arg("out"), py::arg("dw"));
  py::class_<TpGroup>(m, "TpGroup")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, double>(), py::arg("rank"), py::arg("world"),
           py::arg("shard_elems"), py::arg("slot_elems"), py::arg("max_chunks"), py::arg("timeout_s") = 60.0)
      .def("handles", &TpGroup::handles)
      .def("open", &TpGroup::open)
      .def("shard", &TpGroup::shard)
      .def("wait_shard_free", &TpGroup::wait_shard_free)
      .def("ag_gemm", &TpGroup::ag_gemm)
      .def("gemm_rs", &TpGroup::gemm_rs)
      .def("set_slot_bytes", &TpGroup::set_slot_bytes);
  m.def("augment_pad_crop_flip_cutout", &augment_pad_crop_flip_cutout, "fused pad + random crop + flip + cutout");
  py::class_<MultiTensorPlan>(m, "MultiTensorPlan")
      .def(py::init<std::vector<Tensor>, std::vector<Tensor>, std::vector<Tensor>, std::vector<Tensor>,
                    std::vector<c10::optional<Tensor>>, int64_t>())
      .def("adamw", &MultiTensorPlan::adamw)
      .def("grad_norm_clip", &MultiTensorPlan::grad_norm_clip)
      .def("num_chunks", &MultiTensorPlan::num_chunks);
}

// PyTorch bindings for the sm_100a kernels. Kernels live in .cu files that do not
// include torch headers; this file only validates tensors and forwards raw pointers
// plus the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "grouped_gemm.h"
#include "kernels.h"
#include "opt_bind.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DTYPE(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has wrong dtype")
#define CHECK_BF16(x) \
  CHECK_CUDA(x);      \
  CHECK_CONTIG(x);    \
  CHECK_DTYPE(x, at::kBFloat16)

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int* status_ptr(const c10::optional<at::Tensor>& s) {
  if (!s.has_value()) return nullptr;
  CHECK_DTYPE(*s, at::kInt);
  return s->data_ptr<int>();
}

// out[rows, N] = A[rows, K] . W[g]^T with W stored [G, N, K] (K-major weights).
void gg_fwd(const at::Tensor& A, const at::Tensor& W, const at::Tensor& group_off, at::Tensor& out,
            const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(W);
  CHECK_BF16(out);
  CHECK_DTYPE(group_off, at::kInt);
  const c10::cuda::CUDAGuard guard(A.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiBf16;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = W.data_ptr();
  c.b_rows = W.size(0) * W.size(1);
  c.ldb = W.size(2);
  c.b_kmajor = true;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = W.size(0);
  c.p.N = W.size(1);
  c.p.K = W.size(2);
  TORCH_CHECK(A.size(1) == c.p.K, "K mismatch");
  TORCH_CHECK(group_off.numel() == c.p.G + 1, "group_off must have G+1 entries");
  c.p.b_rows_per_group = W.size(1);
  c.p.out = out.data_ptr();
  c.p.ldo = out.size(1);
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_m(c, cur_stream());
}

// out[rows, N] = A[rows, K] . W[g] with W stored [G, K, N] (MN-major weights, dgrad).
void gg_dgrad(const at::Tensor& A, const at::Tensor& W, const at::Tensor& group_off,
              at::Tensor& out, const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(W);
  CHECK_BF16(out);
  const c10::cuda::CUDAGuard guard(A.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiBf16;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = W.data_ptr();
  c.b_rows = W.size(0) * W.size(1);
  c.ldb = W.size(2);
  c.b_kmajor = false;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = W.size(0);
  c.p.K = W.size(1);
  c.p.N = W.size(2);
  TORCH_CHECK(A.size(1) == c.p.K, "K mismatch");
  c.p.b_rows_per_group = W.size(1);
  c.p.out = out.data_ptr();
  c.p.ldo = out.size(1);
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_m(c, cur_stream());
}

// h = silu(g) * u, gu = [g | u] with [g | u] = A . Wgu[e]^T, Wgu stored [G, 2I, K].
void gg_swiglu_fwd(const at::Tensor& A, const at::Tensor& Wgu, const at::Tensor& group_off,
                   at::Tensor& h, at::Tensor& gu, const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(Wgu);
  CHECK_BF16(h);
  CHECK_BF16(gu);
  const c10::cuda::CUDAGuard guard(A.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiSwigluFwd;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = Wgu.data_ptr();
  c.b_rows = Wgu.size(0) * Wgu.size(1);
  c.ldb = Wgu.size(2);
  c.b_kmajor = true;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = Wgu.size(0);
  c.p.K = Wgu.size(2);
  c.p.I = Wgu.size(1) / 2;
  c.p.N = c.p.I;
  TORCH_CHECK(A.size(1) == c.p.K, "K mismatch");
  c.p.b_rows_per_group = Wgu.size(1);
  c.p.out = h.data_ptr();
  c.p.ldo = h.size(1);
  c.p.aux = gu.data_ptr();
  c.p.ld_aux = gu.size(1);
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_m(c, cur_stream());
}

// Backward through down-projection + SwiGLU:
//   dh = dY . Wd[e] (Wd stored [G, H, I]);  dgu = SwiGLU'(gu) * (w * dh);
//   hw = w * silu(g) * u;  row_dw += <dh, silu(g) * u>.
void gg_swiglu_bwd(const at::Tensor& dY, const at::Tensor& Wd, const at::Tensor& group_off,
                   const at::Tensor& gu, const at::Tensor& row_w, at::Tensor& dgu, at::Tensor& hw,
                   at::Tensor& row_dw, const c10::optional<at::Tensor>& status) {
  CHECK_BF16(dY);
  CHECK_BF16(Wd);
  CHECK_BF16(gu);
  CHECK_BF16(dgu);
  CHECK_BF16(hw);
  CHECK_DTYPE(row_w, at::kFloat);
  CHECK_DTYPE(row_dw, at::kFloat);
  const c10::cuda::CUDAGuard guard(dY.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiSwigluBwd;
  c.A = dY.data_ptr();
  c.a_rows = dY.size(0);
  c.lda = dY.size(1);
  c.B = Wd.data_ptr();
  c.b_rows = Wd.size(0) * Wd.size(1);
  c.ldb = Wd.size(2);
  c.b_kmajor = false;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = Wd.size(0);
  c.p.K = Wd.size(1);
  c.p.N = Wd.size(2);
  c.p.I = Wd.size(2);
  TORCH_CHECK(dY.size(1) == c.p.K, "K mismatch");
  c.p.b_rows_per_group = Wd.size(1);
  c.p.out = dgu.data_ptr();
  c.p.ldo = dgu.size(1);
  c.p.aux = const_cast<void*>(gu.data_ptr());
  c.p.ld_aux = gu.size(1);
  c.p.aux2 = hw.data_ptr();
  c.p.ld_aux2 = hw.size(1);
  c.p.row_w = row_w.data_ptr<float>();
  c.p.row_dw = row_dw.data_ptr<float>();
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_m(c, cur_stream());
}

// out[g] (fp32 [M, N]) = A[rows_g, :]^T . B[rows_g, :]  with A [rows, M], B [rows, N].
void gg_wgrad(const at::Tensor& A, const at::Tensor& B, const at::Tensor& group_off,
              at::Tensor& out, const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_CUDA(out);
  CHECK_DTYPE(out, at::kFloat);
  const c10::cuda::CUDAGuard guard(A.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiF32;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = B.data_ptr();
  c.b_rows = B.size(0);
  c.ldb = B.size(1);
  c.b_kmajor = false;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = out.size(0);
  c.p.M = out.size(1);
  c.p.N = out.size(2);
  TORCH_CHECK(A.size(1) == c.p.M && B.size(1) == c.p.N, "shape mismatch");
  c.p.out = out.data_ptr();
  c.p.ldo = out.size(2);
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_k(c, cur_stream());
}

// out (bf16 [M, N]) = A^T . B over all rows, A [rows, M], B [rows, N]: the weight gradient
// of a dense projection (one group; rows a multiple of 64).
void gemm_wgrad_bf16(const at::Tensor& A, const at::Tensor& B, const at::Tensor& group_off, at::Tensor& out,
                     const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_BF16(out);
  CHECK_DTYPE(group_off, at::kInt);
  TORCH_CHECK(A.size(0) == B.size(0) && A.size(0) % 64 == 0, "rows must match and be a multiple of 64");
  TORCH_CHECK(group_off.numel() == 2, "group_off must be the device tensor [0, rows]");
  const c10::cuda::CUDAGuard guard(A.device());
  const at::Tensor& go = group_off;
  sepx::GemmCall c;
  c.epi = sepx::kEpiBf16;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = B.data_ptr();
  c.b_rows = B.size(0);
  c.ldb = B.size(1);
  c.b_kmajor = false;
  c.p.group_off = go.data_ptr<int>();
  c.p.G = 1;
  c.p.M = out.size(0);
  c.p.N = out.size(1);
  TORCH_CHECK(A.size(1) == c.p.M && B.size(1) == c.p.N, "shape mismatch");
  c.p.out = out.data_ptr();
  c.p.ldo = out.size(1);
  c.p.status = status_ptr(status);
  sepx::grouped_gemm_ragged_k(c, cur_stream());
}

// W[g] <- AdamW(W[g], A[rows_g]^T . B[rows_g]): weight gradient with the optimizer update
// fused into the GEMM epilogue (the gradient never reaches HBM). W is [G, M, N].
void gg_wgrad_adamw(const at::Tensor& A, const at::Tensor& B, const at::Tensor& group_off, at::Tensor& W,
                    int64_t kind, const c10::optional<at::Tensor>& master, at::Tensor& m, at::Tensor& v,
                    const c10::optional<at::Tensor>& ms, const c10::optional<at::Tensor>& vs, double lr, double b1,
                    double b2, double eps, double wd, int64_t step, double grad_scale, int64_t seed,
                    const c10::optional<at::Tensor>& status) {
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_BF16(W);
  TORCH_CHECK(W.dim() == 3, "W must be [G, M, N]");
  const c10::cuda::CUDAGuard guard(A.device());
  sepx::GemmCall c;
  c.epi = sepx::kEpiAdamW;
  c.A = A.data_ptr();
  c.a_rows = A.size(0);
  c.lda = A.size(1);
  c.B = B.data_ptr();
  c.b_rows = B.size(0);
  c.ldb = B.size(1);
  c.b_kmajor = false;
  c.p.group_off = group_off.data_ptr<int>();
  c.p.G = W.size(0);
  c.p.M = W.size(1);
  c.p.N = W.size(2);
  TORCH_CHECK(A.size(1) == c.p.M && B.size(1) == c.p.N, "shape mismatch");
  c.p.status = status_ptr(status);
  c.p.opt = sepx::make_opt(W, kind, master, m, v, ms, vs, lr, b1, b2, eps, wd, step, grad_scale, seed);
  sepx::grouped_gemm_wgrad_adamw(c, cur_stream());
}

}  // namespace

void register_kernels(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "spec_ep sm_100a kernels";
  m.def("gg_fwd", &gg_fwd);
  m.def("gemm_wgrad_bf16", &gemm_wgrad_bf16);
  m.def("gemm_set_pairs", &sepx::gemm_set_pairs, "256-column GEMM tiles on CTA pairs (returns the previous setting)");
  m.def("gg_dgrad", &gg_dgrad);
  m.def("gg_swiglu_fwd", &gg_swiglu_fwd);
  m.def("gg_swiglu_bwd", &gg_swiglu_bwd);
  m.def("gg_wgrad", &gg_wgrad);
  m.def("gg_wgrad_adamw", &gg_wgrad_adamw);
  register_kernels(m);
}

// Python bindings of the memory-bound kernels (elementwise.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention.h"
#include "elementwise.h"
#include "opt_bind.h"

namespace {

cudaStream_t cs() { return at::cuda::getCurrentCUDAStream().stream(); }

int num_sms() {
  static int n = 0;
  if (!n) n = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  return n;
}

void req(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}

const int* opt_int(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr<int>() : nullptr; }
const float* opt_f(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr<float>() : nullptr; }

// add / sum (optional, together): y = rmsnorm(x + add), with x + add written to sum.
void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps,
                 const c10::optional<at::Tensor>& add, const c10::optional<at::Tensor>& sum) {
  req(x, at::kBFloat16, "x");
  req(w, at::kBFloat16, "w");
  req(y, at::kBFloat16, "y");
  req(rstd, at::kFloat, "rstd");
  TORCH_CHECK(add.has_value() == sum.has_value(), "add and sum go together");
  if (add.has_value()) {
    req(*add, at::kBFloat16, "add");
    req(*sum, at::kBFloat16, "sum");
    TORCH_CHECK(add->numel() == x.numel() && sum->numel() == x.numel(), "add / sum must match x");
  }
  const int D = x.size(-1);
  const int N = x.numel() / D;
  sepx::rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), N, D, (float)eps, cs(),
                    add.has_value() ? add->data_ptr() : nullptr, sum.has_value() ? sum->data_ptr() : nullptr);
}

// dres (optional): gradient of x from its other uses, added into dx.
void rmsnorm_bwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd, const at::Tensor& dy, at::Tensor& dx,
                 at::Tensor& dw, const c10::optional<at::Tensor>& dres) {
  req(x, at::kBFloat16, "x");
  req(dy, at::kBFloat16, "dy");
  req(dx, at::kBFloat16, "dx");
  req(dw, at::kFloat, "dw");
  if (dres.has_value()) {
    req(*dres, at::kBFloat16, "dres");
    TORCH_CHECK(dres->numel() == x.numel(), "dres must match x");
  }
  const int D = x.size(-1);
  const int N = x.numel() / D;
  sepx::rmsnorm_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(), dx.data_ptr(),
                    dw.data_ptr<float>(), N, D, num_sms(), cs(), dres.has_value() ? dres->data_ptr() : nullptr);
}

void qk_norm_rope_fwd(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, at::Tensor& q, at::Tensor& k,
                      at::Tensor& v, at::Tensor& rstd_q, at::Tensor& rstd_k, const c10::optional<at::Tensor>& pos,
                      int64_t Hq, int64_t Hkv, double eps, double theta) {
  req(qkv, at::kBFloat16, "qkv");
  const int T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * 128, "qkv width must be (Hq + 2 Hkv) * 128");
  sepx::qk_norm_rope_fwd(qkv.data_ptr(), wq.data_ptr(), wk.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                         rstd_q.data_ptr<float>(), rstd_k.data_ptr<float>(), opt_int(pos), T, Hq, Hkv, (float)eps,
                         (float)theta, cs());
}

void qk_norm_rope_bwd(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& rstd_q,
                      const at::Tensor& rstd_k, const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv,
                      at::Tensor& dqkv, at::Tensor& dwq, at::Tensor& dwk, const c10::optional<at::Tensor>& pos,
                      int64_t Hq, int64_t Hkv, double theta) {
  req(dq, at::kBFloat16, "dq");
  req(dk, at::kBFloat16, "dk");
  req(dv, at::kBFloat16, "dv");
  req(dqkv, at::kBFloat16, "dqkv");
  const int T = qkv.size(0);
  sepx::qk_norm_rope_bwd(qkv.data_ptr(), wq.data_ptr(), wk.data_ptr(), rstd_q.data_ptr<float>(),
                         rstd_k.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dqkv.data_ptr(),
                         dwq.data_ptr<float>(), dwk.data_ptr<float>(), opt_int(pos), T, Hq, Hkv, (float)theta,
                         num_sms(), cs());
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& h) {
  req(gu, at::kBFloat16, "gu");
  req(h, at::kBFloat16, "h");
  const int I = h.size(-1);
  sepx::swiglu_fwd(gu.data_ptr(), h.data_ptr(), h.numel() / I, I, num_sms(), cs());
}

void swiglu_bwd(const at::Tensor& gu, const at::Tensor& dh, at::Tensor& dgu) {
  req(gu, at::kBFloat16, "gu");
  req(dh, at::kBFloat16, "dh");
  req(dgu, at::kBFloat16, "dgu");
  const int I = dh.size(-1);
  sepx::swiglu_bwd(gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), dh.numel() / I, I, num_sms(), cs());
}

void router_topk(const at::Tensor& logits, const c10::optional<at::Tensor>& bias, int64_t k, bool renorm,
                 at::Tensor& topk_e, at::Tensor& topk_w, const c10::optional<at::Tensor>& probs) {
  req(logits, at::kFloat, "logits");
  req(topk_e, at::kInt, "topk_e");
  req(topk_w, at::kFloat, "topk_w");
  sepx::router_topk(logits.data_ptr<float>(), opt_f(bias), logits.size(0), logits.size(1), k, renorm,
                    topk_e.data_ptr<int>(), topk_w.data_ptr<float>(),
                    probs.has_value() ? probs->data_ptr<float>() : nullptr, cs());
}

void router_bwd(const at::Tensor& probs, const at::Tensor& topk_e, const at::Tensor& dw, bool renorm, at::Tensor& dlogits) {
  req(probs, at::kFloat, "probs");
  req(dw, at::kFloat, "dw");
  req(dlogits, at::kFloat, "dlogits");
  sepx::router_bwd(probs.data_ptr<float>(), topk_e.data_ptr<int>(), dw.data_ptr<float>(), probs.size(0), probs.size(1),
                   topk_e.size(1), renorm, dlogits.data_ptr<float>(), cs());
}

void adamw_update(at::Tensor& p, const at::Tensor& g, int64_t kind, const c10::optional<at::Tensor>& master,
                  at::Tensor& m, at::Tensor& v, const c10::optional<at::Tensor>& ms, const c10::optional<at::Tensor>& vs,
                  double lr, double b1, double b2, double eps, double wd, int64_t step, double grad_scale,
                  int64_t seed) {
  TORCH_CHECK(g.is_cuda() && g.is_contiguous() && g.numel() == p.numel(), "grad must match the parameter");
  TORCH_CHECK(g.scalar_type() == at::kFloat || g.scalar_type() == at::kBFloat16, "grad must be fp32 or bf16");
  auto h = sepx::make_opt(p, kind, master, m, v, ms, vs, lr, b1, b2, eps, wd, step, grad_scale, seed);
  sepx::adamw_update(h, g.data_ptr(), g.scalar_type() == at::kBFloat16, p.numel(), num_sms(), cs());
}

void xent_fwd_bwd(at::Tensor& logits, const at::Tensor& labels, double scale, at::Tensor& loss) {
  req(logits, at::kBFloat16, "logits");
  req(labels, at::kInt, "labels");
  req(loss, at::kFloat, "loss");
  TORCH_CHECK(logits.size(1) % 8 == 0, "vocab must be a multiple of 8");
  sepx::xent_fwd_bwd(logits.data_ptr(), labels.data_ptr<int>(), logits.size(0), logits.size(1), (float)scale,
                     loss.data_ptr<float>(), cs());
}

void attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                   double scale, const c10::optional<at::Tensor>& status, bool two_tile,
                   const c10::optional<at::Tensor>& trace) {
  req(q, at::kBFloat16, "q");
  req(k, at::kBFloat16, "k");
  req(v, at::kBFloat16, "v");
  req(o, at::kBFloat16, "o");
  req(lse, at::kFloat, "lse");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && k.size(2) == 128, "q/k/v must be [T, heads, 128]");
  const int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  if (two_tile)
    sepx::attention_fwd_pp(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), T, Hq,
                           Hkv, (float)scale, st, cs(),
                           trace.has_value() ? reinterpret_cast<long long*>(trace->data_ptr<int64_t>()) : nullptr);
  else
    sepx::attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), T, Hq, Hkv,
                        (float)scale, st, cs());
}

// Returns (dq, dk, dv), each shaped like its input.
std::vector<at::Tensor> attention_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                      const at::Tensor& o, const at::Tensor& dout, const at::Tensor& lse, double scale,
                                      const c10::optional<at::Tensor>& status) {
  req(q, at::kBFloat16, "q");
  req(k, at::kBFloat16, "k");
  req(v, at::kBFloat16, "v");
  req(o, at::kBFloat16, "o");
  req(dout, at::kBFloat16, "dout");
  req(lse, at::kFloat, "lse");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && k.size(2) == 128, "q/k/v must be [T, heads, 128]");
  const int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  TORCH_CHECK(o.numel() == q.numel() && dout.numel() == q.numel() && lse.numel() == (int64_t)T * Hq,
              "o/dout/lse shapes do not match q");
  auto f32 = q.options().dtype(at::kFloat);
  at::Tensor dsum = at::empty({Hq, T}, f32);
  at::Tensor dq_acc = at::empty({T, Hq, 128}, f32);
  at::Tensor dk_acc = at::empty({T, Hkv, 128}, f32);
  at::Tensor dv_acc = at::empty({T, Hkv, 128}, f32);
  at::Tensor dq = at::empty_like(q), dk = at::empty_like(k), dv = at::empty_like(v);
  sepx::attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr<float>(),
                      dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), dk_acc.data_ptr<float>(),
                      dv_acc.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), T, Hq, Hkv, (float)scale,
                      status.has_value() ? status->data_ptr<int>() : nullptr, cs());
  return {dq, dk, dv};
}

}  // namespace

void register_elementwise(pybind11::module& m) {
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("router_topk", &router_topk);
  m.def("router_bwd", &router_bwd);
  m.def("adamw_update", &adamw_update);
  m.def("xent_fwd_bwd", &xent_fwd_bwd);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_bwd", &attention_bwd);
}

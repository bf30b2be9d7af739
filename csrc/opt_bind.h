// Builds an OptHyper from PyTorch tensors (host side; used by the optimizer bindings).
#pragma once
#include <torch/extension.h>

#include <cmath>

#include "opt_hyper.h"

namespace sepx {

// kind: 1 = fp32 master + moments, 2 = block-wise 8-bit moments (32-element blocks).
inline OptHyper make_opt(at::Tensor& param, int64_t kind, const c10::optional<at::Tensor>& master, at::Tensor& m,
                         at::Tensor& v, const c10::optional<at::Tensor>& m_scale,
                         const c10::optional<at::Tensor>& v_scale, double lr, double b1, double b2, double eps,
                         double wd, int64_t step, double grad_scale, int64_t seed) {
  TORCH_CHECK(param.is_cuda() && param.is_contiguous() && param.scalar_type() == at::kBFloat16,
              "param must be contiguous bf16 on the GPU");
  OptHyper h;
  h.kind = (int)kind;
  h.lr = lr;
  h.beta1 = b1;
  h.beta2 = b2;
  h.eps = eps;
  h.weight_decay = wd;
  h.step = (uint32_t)step;
  h.bc1 = 1.0 / (1.0 - std::pow(b1, (double)step));
  h.bc2 = std::sqrt(1.0 / (1.0 - std::pow(b2, (double)step)));
  h.grad_scale = grad_scale;
  h.seed = (uint32_t)seed;
  h.param = reinterpret_cast<__nv_bfloat16*>(param.data_ptr());
  const int64_t n = param.numel();
  if (kind == 1) {
    TORCH_CHECK(master.has_value() && master->scalar_type() == at::kFloat && master->numel() == n, "fp32 master");
    TORCH_CHECK(m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat && m.numel() == n && v.numel() == n,
                "fp32 moments");
    h.master = master->data_ptr<float>();
  } else if (kind == 2) {
    TORCH_CHECK(n % 32 == 0, "8-bit state needs a multiple of 32 elements");
    TORCH_CHECK(m.scalar_type() == at::kChar && v.scalar_type() == at::kByte && m.numel() == n && v.numel() == n,
                "8-bit moments must be int8 / uint8 with one entry per element");
    TORCH_CHECK(m_scale.has_value() && v_scale.has_value() && m_scale->numel() == n / 32 &&
                    v_scale->numel() == n / 32,
                "8-bit scales: one fp32 per 32 elements");
    h.m_scale = m_scale->data_ptr<float>();
    h.v_scale = v_scale->data_ptr<float>();
  } else {
    TORCH_CHECK(false, "unknown optimizer state kind ", kind);
  }
  h.m = m.data_ptr();
  h.v = v.data_ptr();
  return h;
}

}  // namespace sepx

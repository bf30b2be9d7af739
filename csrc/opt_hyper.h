// Optimizer hyper-parameters and state pointers for one AdamW update (host-safe header;
// the update math is in adamw_math.cuh).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace sepx {

enum : int { kOptNone = 0, kOptFp32 = 1, kOpt8bit = 2 };

struct OptHyper {
  int kind = kOptNone;
  float lr = 0.f, beta1 = 0.9f, beta2 = 0.95f, eps = 1e-8f, weight_decay = 0.f;
  float bc1 = 1.f;  // 1 / (1 - beta1^step)
  float bc2 = 1.f;  // sqrt(1 / (1 - beta2^step))
  float grad_scale = 1.f;
  uint32_t step = 1, seed = 0;
  __nv_bfloat16* param = nullptr;  // bf16 weights (updated in place)
  float* master = nullptr;         // kOptFp32
  void* m = nullptr;               // float* (fp32) or int8_t* (8-bit)
  void* v = nullptr;               // float* (fp32) or uint8_t* (8-bit)
  float* m_scale = nullptr;        // 8-bit: one per 32 elements
  float* v_scale = nullptr;
};

}  // namespace sepx

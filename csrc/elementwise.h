// Launchers of the memory-bound kernels in elementwise.cu.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sepx {

struct AdamWHyper {
  float lr = 1e-4f, beta1 = 0.9f, beta2 = 0.95f, eps = 1e-8f, weight_decay = 0.1f;
  float bc1 = 1.f, bc2 = 1.f;  // 1/(1-beta1^t), 1/(1-beta2^t)
  float grad_scale = 1.f;
  int step = 1;
  uint32_t seed = 0;
};

void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int N, int D, float eps, cudaStream_t st);
void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, void* dx, float* dw, int N, int D,
                 int num_sms, cudaStream_t st);
void qk_norm_rope_fwd(const void* qkv, const void* wq, const void* wk, void* q, void* k, void* v, float* rstd_q,
                      float* rstd_k, const int* pos_ids, int T, int Hq, int Hkv, float eps, float theta,
                      cudaStream_t st);
void qk_norm_rope_bwd(const void* qkv, const void* wq, const void* wk, const float* rstd_q, const float* rstd_k,
                      const void* dq, const void* dk, const void* dv, void* dqkv, float* dwq, float* dwk,
                      const int* pos_ids, int T, int Hq, int Hkv, float theta, int num_sms, cudaStream_t st);
void swiglu_fwd(const void* gu, void* h, int N, int I, int num_sms, cudaStream_t st);
void swiglu_bwd(const void* gu, const void* dh, void* dgu, int N, int I, int num_sms, cudaStream_t st);
void router_topk(const float* logits, const float* bias, int T, int E, int k, bool renorm, int* topk_e,
                 float* topk_w, float* probs, cudaStream_t st);
void router_bwd(const float* probs, const int* topk_e, const float* dw, int T, int E, int k, bool renorm,
                float* dlogits, cudaStream_t st);
void adamw_fp32(void* p, float* master, const float* g, float* m, float* v, size_t n, const AdamWHyper& h,
                int num_sms, cudaStream_t st);
void adamw_8bit(void* p, const float* g, int8_t* mq, float* ms, uint8_t* vq, float* vs, size_t n,
                const AdamWHyper& h, int num_sms, cudaStream_t st);
void xent_fwd_bwd(void* logits, const int* labels, int T, int V, float scale, float* loss, cudaStream_t st);

}  // namespace sepx

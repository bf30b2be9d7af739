// Launchers of the memory-bound kernels in elementwise.cu.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "opt_hyper.h"

namespace sepx {

// add / sum (optional, together): normalise s = x + add and write s to sum.
void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int N, int D, float eps, cudaStream_t st,
                 const void* add = nullptr, void* sum = nullptr);
// dres (optional): the input's gradient from its other uses, added to dx (as a bf16 add).
void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, void* dx, float* dw, int N, int D,
                 int num_sms, cudaStream_t st, const void* dres = nullptr);
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
// AdamW over n contiguous elements; h.kind selects fp32 or block-wise 8-bit state.
void adamw_update(const OptHyper& h, const void* g, bool g_bf16, size_t n, int num_sms, cudaStream_t st);
void xent_fwd_bwd(void* logits, const int* labels, int T, int V, float scale, float* loss, cudaStream_t st);

}  // namespace sepx

// Causal GQA attention on tcgen05 (head_dim 128): launch parameters and launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sepx {

struct AttnParams {
  int T = 0, Hq = 0, Hkv = 0;
  float scale_log2 = 0.f;  // softmax scale * log2(e)
  void* o = nullptr;       // [T, Hq * 128] bf16
  float* lse = nullptr;    // [Hq, T] natural-log log-sum-exp of the scaled logits
  int* status = nullptr;
  unsigned long long timeout_ns = 2000000000ull;
  // Optional trace (two-tile forward, CTA 0 only): SM-clock stamps per 128-key block j,
  // [role][j][event] with roles 0/1 = MMA issue for tile A/B (P ready, P V issued, P V
  // done, next S issued) and 2/3 = a softmax warp of tile A/B (S ready, P computed,
  // P published, -). Laid out as int64 [4][64][4]; null disables it.
  long long* trace = nullptr;
};

struct AttnBwdParams {
  int T = 0, Hq = 0, Hkv = 0;
  float scale = 0.f, scale_log2 = 0.f;
  const float* lse = nullptr;   // [Hq, T]
  const float* dsum = nullptr;  // [Hq, T] rowsum(dO * O)
  float* dq_acc = nullptr;      // [T, Hq, 128] fp32
  float* dk_acc = nullptr;      // [T, Hkv, 128] fp32
  float* dv_acc = nullptr;      // [T, Hkv, 128] fp32
  int* status = nullptr;
  unsigned long long timeout_ns = 2000000000ull;
};

// q [T, Hq*128], k/v [T, Hkv*128] bf16 (token-major) -> o [T, Hq*128], lse [Hq, T].
void attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int T, int Hq, int Hkv,
                   float scale, int* status, cudaStream_t st);

// Same result, two query tiles per CTA sharing K/V loads (P kept in TMEM).
void attention_fwd_pp(const void* q, const void* k, const void* v, void* o, float* lse, int T, int Hq, int Hkv,
                      float scale, int* status, cudaStream_t st, long long* trace = nullptr);

// Backward: dq/dk/dv (bf16) from dout, using the forward's o and lse. dsum, dq_acc,
// dk_acc, dv_acc are fp32 scratch ([Hq*T], [T*Hq*128], [T*Hkv*128] x2).
void attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                   float* dsum, float* dq_acc, float* dk_acc, float* dv_acc, void* dq, void* dk, void* dv, int T,
                   int Hq, int Hkv, float scale, int* status, cudaStream_t st);

}  // namespace sepx

// Host-facing description of the tcgen05 grouped GEMM (see grouped_gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "opt_hyper.h"

namespace sepx {

enum : int {
  kEpiBf16 = 0,       // D -> bf16 [rows, ldo]
  kEpiSwigluFwd = 1,  // D = [gate | up] -> h = silu(g) * u (out), pre-activation gu (aux)
  kEpiSwigluBwd = 2,  // D = dh (unweighted) -> dgu (out), w*h (aux2), dw += <dh, h> (row_dw)
  kEpiF32 = 3,        // D -> fp32 [G, M, ldo] (weight gradients)
  kEpiAdamW = 4,      // D = weight gradient -> AdamW update of W[G, M, N] in place (fp32 state)
  kEpiAdamW8 = 5,     // same, 8-bit state, with the state streamed through a TMA ring
  kEpiRouter = 6,     // D = router logits [T, 128] -> softmax, top-k, routing tables (RouterEpi)
};

// kEpiRouter: the MoE router's softmax / top-k / renormalisation (and, with e2r / e2l, the
// expert-parallel routing tables) applied to each logit row straight from TMEM. Logits are
// rounded to bf16 first, as a bf16 projection followed by the standalone router would.
struct RouterEpi {
  const float* logit_bias = nullptr;  // [E] added to the logits (optional)
  const float* sel_bias = nullptr;    // [E] added to the probabilities for the selection only (optional)
  float* probs = nullptr;             // [T, E] softmax, kept for the backward
  int* topk_e = nullptr;              // [T, k]
  float* topk_w = nullptr;            // [T, k]
  const int* e2r = nullptr;           // [E] expert -> rank, and local slot (optional, together)
  const int* e2l = nullptr;
  int* dst = nullptr;                 // [T, k] destination rank / local slot per choice (with e2r)
  int* meta = nullptr;
  int k = 0;
  int renorm = 1;
};

struct GemmParams {
  const int* group_off = nullptr;  // [G+1] device offsets of the ragged dimension
  int G = 1;
  int M = 0;                 // ragged-K: output rows per group
  int N = 0;                 // output columns
  int K = 0;                 // ragged-M: reduction length
  int b_rows_per_group = 0;  // rows of B's 2-D view that belong to one group
  int n_tiles = 0;           // set by the launcher
  int I = 0;                 // SwiGLU intermediate size (gate and up halves)
  void* out = nullptr;
  int64_t ldo = 0;
  void* aux = nullptr;
  int64_t ld_aux = 0;
  void* aux2 = nullptr;
  int64_t ld_aux2 = 0;
  const float* row_w = nullptr;
  float* row_dw = nullptr;
  int* status = nullptr;
  unsigned long long timeout_ns = 2000000000ull;
  OptHyper opt;  // kEpiAdamW
  RouterEpi router;  // kEpiRouter
};

struct GemmCall {
  GemmParams p;
  int epi = kEpiBf16;
  const void* A = nullptr;
  int64_t a_rows = 0;
  int64_t lda = 0;
  const void* B = nullptr;
  int64_t b_rows = 0;
  int64_t ldb = 0;
  bool b_kmajor = true;
};

void grouped_gemm_ragged_m(const GemmCall& c, cudaStream_t stream);
void grouped_gemm_ragged_k(const GemmCall& c, cudaStream_t stream);
// weight gradient with the AdamW update fused into the epilogue (c.p.opt describes W)
void grouped_gemm_wgrad_adamw(const GemmCall& c, cudaStream_t stream);
// Whether 256-column tiles run on CTA pairs (tcgen05.mma.cta_group::2); returns the
// previous setting.
bool gemm_set_pairs(bool on);

}  // namespace sepx
